// Minimal JSON reader for the CLIs (objects, arrays, numbers, strings, bools,
// null). Enough for the chunk-rule fixture format of spock-deltanet-chunk.
#pragma once
#include <cctype>
#include <cstdlib>
#include <fstream>
#include <map>
#include <memory>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

namespace jm {

struct Value {
  enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
  bool b = false;
  double num = 0;
  std::string str;
  std::vector<Value> arr;
  std::map<std::string, Value> obj;
  const Value* get(const std::string& k) const {
    auto it = obj.find(k);
    return it == obj.end() ? nullptr : &it->second;
  }
};

class Parser {
 public:
  explicit Parser(const std::string& s) : s_(s) {}
  Value parse() {
    Value v = value();
    ws();
    if (i_ != s_.size()) fail("trailing characters");
    return v;
  }

 private:
  const std::string& s_;
  size_t i_ = 0;
  [[noreturn]] void fail(const char* what) {
    throw std::runtime_error(std::string("json: ") + what + " at offset " + std::to_string(i_));
  }
  void ws() {
    while (i_ < s_.size() && std::isspace((unsigned char)s_[i_])) ++i_;
  }
  Value value() {
    ws();
    if (i_ >= s_.size()) fail("unexpected end");
    const char c = s_[i_];
    Value v;
    if (c == '{') {
      v.kind = Value::Object;
      ++i_;
      ws();
      if (s_[i_] == '}') {
        ++i_;
        return v;
      }
      while (true) {
        ws();
        Value k = value();
        if (k.kind != Value::String) fail("object key must be a string");
        ws();
        if (s_[i_++] != ':') fail("expected ':'");
        v.obj[k.str] = value();
        ws();
        if (s_[i_] == ',') {
          ++i_;
          continue;
        }
        if (s_[i_++] != '}') fail("expected '}'");
        return v;
      }
    }
    if (c == '[') {
      v.kind = Value::Array;
      ++i_;
      ws();
      if (s_[i_] == ']') {
        ++i_;
        return v;
      }
      while (true) {
        v.arr.push_back(value());
        ws();
        if (s_[i_] == ',') {
          ++i_;
          continue;
        }
        if (s_[i_++] != ']') fail("expected ']'");
        return v;
      }
    }
    if (c == '"') {
      v.kind = Value::String;
      ++i_;
      while (i_ < s_.size() && s_[i_] != '"') {
        if (s_[i_] == '\\') ++i_;
        v.str += s_[i_++];
      }
      ++i_;
      return v;
    }
    if (s_.compare(i_, 4, "true") == 0) {
      i_ += 4;
      v.kind = Value::Bool;
      v.b = true;
      return v;
    }
    if (s_.compare(i_, 5, "false") == 0) {
      i_ += 5;
      v.kind = Value::Bool;
      return v;
    }
    if (s_.compare(i_, 4, "null") == 0) {
      i_ += 4;
      return v;
    }
    char* end = nullptr;
    v.num = std::strtod(s_.c_str() + i_, &end);
    if (end == s_.c_str() + i_) fail("bad value");
    i_ = end - s_.c_str();
    v.kind = Value::Number;
    return v;
  }
};

inline Value read_file(const std::string& path) {
  std::ifstream f(path);
  if (!f) throw std::runtime_error("cannot open " + path);
  std::stringstream ss;
  ss << f.rdbuf();
  const std::string text = ss.str();
  return Parser(text).parse();
}

}  // namespace jm
