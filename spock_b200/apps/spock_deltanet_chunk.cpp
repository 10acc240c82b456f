// spock-deltanet-chunk: the reference CLI (apps/spock-deltanet-chunk.cpp:40-103)
// with the chunk rule run by libspock_b200 on the GPU. Same flags, same JSON
// input (num_heads, sequence_length, key_dim, value_dim, chunk_size,
// use_qk_l2norm, query, key, value, g, beta, optional initial_state) and
// output ({"core_attn_out": [...], "final_state": [...]}, 9 significant
// digits); exit 2 on usage errors, 1 on any failure.
#include <cuda_runtime.h>

#include <iomanip>
#include <iostream>
#include <string>
#include <vector>

#include "../../include/spock_b200.h"
#include "json_min.h"

namespace {
std::vector<float> floats(const jm::Value* v, const char* name) {
  if (!v || v->kind != jm::Value::Array) throw std::runtime_error(std::string("missing array field: ") + name);
  std::vector<float> r;
  r.reserve(v->arr.size());
  for (const auto& e : v->arr) {
    if (e.kind != jm::Value::Number) throw std::runtime_error(std::string("non-numeric value in field: ") + name);
    r.push_back((float)e.num);
  }
  return r;
}
int64_t integer(const jm::Value& root, const char* name, int64_t def, bool required) {
  const jm::Value* v = root.get(name);
  if (!v) {
    if (required) throw std::runtime_error(std::string("missing integer field: ") + name);
    return def;
  }
  if (v->kind != jm::Value::Number) throw std::runtime_error(std::string("field must be a number: ") + name);
  return (int64_t)v->num;
}
void print_array(const std::vector<float>& a) {
  std::cout << "[";
  for (size_t i = 0; i < a.size(); ++i) std::cout << (i ? ", " : "") << a[i];
  std::cout << "]";
}
struct Dev {
  void* p = nullptr;
  explicit Dev(size_t bytes) {
    if (bytes && cudaMalloc(&p, bytes) != cudaSuccess) throw std::runtime_error("cudaMalloc failed");
  }
  ~Dev() { cudaFree(p); }
};
}  // namespace

int main(int argc, char** argv) {
  std::string input;
  for (int i = 1; i < argc; ++i) {
    const std::string a = argv[i];
    if (a == "--input" && i + 1 < argc) {
      input = argv[++i];
    } else if (a == "--help") {
      std::cout << "usage: spock-deltanet-chunk --input FILE\n";
      return 0;
    }
  }
  if (input.empty()) {
    std::cerr << "spock-deltanet-chunk: --input is required\n";
    return 2;
  }
  spock_ctx* ctx = nullptr;
  try {
    const jm::Value root = jm::read_file(input);
    if (root.kind != jm::Value::Object) throw std::runtime_error("root JSON value must be an object");
    spock_chunk_desc d{};
    d.batch = 1;
    d.num_heads = integer(root, "num_heads", 0, true);
    d.seq_len = integer(root, "sequence_length", 0, true);
    d.key_dim = integer(root, "key_dim", 0, true);
    d.value_dim = integer(root, "value_dim", 0, true);
    d.chunk_size = integer(root, "chunk_size", 64, false);
    d.use_qk_l2norm = 1;
    if (const jm::Value* u = root.get("use_qk_l2norm")) {
      if (u->kind != jm::Value::Bool) throw std::runtime_error("use_qk_l2norm must be a boolean");
      d.use_qk_l2norm = u->b ? 1 : 0;
    }
    d.dtype_in = SPOCK_F32;
    d.dtype_out = SPOCK_F32;
    const auto q = floats(root.get("query"), "query"), k = floats(root.get("key"), "key"),
               v = floats(root.get("value"), "value"), g = floats(root.get("g"), "g"),
               b = floats(root.get("beta"), "beta");
    std::vector<float> init;
    if (const jm::Value* iv = root.get("initial_state"))
      if (iv->kind != jm::Value::Null) init = floats(iv, "initial_state");
    // the reference's size checks (deltanet_chunk.cpp:41-49)
    auto check = [](const std::vector<float>& x, int64_t n, const char* name) {
      if ((int64_t)x.size() != n)
        throw std::runtime_error(std::string(name) + " size mismatch: expected " + std::to_string(n) + ", got " +
                                 std::to_string(x.size()));
    };
    if (d.num_heads <= 0 || d.seq_len <= 0 || d.key_dim <= 0 || d.value_dim <= 0 || d.chunk_size <= 0)
      throw std::runtime_error("DeltaNet chunk config fields must be non-zero");
    const int64_t H = d.num_heads, S = d.seq_len, K = d.key_dim, V = d.value_dim;
    check(q, H * S * K, "query");
    check(k, H * S * K, "key");
    check(v, H * S * V, "value");
    check(g, H * S, "g");
    check(b, H * S, "beta");
    if (!init.empty()) check(init, H * K * V, "initial_state");
    if (spock_create(0, &ctx) != SPOCK_OK) throw std::runtime_error(spock_last_error(nullptr));
    Dev dq(q.size() * 4), dk(k.size() * 4), dv(v.size() * 4), dg(g.size() * 4), db(b.size() * 4),
        di(init.size() * 4), dout((size_t)H * S * V * 4), dst((size_t)H * K * V * 4);
    cudaMemcpy(dq.p, q.data(), q.size() * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(dk.p, k.data(), k.size() * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(dv.p, v.data(), v.size() * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(dg.p, g.data(), g.size() * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(db.p, b.data(), b.size() * 4, cudaMemcpyHostToDevice);
    if (!init.empty()) cudaMemcpy(di.p, init.data(), init.size() * 4, cudaMemcpyHostToDevice);
    int rc = spock_chunk_prefill(ctx, &d, dq.p, dk.p, dv.p, (const float*)dg.p, (const float*)db.p,
                                 init.empty() ? nullptr : (const float*)di.p, dout.p, (float*)dst.p, nullptr);
    if (rc == SPOCK_OK) rc = spock_sync(ctx, nullptr);
    if (rc != SPOCK_OK) throw std::runtime_error(spock_last_error(ctx));
    std::vector<float> out((size_t)H * S * V), st((size_t)H * K * V);
    cudaMemcpy(out.data(), dout.p, out.size() * 4, cudaMemcpyDeviceToHost);
    cudaMemcpy(st.data(), dst.p, st.size() * 4, cudaMemcpyDeviceToHost);
    std::cout << std::setprecision(9);
    std::cout << "{\n  \"core_attn_out\": ";
    print_array(out);
    std::cout << ",\n  \"final_state\": ";
    print_array(st);
    std::cout << "\n}\n";
  } catch (const std::exception& e) {
    std::cerr << "spock-deltanet-chunk: " << e.what() << "\n";
    if (ctx) spock_destroy(ctx);
    return 1;
  }
  spock_destroy(ctx);
  return 0;
}
