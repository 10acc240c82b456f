// spock-decode: greedy decode CLI (the reference's apps/spock-decode.cpp:17-173)
// over libspock_b200's model session. Same flags where they apply (--tokens
// FILE, --max-new-tokens N, --verbose, --help) and the same JSON keys
// (prompt_tokens, generated_tokens, generated_count, elapsed_ms, prefill_ms,
// decode_ms). Weights come from a repacked text artifact (--repack-dir, the
// reference's text_repack_manifest.json + text_weights.bin) or, when none is
// given, from a seeded random init of the Qwen3.5-0.8B layout (--seed,
// --layers, --vocab).
#include <chrono>
#include <fstream>
#include <iostream>
#include <sstream>

#include "model_common.h"

int main(int argc, char** argv) {
  std::string token_file, repack_dir;
  int max_new = 16, layers = 24, vocab = 248320;
  uint64_t seed = 0;
  bool verbose = false;
  for (int i = 1; i < argc; ++i) {
    const std::string a = argv[i];
    if (a == "--tokens" && i + 1 < argc) token_file = argv[++i];
    else if (a == "--max-new-tokens" && i + 1 < argc) max_new = std::stoi(argv[++i]);
    else if (a == "--layers" && i + 1 < argc) layers = std::stoi(argv[++i]);
    else if (a == "--vocab" && i + 1 < argc) vocab = std::stoi(argv[++i]);
    else if (a == "--seed" && i + 1 < argc) seed = std::stoull(argv[++i]);
    else if (a == "--verbose" || a == "-v") verbose = true;
    else if (a == "--repack-dir" && i + 1 < argc) repack_dir = argv[++i];
    else if (a == "--help") {
      std::cout << "usage: spock-decode --tokens FILE [--max-new-tokens N] [--repack-dir DIR] [--layers N] [--vocab N] [--seed S]\n";
      return 0;
    }
  }
  std::vector<int32_t> prompt = {9419, 11, 1814, 0};  // the reference's default prompt ids
  if (!token_file.empty()) {
    std::ifstream f(token_file);
    if (!f) {
      std::cerr << "spock-decode: cannot open " << token_file << "\n";
      return 2;
    }
    prompt.clear();
    int32_t t;
    while (f >> t) prompt.push_back(t);
    if (prompt.empty()) {
      std::cerr << "spock-decode: token file is empty\n";
      return 2;
    }
  }
  spock_ctx* ctx = nullptr;
  spock_model* m = nullptr;
  try {
    const auto t0 = std::chrono::steady_clock::now();
    if (spock_create(0, &ctx) != SPOCK_OK) throw std::runtime_error(spock_last_error(nullptr));
    spock_model_desc d{layers, vocab, 1, (int32_t)(prompt.size() + max_new + 8), 1e-6f, 1e7f};
    if (spock_model_create(ctx, &d, &m) != SPOCK_OK) throw std::runtime_error("spock_model_create failed");
    if (!repack_dir.empty()) {
      if (spock_model_load_artifact(m, repack_dir.c_str()) != SPOCK_OK) throw std::runtime_error(spock_model_last_error(m));
    } else {
      app::random_init(m, layers, vocab, seed);
    }
    if (verbose) std::cerr << "spock-decode: weights uploaded\n";
    spock_model_reset(m, 1);
    cudaStream_t st;
    cudaStreamCreate(&st);
    int32_t *dp = nullptr, *dout = nullptr, *dtok = nullptr;
    cudaMalloc(&dp, prompt.size() * 4);
    cudaMalloc(&dout, (max_new + 1) * 4);
    cudaMalloc(&dtok, 4);
    cudaMemcpy(dp, prompt.data(), prompt.size() * 4, cudaMemcpyHostToDevice);
    cudaEvent_t e0, e1, e2;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaEventCreate(&e2);
    cudaEventRecord(e0, st);
    // prefill (token-serial) + the first generated token
    if (spock_model_generate(m, dp, (int32_t)prompt.size(), 1, dout, st) != SPOCK_OK)
      throw std::runtime_error(spock_model_last_error(m));
    cudaEventRecord(e1, st);
    cudaMemcpyAsync(dtok, dout, 4, cudaMemcpyDeviceToDevice, st);
    for (int i = 1; i < max_new; ++i) {
      if (spock_model_step(m, dtok, dtok, nullptr, st) != SPOCK_OK) throw std::runtime_error(spock_model_last_error(m));
      cudaMemcpyAsync(dout + i, dtok, 4, cudaMemcpyDeviceToDevice, st);
    }
    cudaEventRecord(e2, st);
    cudaStreamSynchronize(st);
    std::vector<int32_t> gen(max_new);
    if (max_new > 0) cudaMemcpy(gen.data(), dout, max_new * 4, cudaMemcpyDeviceToHost);
    float prefill_ms = 0, decode_ms = 0;
    cudaEventElapsedTime(&prefill_ms, e0, e1);
    cudaEventElapsedTime(&decode_ms, e1, e2);
    const double elapsed =
        std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    std::cout << "{\n  \"prompt_tokens\": [";
    for (size_t i = 0; i < prompt.size(); ++i) std::cout << (i ? ", " : "") << prompt[i];
    std::cout << "],\n  \"generated_tokens\": [";
    for (int i = 0; i < max_new; ++i) std::cout << (i ? ", " : "") << gen[i];
    std::cout << "],\n  \"generated_count\": " << max_new << ",\n  \"elapsed_ms\": " << elapsed
              << ",\n  \"prefill_ms\": " << prefill_ms << ",\n  \"decode_ms\": " << decode_ms
              << ",\n  \"weights\": \"" << (repack_dir.empty() ? "random-init (seed " + std::to_string(seed) + ")" : repack_dir)
              << "\"\n}\n";
    cudaFree(dp);
    cudaFree(dout);
    cudaFree(dtok);
    cudaStreamDestroy(st);
  } catch (const std::exception& e) {
    std::cout << "{\n  \"error\": \"" << e.what() << "\"\n}\n";
    if (m) spock_model_destroy(m);
    if (ctx) spock_destroy(ctx);
    return 1;
  }
  spock_model_destroy(m);
  spock_destroy(ctx);
  return 0;
}
