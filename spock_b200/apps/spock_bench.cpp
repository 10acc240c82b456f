// spock-bench: the reference's benchmark CLI (apps/spock-bench.cpp:8-43), whose
// body there is a placeholder sleep loop (src/runtime/benchmark.cpp:41-58).
// Same flags: --mode pp520|tg128|correctness [--json|--csv] [--warmup N]
// [--runs N] [--output PATH]. Here every mode runs on the GPU with CUDA-event
// timing over a seeded random-init Qwen3.5-0.8B-layout model:
//   pp520        520-token prompt through the layer-major prefill
//                (layer_major_prefill semantics, batched over the prompt): ms and tok/s
//   tg128        128 greedy decode tokens after an 8-token prompt
//   correctness  the same prompt decoded twice must give identical tokens,
//                and a chunk-rule call must produce finite outputs
#include <algorithm>
#include <fstream>
#include <iostream>
#include <sstream>

#include "model_common.h"

namespace {
struct Result {
  std::string mode;
  std::vector<double> ms;
  double tok = 0;
  bool ok = true;
  std::string note;
};

double median(std::vector<double> v) {
  std::sort(v.begin(), v.end());
  return v.empty() ? 0 : v[v.size() / 2];
}
}  // namespace

int main(int argc, char** argv) {
  std::string mode = "tg128", output;
  bool csv = false;
  int warmup = 1, runs = 3, layers = 24, vocab = 248320;
  for (int i = 1; i < argc; ++i) {
    const std::string a = argv[i];
    if (a == "--mode" && i + 1 < argc) mode = argv[++i];
    else if (a == "--json") csv = false;
    else if (a == "--csv") csv = true;
    else if (a == "--warmup" && i + 1 < argc) warmup = std::stoi(argv[++i]);
    else if (a == "--runs" && i + 1 < argc) runs = std::stoi(argv[++i]);
    else if (a == "--output" && i + 1 < argc) output = argv[++i];
    else if (a == "--layers" && i + 1 < argc) layers = std::stoi(argv[++i]);
    else if (a == "--vocab" && i + 1 < argc) vocab = std::stoi(argv[++i]);
    else if (a == "--help") {
      std::cout << "usage: spock-bench --mode pp520|tg128|correctness [--json|--csv] [--warmup N] [--runs N] [--output PATH]\n";
      return 0;
    }
  }
  if (mode != "pp520" && mode != "tg128" && mode != "correctness") {
    std::cerr << "spock-bench: unknown mode " << mode << "\n";
    return 2;
  }
  Result r;
  r.mode = mode;
  spock_ctx* ctx = nullptr;
  spock_model* m = nullptr;
  try {
    if (spock_create(0, &ctx) != SPOCK_OK) throw std::runtime_error(spock_last_error(nullptr));
    const int P = mode == "pp520" ? 520 : 8, N = mode == "tg128" ? 128 : (mode == "correctness" ? 16 : 1);
    spock_model_desc d{layers, vocab, 1, P + N + 8, 1e-6f, 1e7f};
    if (spock_model_create(ctx, &d, &m) != SPOCK_OK) throw std::runtime_error("spock_model_create failed");
    app::random_init(m, layers, vocab, 1);
    std::vector<int32_t> prompt(P);
    for (int i = 0; i < P; ++i) prompt[i] = (int32_t)(app::mix(i + 77) % (uint64_t)vocab);
    cudaStream_t st;
    cudaStreamCreate(&st);
    int32_t *dp, *dout;
    cudaMalloc(&dp, P * 4);
    cudaMalloc(&dout, N * 4);
    cudaMemcpy(dp, prompt.data(), P * 4, cudaMemcpyHostToDevice);
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    std::vector<int32_t> first;
    for (int it = 0; it < warmup + runs; ++it) {
      spock_model_reset(m, 1);
      cudaEventRecord(e0, st);
      if (spock_model_generate(m, dp, P, N, dout, st) != SPOCK_OK) throw std::runtime_error(spock_model_last_error(m));
      cudaEventRecord(e1, st);
      cudaStreamSynchronize(st);
      float ms = 0;
      cudaEventElapsedTime(&ms, e0, e1);
      std::vector<int32_t> toks(N);
      cudaMemcpy(toks.data(), dout, N * 4, cudaMemcpyDeviceToHost);
      if (it == 0) first = toks;
      else if (mode == "correctness" && toks != first) r.ok = false;
      if (it >= warmup) r.ms.push_back(ms);
    }
    r.tok = mode == "pp520" ? P : (mode == "tg128" ? P + N - 1 : P + N - 1);
    if (mode == "correctness") {
      // chunk rule: finite outputs on a seeded case
      const int H = 2, S = 70;
      std::vector<float> q(H * S * 128), k(H * S * 128), v(H * S * 128), g(H * S), b(H * S);
      for (size_t i = 0; i < q.size(); ++i) {
        q[i] = ((int)(app::mix(i) % 2001) - 1000) / 8000.0f;
        k[i] = ((int)(app::mix(i + 5000000) % 2001) - 1000) / 8000.0f;
        v[i] = ((int)(app::mix(i + 9000000) % 2001) - 1000) / 1000.0f;
      }
      for (int i = 0; i < H * S; ++i) {
        g[i] = -0.01f - 0.99f * (float)(app::mix(i + 1) % 1000) / 1000.0f;
        b[i] = (float)(app::mix(i + 2) % 1000) / 1000.0f;
      }
      float *dq, *dk, *dv, *dg, *db, *dO, *dS;
      cudaMalloc(&dq, q.size() * 4);
      cudaMalloc(&dk, k.size() * 4);
      cudaMalloc(&dv, v.size() * 4);
      cudaMalloc(&dg, g.size() * 4);
      cudaMalloc(&db, b.size() * 4);
      cudaMalloc(&dO, v.size() * 4);
      cudaMalloc(&dS, (size_t)H * 128 * 128 * 4);
      cudaMemcpy(dq, q.data(), q.size() * 4, cudaMemcpyHostToDevice);
      cudaMemcpy(dk, k.data(), k.size() * 4, cudaMemcpyHostToDevice);
      cudaMemcpy(dv, v.data(), v.size() * 4, cudaMemcpyHostToDevice);
      cudaMemcpy(dg, g.data(), g.size() * 4, cudaMemcpyHostToDevice);
      cudaMemcpy(db, b.data(), b.size() * 4, cudaMemcpyHostToDevice);
      spock_chunk_desc cd{1, H, S, 128, 128, 64, SPOCK_F32, SPOCK_F32, 1, 0};
      if (spock_chunk_prefill(ctx, &cd, dq, dk, dv, dg, db, nullptr, dO, dS, nullptr) != SPOCK_OK ||
          spock_sync(ctx, nullptr) != SPOCK_OK)
        throw std::runtime_error(spock_last_error(ctx));
      std::vector<float> o(v.size());
      cudaMemcpy(o.data(), dO, o.size() * 4, cudaMemcpyDeviceToHost);
      for (float x : o)
        if (!std::isfinite(x)) r.ok = false;
      for (float* p : {dq, dk, dv, dg, db, dO, dS}) cudaFree(p);
      r.note = "decode repeatable and chunk-rule outputs finite";
    }
    cudaFree(dp);
    cudaFree(dout);
    cudaStreamDestroy(st);
  } catch (const std::exception& e) {
    std::cerr << "spock-bench: " << e.what() << "\n";
    if (m) spock_model_destroy(m);
    if (ctx) spock_destroy(ctx);
    return 1;
  }
  spock_model_destroy(m);
  spock_destroy(ctx);
  const double med = median(r.ms);
  std::ostringstream os;
  if (csv) {
    os << "mode,runs,median_ms,tok_per_s,ok\n"
       << r.mode << "," << r.ms.size() << "," << med << "," << (med > 0 ? r.tok / (med / 1e3) : 0) << ","
       << (r.ok ? 1 : 0) << "\n";
  } else {
    os << "{\"mode\": \"" << r.mode << "\", \"runs\": " << r.ms.size() << ", \"median_ms\": " << med
       << ", \"tok_per_s\": " << (med > 0 ? r.tok / (med / 1e3) : 0) << ", \"timer\": \"cuda-events\", \"ok\": "
       << (r.ok ? "true" : "false") << ", \"weights\": \"random-init\"" << (r.note.empty() ? "" : ", \"note\": \"" + r.note + "\"")
       << "}\n";
  }
  if (!output.empty()) std::ofstream(output) << os.str();
  std::cout << os.str();
  return r.ok ? 0 : 1;
}
