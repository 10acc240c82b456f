// spock-bench: the reference's benchmark CLI (apps/spock-bench.cpp:8-43), whose
// body there is a placeholder sleep loop (src/runtime/benchmark.cpp:41-58).
// Same flags: --mode pp520|tg128|correctness [--json|--csv] [--warmup N]
// [--runs N] [--output PATH], plus --config 0..4 [--gpus N] [--exact] for the
// five benchmark configurations on 1..N GPUs of one node. Every mode runs on
// the GPU with CUDA-event timing; the model modes use a seeded random-init
// Qwen3.5-0.8B-layout model:
//   pp520        520-token prompt through the layer-major prefill
//                (layer_major_prefill semantics, batched over the prompt): ms and tok/s
//   tg128        128 greedy decode tokens after an 8-token prompt
//   correctness  the same prompt decoded twice must give identical tokens,
//                and a chunk-rule call must produce finite outputs
#include <algorithm>
#include <cuda_bf16.h>
#include <functional>
#include <fstream>
#include <iostream>
#include <sstream>

#include "model_common.h"

namespace {

// ---- --config 0..4 [--gpus N]: BASELINE's configurations on the C ABI -------
// Seeded device-side inputs (a counter hash per element), CUDA-event timing,
// one host thread per GPU; sequences of configs 2 and 4 are split contiguously
// over the GPUs (strong scaling), configs 0, 1 and 3 run one replica per GPU.
__device__ __forceinline__ uint64_t dmix(uint64_t x) {
  x += 0x9e3779b97f4a7c15ull;
  x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
  x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
  return x ^ (x >> 31);
}
__device__ __forceinline__ float u01(uint64_t h) { return ((h >> 40) + 0.5f) * (1.0f / 16777216.0f); }
__device__ __forceinline__ float nrm(uint64_t h) {  // Box-Muller from two 24-bit uniforms
  return sqrtf(-2.0f * logf(u01(h))) * cospif(2.0f * u01(dmix(h)));
}
// rows x width values (width <= 256): kind 0 N(0,1) then L2-normalised per row, 1 N(0,1),
// 2 U(-1,-0.01), 3 U(0,1), 4 N(0, 0.02), 5 fp16 N(0,1) bits
template <typename T>
__global__ void fill_rows(T* out, int64_t rows, int width, int kind, uint64_t seed) {
  const int64_t r = (int64_t)blockIdx.x * blockDim.y + threadIdx.y;
  if (r >= rows) return;
  const int lane = threadIdx.x;  // 32 lanes per row
  float v[8];
  float ss = 0.f;
  const int per = (width + 31) / 32;
  for (int i = 0; i < per && i < 8; ++i) {
    const int c = lane * per + i;
    const uint64_t h = dmix(seed * 0x100000001b3ull + (uint64_t)r * width + c);
    float x = 0.f;
    if (c < width) {
      if (kind == 0 || kind == 1 || kind == 5) x = nrm(h);
      else if (kind == 2) x = -1.0f + 0.99f * u01(h);
      else if (kind == 3) x = u01(h);
      else x = 0.02f * nrm(h);
    }
    v[i] = x;
    ss += x * x;
  }
  if (kind == 0) {
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = 1.0f / sqrtf(ss + 1e-6f);
    for (int i = 0; i < per && i < 8; ++i) v[i] *= inv;
  }
  for (int i = 0; i < per && i < 8; ++i) {
    const int c = lane * per + i;
    if (c < width) out[r * width + c] = (T)v[i];
  }
}
template <typename T>
void fill(T* p, int64_t rows, int width, int kind, uint64_t seed) {
  fill_rows<T><<<(unsigned)((rows + 7) / 8), dim3(32, 8)>>>(p, rows, width, kind, seed);
}

struct CfgOut {
  double ms = 0;      // per step (max over GPUs)
  double work = 0;    // units per step over all GPUs
  std::string unit, what;
  bool ok = true;
  std::string err;
};

template <class F>
void on_gpus(int gpus, F f, std::vector<std::string>& errs) {
  std::vector<std::thread> th;
  errs.assign(gpus, "");
  for (int gi = 0; gi < gpus; ++gi)
    th.emplace_back([&, gi] {
      try {
        if (cudaSetDevice(gi) != cudaSuccess) throw std::runtime_error("cudaSetDevice failed");
        f(gi);
      } catch (const std::exception& e) {
        errs[gi] = e.what();
      }
    });
  for (auto& t : th) t.join();
}

double time_steps(cudaStream_t st, int warmup, int runs, const std::function<void()>& step) {
  for (int i = 0; i < warmup; ++i) step();
  cudaStreamSynchronize(st);
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  cudaEventRecord(e0, st);
  for (int i = 0; i < runs; ++i) step();
  cudaEventRecord(e1, st);
  cudaEventSynchronize(e1);
  float ms = 0;
  cudaEventElapsedTime(&ms, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  return ms / runs;
}

CfgOut run_config(int cfg, int gpus, int warmup, int runs, bool exact) {
  CfgOut o;
  std::vector<double> ms(gpus, 0);
  std::vector<std::string> errs;
  const int total_seqs = cfg == 2 ? 64 : (cfg == 4 ? 256 : 1);
  auto share = [&](int gi) {
    const int base = total_seqs / gpus, extra = total_seqs % gpus;
    return base + (gi < extra ? 1 : 0);
  };
  on_gpus(gpus, [&](int gi) {
    spock_ctx* ctx = nullptr;
    if (spock_create(gi, &ctx) != SPOCK_OK) throw std::runtime_error(spock_last_error(nullptr));
    cudaStream_t st;
    cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking);
    std::vector<void*> bufs;
    auto dalloc = [&](size_t bytes) {
      void* p = nullptr;
      if (cudaMalloc(&p, bytes) != cudaSuccess) throw std::runtime_error("cudaMalloc failed");
      bufs.push_back(p);
      return p;
    };
    auto check = [&](int rc) {
      if (rc != SPOCK_OK) throw std::runtime_error(spock_last_error(ctx));
    };
    if (cfg == 0 || cfg == 2) {
      const int64_t B = cfg == 0 ? 1 : share(gi), H = 16, S = cfg == 0 ? 104 : 8192;
      const int64_t rows = B * H * S;
      const int dt = cfg == 0 ? SPOCK_F32 : SPOCK_BF16;
      const size_t es = cfg == 0 ? 4 : 2;
      void *q = dalloc(rows * 128 * es), *k = dalloc(rows * 128 * es), *v = dalloc(rows * 128 * es);
      float *g = (float*)dalloc(rows * 4), *b = (float*)dalloc(rows * 4);
      void* out = dalloc(rows * 128 * es);
      float* fs = (float*)dalloc(B * H * 128 * 128 * 4);
      const uint64_t seed = 1000 + gi * 17;
      if (cfg == 0) {
        fill((float*)q, rows, 128, 0, seed);
        fill((float*)k, rows, 128, 0, seed + 1);
        fill((float*)v, rows, 128, 1, seed + 2);
      } else {
        fill((__nv_bfloat16*)q, rows, 128, 0, seed);
        fill((__nv_bfloat16*)k, rows, 128, 0, seed + 1);
        fill((__nv_bfloat16*)v, rows, 128, 1, seed + 2);
      }
      fill(g, rows, 1, 2, seed + 3);
      fill(b, rows, 1, 3, seed + 4);
      cudaDeviceSynchronize();
      spock_chunk_desc d{B, H, S, 128, 128, 64, dt, dt, 0, 0};
      ms[gi] = time_steps(st, warmup, runs, [&] { check(spock_chunk_prefill(ctx, &d, q, k, v, g, b, nullptr, out, fs, st)); });
      check(spock_sync(ctx, st));
    } else if (cfg == 1) {
      const int B = 64, layers = 18;
      const size_t conv = 6144;
      uint16_t* cw = (uint16_t*)dalloc(conv * 4 * 2);
      float* alb = (float*)dalloc(16 * 2 * 4);
      float* nw = (float*)dalloc(128 * 4);
      fill((__half*)cw, conv, 4, 4, 7);
      std::vector<float> h_alb(32), h_nw(128, 1.0f);
      for (int i = 0; i < 16; ++i) {
        h_alb[2 * i] = -2.0f + 3.0f * (float)(app::mix(i) % 1000) / 1000.0f;
        h_alb[2 * i + 1] = 0.1f * ((float)(app::mix(i + 99) % 2001) - 1000.0f) / 1000.0f;
      }
      cudaMemcpy(alb, h_alb.data(), 32 * 4, cudaMemcpyHostToDevice);
      cudaMemcpy(nw, h_nw.data(), 128 * 4, cudaMemcpyHostToDevice);
      spock_dn_layer L{16, 128, 128, 4, cw, alb, nw, 1e-6f, 0};
      std::vector<void*> qkv(layers), cs(layers), stt(layers);
      for (int l = 0; l < layers; ++l) {
        qkv[l] = dalloc(B * conv * 2);
        cs[l] = dalloc(B * conv * 4 * 2);
        stt[l] = dalloc((size_t)B * 16 * 128 * 128 * 4);
        fill((__half*)qkv[l], (int64_t)B * conv / 128, 128, 5, 100 + l);
        fill((__half*)cs[l], B * conv, 4, 5, 200 + l);
        fill((float*)stt[l], (int64_t)B * 16 * 128, 128, 4, 300 + l);
      }
      void *a = dalloc(B * 16 * 2), *bb = dalloc(B * 16 * 2), *z = dalloc(B * 2048 * 2), *out = dalloc(B * 2048 * 2);
      fill((__half*)a, B, 16, 5, 11);
      fill((__half*)bb, B, 16, 5, 12);
      fill((__half*)z, (int64_t)B * 2048 / 128, 128, 5, 13);
      cudaDeviceSynchronize();
      ms[gi] = time_steps(st, warmup, runs, [&] {
        for (int l = 0; l < layers; ++l)
          check(spock_deltanet_decode_step(ctx, &L, B, qkv[l], cs[l], (float*)stt[l], a, bb, z, out, nullptr, st));
      });
      check(spock_sync(ctx, st));
    } else {  // 3, 4: the random-init model
      const int B = cfg == 3 ? 1 : share(gi), P = 512, N = cfg == 4 ? 128 : 1;
      spock_model* m = nullptr;
      spock_model_desc d{24, 248320, B, P + N + 8, 1e-6f, 1e7f, exact ? 1 : 0, 0};
      if (spock_model_create(ctx, &d, &m) != SPOCK_OK) throw std::runtime_error("spock_model_create failed");
      app::random_init(m, 24, 248320, 1);
      int32_t* dp = (int32_t*)dalloc((size_t)B * P * 4);
      int32_t* dout = (int32_t*)dalloc((size_t)B * N * 4);
      std::vector<int32_t> prompt((size_t)B * P);
      for (size_t i = 0; i < prompt.size(); ++i) prompt[i] = (int32_t)(app::mix(i + 77 + gi * 1000003ull) % 248320);
      cudaMemcpy(dp, prompt.data(), prompt.size() * 4, cudaMemcpyHostToDevice);
      auto gen = [&] {
        if (spock_model_reset(m, B) != SPOCK_OK || spock_model_generate(m, dp, P, N, dout, st) != SPOCK_OK)
          throw std::runtime_error(spock_model_last_error(m));
      };
      ms[gi] = time_steps(st, warmup, runs, gen);
      if (spock_model_sync(m, st) != SPOCK_OK) throw std::runtime_error(spock_model_last_error(m));
      spock_model_destroy(m);
    }
    for (void* p : bufs) cudaFree(p);
    cudaStreamDestroy(st);
    spock_destroy(ctx);
  }, errs);
  for (int gi = 0; gi < gpus; ++gi)
    if (!errs[gi].empty()) {
      o.ok = false;
      o.err = "gpu " + std::to_string(gi) + ": " + errs[gi];
    }
  o.ms = *std::max_element(ms.begin(), ms.end());
  switch (cfg) {
    case 0: o.work = 1; o.unit = "calls/s"; o.what = "chunk rule H16 S104 fp32, one call per GPU (replicas)"; break;
    case 1: o.work = 64.0 * 18 * gpus; o.unit = "sequence-layer steps/s"; o.what = "fused decode step, batch 64, 18 layers per GPU (replicas)"; break;
    case 2: o.work = 64.0 * 8192; o.unit = "tok/s"; o.what = "chunk prefill, 64 x 16 heads x 8192 bf16, sequences split over GPUs"; break;
    case 3: o.work = 512.0 * gpus; o.unit = "tok/s"; o.what = "layer-major prefill of a 512-token prompt (+1 token), one per GPU"; break;
    default: o.work = 256.0 * (512 + 128 - 1); o.unit = "tok/s"; o.what = "512-token prompt + 128 greedy tokens, 256 sequences split over GPUs (prefill included)"; break;
  }
  if (cfg == 0) o.work = gpus;
  return o;
}

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
  bool csv = false, exact = false;
  int warmup = 1, runs = 3, layers = 24, vocab = 248320, config = -1, gpus = 1;
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
    else if (a == "--config" && i + 1 < argc) config = std::stoi(argv[++i]);
    else if (a == "--gpus" && i + 1 < argc) gpus = std::stoi(argv[++i]);
    else if (a == "--exact") exact = true;
    else if (a == "--help") {
      std::cout << "usage: spock-bench --mode pp520|tg128|correctness [--json|--csv] [--warmup N] [--runs N] [--output PATH]\n"
                   "       spock-bench --config 0|1|2|3|4 [--gpus N] [--exact] [--warmup N] [--runs N] [--json|--csv]\n";
      return 0;
    }
  }
  if (config >= 0) {
    int ndev = 0;
    cudaGetDeviceCount(&ndev);
    if (config > 4 || gpus < 1 || gpus > ndev) {
      std::cerr << "spock-bench: --config 0..4 and 1 <= --gpus <= " << ndev << "\n";
      return 2;
    }
    CfgOut o = run_config(config, gpus, warmup, runs, exact);
    if (!o.ok) {
      std::cerr << "spock-bench: " << o.err << "\n";
      return 1;
    }
    const double rate = o.work / (o.ms / 1e3);
    std::ostringstream os;
    if (csv)
      os << "config,gpus,runs,ms_per_step,rate,unit\n"
         << config << "," << gpus << "," << runs << "," << o.ms << "," << rate << "," << o.unit << "\n";
    else
      os << "{\"config\": " << config << ", \"gpus\": " << gpus << ", \"runs\": " << runs << ", \"ms_per_step\": "
         << o.ms << ", \"rate\": " << rate << ", \"unit\": \"" << o.unit << "\", \"timer\": \"cuda-events, max over GPUs\", "
         << "\"workload\": \"" << o.what << "\"" << (exact ? ", \"path\": \"exact\"" : "") << "}\n";
    if (!output.empty()) std::ofstream(output) << os.str();
    std::cout << os.str();
    return 0;
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
