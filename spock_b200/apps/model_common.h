// Shared by spock-decode and spock-bench: a random-init Qwen3.5-0.8B-layout
// model (no checkpoint is loaded: weights ~ N(0, 0.02), (1+w) norm weights
// ~ N(0, 0.1), A_log ~ U(-2, 1), dt_bias ~ N(0, 0.1), gated-norm weight
// 1 + N(0, 0.1)), uploaded through spock_model_set_weight by role name.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "../../include/spock_b200.h"

namespace app {

// splitmix64 stream per (seed, tensor, block) so threads generate independently
inline uint64_t mix(uint64_t x) {
  x += 0x9e3779b97f4a7c15ull;
  x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
  x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
  return x ^ (x >> 31);
}

inline void fill_normal_f16(std::vector<uint16_t>& out, size_t n, float sd, uint64_t seed) {
  out.resize(n);
  const int T = std::max(1u, std::thread::hardware_concurrency());
  std::vector<std::thread> th;
  for (int t = 0; t < T; ++t)
    th.emplace_back([&, t] {
      for (size_t i = (size_t)t * 2; i < n; i += (size_t)T * 2) {
        const uint64_t r = mix(seed * 0x100000001b3ull + i);
        const double u1 = ((r >> 11) + 1.0) * (1.0 / 9007199254740993.0);
        const double u2 = (mix(r) >> 11) * (1.0 / 9007199254740992.0);
        const double rad = std::sqrt(-2.0 * std::log(u1));
        const __half a = __float2half((float)(rad * std::cos(6.283185307179586 * u2)) * sd);
        const __half b = __float2half((float)(rad * std::sin(6.283185307179586 * u2)) * sd);
        out[i] = *reinterpret_cast<const uint16_t*>(&a);
        if (i + 1 < n) out[i + 1] = *reinterpret_cast<const uint16_t*>(&b);
      }
    });
  for (auto& x : th) x.join();
}

inline void set(spock_model* m, const std::string& role, const void* p, size_t bytes) {
  if (spock_model_set_weight(m, role.c_str(), p, bytes) != SPOCK_OK)
    throw std::runtime_error(std::string("set_weight ") + role + ": " + spock_model_last_error(m));
}

inline void random_init(spock_model* m, int layers, int vocab, uint64_t seed) {
  std::vector<uint16_t> buf;
  uint64_t tag = seed * 1000003ull;
  auto mat = [&](const std::string& role, size_t o, size_t i, float sd) {
    fill_normal_f16(buf, o * i, sd, ++tag);
    set(m, role, buf.data(), buf.size() * 2);
  };
  mat("embedding", vocab, 1024, 0.02f);
  mat("final_norm", 1024, 1, 0.1f);
  for (int l = 0; l < layers; ++l) {
    const std::string p = "layer." + std::to_string(l) + ".";
    mat(p + "input_norm", 1024, 1, 0.1f);
    mat(p + "post_norm", 1024, 1, 0.1f);
    mat(p + "mlp_gate", 3584, 1024, 0.02f);
    mat(p + "mlp_up", 3584, 1024, 0.02f);
    mat(p + "mlp_down", 1024, 3584, 0.02f);
    if (l % 4 == 3) {
      mat(p + "attn_q", 4096, 1024, 0.02f);
      mat(p + "attn_k", 512, 1024, 0.02f);
      mat(p + "attn_v", 512, 1024, 0.02f);
      mat(p + "attn_q_norm", 256, 1, 0.1f);
      mat(p + "attn_k_norm", 256, 1, 0.1f);
      mat(p + "attn_o", 1024, 2048, 0.02f);
    } else {
      mat(p + "delta_in_proj_qkv", 6144, 1024, 0.02f);
      mat(p + "delta_in_proj_z", 2048, 1024, 0.02f);
      mat(p + "delta_in_proj_a", 16, 1024, 0.02f);
      mat(p + "delta_in_proj_b", 16, 1024, 0.02f);
      mat(p + "delta_conv", 6144, 4, 0.02f);
      mat(p + "delta_dt_bias", 16, 1, 0.1f);
      std::vector<float> f(128);
      for (int i = 0; i < 128; ++i) f[i] = 1.0f + 0.1f * (float)((int)(mix(++tag) % 2001) - 1000) / 577.0f;
      set(m, p + "delta_norm", f.data(), 128 * 4);
      std::vector<float> al(16);
      for (int i = 0; i < 16; ++i) al[i] = -2.0f + 3.0f * (float)(mix(++tag) % 1000001) / 1000000.0f;
      set(m, p + "delta_a_log", al.data(), 16 * 4);
    }
  }
}

}  // namespace app
