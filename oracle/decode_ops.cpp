// CPU oracle for the fused single-token DeltaNet decode step.
//
// TEST INFRASTRUCTURE ONLY (never linked into the product library).
// The reference has no CPU decode (src/reference/qwen35_cpu_reference.cpp:14-25
// is a placeholder), so this restates its GLSL shaders directly:
//   oracle_conv_l2_qk   <- shaders/deltanet_conv_l2_qk.comp:48-110
//   oracle_rec_norm_gate <- shaders/deltanet_recurrent_gbeta_norm_gate.comp:91-224
//   oracle_recurrent_raw <- shaders/deltanet_recurrent.comp:55-125 (g/beta read
//                           from the state tail, raw output, no norm-gate)
// fp16 storage points are reproduced exactly (conv output stored as fp16
// before the L2 pass, w*norm rounded to fp16 before the SiLU gate, fp16
// outputs). Reductions follow the shaders' orders: sequential over k for the
// mat-vecs, a stride-64..1 pairwise tree for the 128-wide sums of squares.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

#include "half.h"
#include "oracle.h"

using oracle::f2h;
using oracle::h2f;

namespace {

float tree_sum128(float* s) {  // shaders' shared-memory tree, strides 64..1
  for (int stride = 64; stride > 0; stride >>= 1)
    for (int i = 0; i < stride; ++i) s[i] += s[i + stride];
  return s[0];
}

void conv_l2_one(int conv_dim, int ks, int key_total, int num_heads, uint16_t* qkv,
                 uint16_t* conv_state, const uint16_t* conv_w) {
  // Phase 1: shift and insert (deltanet_conv_l2_qk.comp:48-58)
  for (int ch = 0; ch < conv_dim; ++ch) {
    for (int i = 0; i < ks - 1; ++i) conv_state[ch * ks + i] = conv_state[ch * ks + i + 1];
    conv_state[ch * ks + ks - 1] = qkv[ch];
  }
  // Phase 2: depthwise conv + SiLU, stored as fp16 (:62-75)
  for (int ch = 0; ch < conv_dim; ++ch) {
    float sum = 0.f;
    for (int i = 0; i < ks; ++i) sum += h2f(conv_state[ch * ks + i]) * h2f(conv_w[ch * ks + i]);
    float silu = sum / (1.0f + oracle::exp_d(-sum));
    qkv[ch] = f2h(silu);
  }
  // Phase 3: L2 of the Q and K 128-blocks (:79-110)
  const int blocks = (conv_dim + 127) / 128;
  (void)key_total;
  for (int wg = 0; wg < blocks; ++wg) {
    bool is_q = wg < num_heads;
    bool is_k = !is_q && wg < 2 * num_heads;
    if (!(is_q || is_k)) continue;
    float s[128];
    for (int l = 0; l < 128; ++l) {
      float v = h2f(qkv[wg * 128 + l]);
      s[l] = v * v;
    }
    float inv = 1.0f / std::sqrt(tree_sum128(s) + 1e-6f);
    for (int l = 0; l < 128; ++l) qkv[wg * 128 + l] = f2h(h2f(qkv[wg * 128 + l]) * inv);
  }
}

void rec_norm_gate_one(int H, int kd, int vd, float q_scale, float eps, const uint16_t* a,
                       const uint16_t* b, const float* a_log_bias /* [H][2] of this layer */,
                       const uint16_t* q, const uint16_t* k, const uint16_t* v, float* state,
                       const uint16_t* z, const float* norm_w, uint16_t* out) {
  for (int h = 0; h < H; ++h) {
    float* S = state + (size_t)h * kd * vd;
    const float a_val = h2f(a[h]), b_val = h2f(b[h]);
    const float a_log = a_log_bias[h * 2 + 0], dt_bias = a_log_bias[h * 2 + 1];
    const float sp = oracle::log_d(1.0f + oracle::exp_d(a_val + dt_bias));
    const float g = -oracle::exp_d(a_log) * sp;
    const float beta = 1.0f / (1.0f + oracle::exp_d(-b_val));
    std::vector<float> sq(kd), sk(kd), sv(vd), kv(vd), delta(vd), o(vd);
    for (int i = 0; i < kd; ++i) {
      sq[i] = h2f(q[h * kd + i]) * q_scale;
      sk[i] = h2f(k[h * kd + i]);
    }
    for (int j = 0; j < vd; ++j) sv[j] = h2f(v[h * vd + j]);
    const float eg = oracle::exp_d(g);
    for (int e = 0; e < kd * vd; ++e) S[e] *= eg;
    for (int j = 0; j < vd; ++j) {
      float s = 0.f;
      for (int i = 0; i < kd; ++i) s += S[i * vd + j] * sk[i];
      kv[j] = s;
    }
    for (int j = 0; j < vd; ++j) delta[j] = (sv[j] - kv[j]) * beta;
    for (int i = 0; i < kd; ++i)
      for (int j = 0; j < vd; ++j) S[i * vd + j] += sk[i] * delta[j];
    for (int j = 0; j < vd; ++j) {
      float s = 0.f;
      for (int i = 0; i < kd; ++i) s += S[i * vd + j] * sq[i];
      o[j] = s;
    }
    float t[128] = {0};
    for (int j = 0; j < vd && j < 128; ++j) t[j] = o[j] * o[j];
    const float nf = 1.0f / std::sqrt(tree_sum128(t) / (float)vd + eps);
    for (int j = 0; j < vd; ++j) {
      const float normed = o[j] * nf;
      const float zz = h2f(z[h * vd + j]);
      const float silu = zz / (1.0f + oracle::exp_d(-zz));
      const float weighted = h2f(f2h(norm_w[j] * normed));
      out[h * vd + j] = f2h(weighted * silu);
    }
  }
}

template <class F>
void parallel_for(int n, int threads, F f) {
  if (threads <= 1 || n <= 1) {
    for (int i = 0; i < n; ++i) f(i);
    return;
  }
  std::vector<std::thread> th;
  for (int t = 0; t < threads; ++t)
    th.emplace_back([&, t] {
      for (int i = t; i < n; i += threads) f(i);
    });
  for (auto& x : th) x.join();
}

}  // namespace

extern "C" int oracle_conv_l2_qk(int batch, int conv_dim, int kernel_size, int key_total,
                                 int num_heads, uint16_t* qkv, uint16_t* conv_state,
                                 const uint16_t* conv_w, int num_threads) {
  if (batch <= 0 || conv_dim <= 0 || kernel_size <= 0) return -1;
  parallel_for(batch, num_threads, [&](int s) {
    conv_l2_one(conv_dim, kernel_size, key_total, num_heads, qkv + (size_t)s * conv_dim,
                conv_state + (size_t)s * conv_dim * kernel_size, conv_w);
  });
  return 0;
}

extern "C" int oracle_rec_norm_gate(int batch, int num_heads, int k_dim, int v_dim,
                                    float q_scale, float eps, const uint16_t* a,
                                    const uint16_t* b, const float* a_log_bias,
                                    const uint16_t* qkv, float* state, const uint16_t* z,
                                    const float* norm_w, uint16_t* out, int num_threads) {
  if (batch <= 0 || num_heads <= 0 || k_dim <= 0 || v_dim <= 0 || v_dim > 128) return -1;
  const size_t conv_dim = (size_t)num_heads * (2 * k_dim + v_dim);
  parallel_for(batch, num_threads, [&](int s) {
    const uint16_t* x = qkv + s * conv_dim;
    rec_norm_gate_one(num_heads, k_dim, v_dim, q_scale, eps, a + s * num_heads,
                      b + s * num_heads, a_log_bias, x, x + num_heads * k_dim,
                      x + 2 * num_heads * k_dim, state + (size_t)s * num_heads * k_dim * v_dim,
                      z + (size_t)s * num_heads * v_dim, norm_w,
                      out + (size_t)s * num_heads * v_dim);
  });
  return 0;
}

// deltanet_recurrent.comp: g/beta come from the state tail
// [H*kd*vd floats][g H][beta H]; output is the raw S^T q in fp16.
extern "C" int oracle_recurrent_raw(int num_heads, int k_dim, int v_dim, float q_scale,
                                    const uint16_t* q, const uint16_t* k, const uint16_t* v,
                                    float* state_with_tail, uint16_t* out) {
  const size_t total = (size_t)num_heads * k_dim * v_dim;
  for (int h = 0; h < num_heads; ++h) {
    float* S = state_with_tail + (size_t)h * k_dim * v_dim;
    const float g = state_with_tail[total + h];
    const float beta = state_with_tail[total + num_heads + h];
    std::vector<float> sq(k_dim), sk(k_dim), sv(v_dim), delta(v_dim);
    for (int i = 0; i < k_dim; ++i) {
      sq[i] = h2f(q[h * k_dim + i]) * q_scale;
      sk[i] = h2f(k[h * k_dim + i]);
    }
    for (int j = 0; j < v_dim; ++j) sv[j] = h2f(v[h * v_dim + j]);
    const float eg = oracle::exp_d(g);
    for (int e = 0; e < k_dim * v_dim; ++e) S[e] *= eg;
    for (int j = 0; j < v_dim; ++j) {
      float s = 0.f;
      for (int i = 0; i < k_dim; ++i) s += S[i * v_dim + j] * sk[i];
      delta[j] = (sv[j] - s) * beta;
    }
    for (int i = 0; i < k_dim; ++i)
      for (int j = 0; j < v_dim; ++j) S[i * v_dim + j] += sk[i] * delta[j];
    for (int j = 0; j < v_dim; ++j) {
      float s = 0.f;
      for (int i = 0; i < k_dim; ++i) s += S[i * v_dim + j] * sq[i];
      out[h * v_dim + j] = f2h(s);
    }
  }
  return 0;
}

// silu_gate.comp:main: out = fp16(silu(g) * u), silu(g) = g / (1 + exp(-g)).
extern "C" void oracle_silu_gate(int64_t n, const uint16_t* gate, const uint16_t* up, uint16_t* out) {
  for (int64_t i = 0; i < n; ++i) {
    const float g = h2f(gate[i]);
    out[i] = f2h((g / (1.0f + oracle::exp_d(-g))) * h2f(up[i]));
  }
}

// residual_add.comp: out = fp16(a + b) (out may alias a).
extern "C" void oracle_residual_add(int64_t n, const uint16_t* a, const uint16_t* b, uint16_t* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = f2h(h2f(a[i]) + h2f(b[i]));
}

// deltanet_recurrent_gbeta_norm_gate.comp:101-115 (phase 1), per head:
// g = -exp(A_log) * log(1 + exp(a + dt_bias)), beta = 1 / (1 + exp(-b)).
extern "C" void oracle_gbeta(int H, const uint16_t* a, const uint16_t* b, const float* a_log_bias, float* g,
                             float* beta) {
  for (int h = 0; h < H; ++h) {
    const float sp = oracle::log_d(1.0f + oracle::exp_d(h2f(a[h]) + a_log_bias[2 * h + 1]));
    g[h] = -oracle::exp_d(a_log_bias[2 * h]) * sp;
    beta[h] = 1.0f / (1.0f + oracle::exp_d(-h2f(b[h])));
  }
}

extern "C" void oracle_f32_to_f16(const float* x, uint16_t* y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) y[i] = f2h(x[i]);
}
extern "C" void oracle_f16_to_f32(const uint16_t* x, float* y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) y[i] = h2f(x[i]);
}
