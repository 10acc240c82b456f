// CPU oracle for the chunked gated delta rule.
//
// TEST INFRASTRUCTURE ONLY. This file is the checker that the CUDA path is
// compared against; it is never linked into libspock_b200.so and the product
// path never calls it. Only tests/, __graft_entry__.smoke() and bench.py's
// CPU-baseline leg load liboracle.so.
//
// It restates spock's run_deltanet_chunk_rule
// (src/runtime/deltanet_chunk.cpp:53-284) step by step, in the same floating
// point operation order, so that it agrees bit for bit with the reference
// compiled by oracle/Makefile into oracle/_ref (tests assert that):
//   * optional per-token L2 norm, eps 1e-6 inside the sqrt   (deltanet_chunk.cpp:27-39, 78-85)
//   * q scaled by 1/sqrt(k_dim)                             (:87-88)
//   * zero padding to a multiple of chunk_size              (:90-113)
//   * per head, per chunk: cumulative g, decay matrix,
//     strictly lower -(beta k_i.k_j) decay, row-wise forward
//     substitution, +I, A.(v beta), A.(k beta e^g), q k^T decay,
//     v_prime / v_new / attn_inter, output, state update      (:134-270)
//   * un-padding of the output                              (:272-283)
// Heads are independent in the reference, so they are spread over threads
// here; each head's arithmetic is unchanged, so results do not depend on the
// thread count.
#include <algorithm>
#include <cmath>
#include <cstddef>
#include <cstring>
#include <thread>
#include <vector>

#include "oracle.h"

namespace {

struct Dims {
  size_t heads, seq, kd, vd, chunk, total;
};

void run_head(const Dims& d, size_t head, std::vector<float>& q, std::vector<float>& k,
              const float* v_in, const float* g_in, const float* b_in, float* out,
              float* state /* [kd][vd] for this head */) {
  const size_t seq = d.seq, kd = d.kd, vd = d.vd, C = d.chunk, total = d.total;
  // Padded per-head copies (reference :90-113), zero-filled beyond seq.
  std::vector<float> qp(total * kd, 0.f), kp(total * kd, 0.f), vp(total * vd, 0.f);
  std::vector<float> gp(total, 0.f), bp(total, 0.f);
  for (size_t t = 0; t < seq; ++t) {
    for (size_t x = 0; x < kd; ++x) {
      qp[t * kd + x] = q[(head * seq + t) * kd + x];
      kp[t * kd + x] = k[(head * seq + t) * kd + x];
    }
    for (size_t x = 0; x < vd; ++x) vp[t * vd + x] = v_in[(head * seq + t) * vd + x];
    gp[t] = g_in[head * seq + t];
    bp[t] = b_in[head * seq + t];
  }
  std::vector<float> decay(C * C), attn(C * C), solved(C * vd), kcum(C * kd);
  std::vector<float> qc(C * kd), kc(C * kd), vc(C * vd), gcum(C), bc(C);
  std::vector<float> local(C * C), vnew(C * vd), inter(C * vd), wstate(kd * vd), upd(kd * vd);
  std::vector<float> old_row(C);
  std::vector<float> outp(total * vd, 0.f);

  for (size_t c0 = 0; c0 < total; c0 += C) {
    float run = 0.f;
    for (size_t t = 0; t < C; ++t) {
      gcum[t] = run + gp[c0 + t];
      run = gcum[t];
      bc[t] = bp[c0 + t];
      std::memcpy(&qc[t * kd], &qp[(c0 + t) * kd], kd * sizeof(float));
      std::memcpy(&kc[t * kd], &kp[(c0 + t) * kd], kd * sizeof(float));
      std::memcpy(&vc[t * vd], &vp[(c0 + t) * vd], vd * sizeof(float));
    }
    std::fill(decay.begin(), decay.end(), 0.f);
    std::fill(attn.begin(), attn.end(), 0.f);
    for (size_t r = 0; r < C; ++r)
      for (size_t c = 0; c <= r; ++c) decay[r * C + c] = std::exp(gcum[r] - gcum[c]);
    // strictly lower -(beta_r k_r . k_c) * decay
    for (size_t r = 0; r < C; ++r)
      for (size_t c = 0; c < r; ++c) {
        float dot = 0.f;
        for (size_t x = 0; x < kd; ++x) dot += (kc[r * kd + x] * bc[r]) * kc[c * kd + x];
        attn[r * C + c] = -dot * decay[r * C + c];
      }
    // row-wise forward substitution, then +I
    for (size_t r = 1; r < C; ++r) {
      for (size_t c = 0; c < r; ++c) old_row[c] = attn[r * C + c];
      for (size_t c = 0; c < r; ++c) {
        float s = old_row[c];
        for (size_t m = 0; m < r; ++m) s += old_row[m] * attn[m * C + c];
        attn[r * C + c] = s;
      }
    }
    for (size_t x = 0; x < C; ++x) attn[x * C + x] += 1.f;
    // A.(v beta) and A.(k beta e^gcum), skipping zero coefficients
    std::fill(solved.begin(), solved.end(), 0.f);
    std::fill(kcum.begin(), kcum.end(), 0.f);
    for (size_t r = 0; r < C; ++r)
      for (size_t c = 0; c < C; ++c) {
        const float coeff = attn[r * C + c];
        if (coeff == 0.f) continue;
        const float bcol = bc[c];
        const float egc = std::exp(gcum[c]);
        for (size_t x = 0; x < vd; ++x) solved[r * vd + x] += coeff * (vc[c * vd + x] * bcol);
        for (size_t x = 0; x < kd; ++x) kcum[r * kd + x] += coeff * (kc[c * kd + x] * bcol * egc);
      }
    // q k^T decay, lower triangle including the diagonal
    std::fill(local.begin(), local.end(), 0.f);
    for (size_t r = 0; r < C; ++r)
      for (size_t c = 0; c <= r; ++c) {
        float dot = 0.f;
        for (size_t x = 0; x < kd; ++x) dot += qc[r * kd + x] * kc[c * kd + x];
        local[r * C + c] = dot * decay[r * C + c];
      }
    // v_prime, v_new, attn_inter against the running state
    for (size_t r = 0; r < C; ++r) {
      const float eg = std::exp(gcum[r]);
      for (size_t y = 0; y < vd; ++y) {
        float carry = 0.f, in = 0.f;
        for (size_t x = 0; x < kd; ++x) {
          carry += kcum[r * kd + x] * state[x * vd + y];
          in += (qc[r * kd + x] * eg) * state[x * vd + y];
        }
        vnew[r * vd + y] = solved[r * vd + y] - carry;
        inter[r * vd + y] = in;
      }
    }
    for (size_t r = 0; r < C; ++r)
      for (size_t y = 0; y < vd; ++y) {
        float s = inter[r * vd + y];
        for (size_t c = 0; c <= r; ++c) s += local[r * C + c] * vnew[c * vd + y];
        outp[(c0 + r) * vd + y] = s;
      }
    // state = state e^{gcum_last} + sum_r (k_r e^{gcum_last - gcum_r}) (x) v_new_r
    const float egl = std::exp(gcum[C - 1]);
    for (size_t x = 0; x < kd; ++x)
      for (size_t y = 0; y < vd; ++y) wstate[x * vd + y] = state[x * vd + y] * egl;
    std::fill(upd.begin(), upd.end(), 0.f);
    for (size_t r = 0; r < C; ++r) {
      const float w = std::exp(gcum[C - 1] - gcum[r]);
      for (size_t x = 0; x < kd; ++x) {
        const float sk = kc[r * kd + x] * w;
        for (size_t y = 0; y < vd; ++y) upd[x * vd + y] += sk * vnew[r * vd + y];
      }
    }
    for (size_t x = 0; x < kd * vd; ++x) state[x] = wstate[x] + upd[x];
  }
  for (size_t t = 0; t < seq; ++t)
    std::memcpy(&out[(head * seq + t) * vd], &outp[t * vd], vd * sizeof(float));
}

void l2_norm_token(std::vector<float>& a, size_t base, size_t width) {
  const float eps = 1e-6f;
  float ss = 0.f;
  for (size_t x = 0; x < width; ++x) ss += a[base + x] * a[base + x];
  const float inv = 1.0f / std::sqrt(ss + eps);
  for (size_t x = 0; x < width; ++x) a[base + x] *= inv;
}

}  // namespace

extern "C" int oracle_chunk_rule(int64_t num_heads, int64_t seq_len, int64_t key_dim,
                                 int64_t value_dim, int64_t chunk_size, int use_qk_l2norm,
                                 const float* query, const float* key, const float* value,
                                 const float* g, const float* beta, const float* initial_state,
                                 float* core_attn_out, float* final_state, int num_threads) {
  if (num_heads <= 0 || seq_len <= 0 || key_dim <= 0 || value_dim <= 0 || chunk_size <= 0)
    return -1;  // reference: "DeltaNet chunk config fields must be non-zero" (:55-58)
  Dims d;
  d.heads = (size_t)num_heads;
  d.seq = (size_t)seq_len;
  d.kd = (size_t)key_dim;
  d.vd = (size_t)value_dim;
  d.chunk = (size_t)chunk_size;
  d.total = d.seq + (d.chunk - d.seq % d.chunk) % d.chunk;
  std::vector<float> q(query, query + d.heads * d.seq * d.kd);
  std::vector<float> k(key, key + d.heads * d.seq * d.kd);
  if (use_qk_l2norm) {
    for (size_t h = 0; h < d.heads; ++h)
      for (size_t t = 0; t < d.seq; ++t) {
        l2_norm_token(q, (h * d.seq + t) * d.kd, d.kd);
        l2_norm_token(k, (h * d.seq + t) * d.kd, d.kd);
      }
  }
  const float q_scale = 1.0f / std::sqrt(static_cast<float>(d.kd));
  for (float& x : q) x *= q_scale;
  const size_t ss = d.kd * d.vd;
  if (initial_state)
    std::memcpy(final_state, initial_state, d.heads * ss * sizeof(float));
  else
    std::memset(final_state, 0, d.heads * ss * sizeof(float));
  int nt = std::max(1, std::min<int>(num_threads, (int)d.heads));
  auto worker = [&](int tid) {
    for (size_t h = (size_t)tid; h < d.heads; h += (size_t)nt)
      run_head(d, h, q, k, value, g, beta, core_attn_out, final_state + h * ss);
  };
  if (nt == 1) {
    worker(0);
  } else {
    std::vector<std::thread> th;
    for (int t = 0; t < nt; ++t) th.emplace_back(worker, t);
    for (auto& t : th) t.join();
  }
  return 0;
}
