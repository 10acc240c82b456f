// CPU oracle for one full-model decode step of the Qwen3.5-0.8B layout.
//
// TEST INFRASTRUCTURE ONLY (never linked into the product library). The
// reference's CPU model is a placeholder (src/reference/qwen35_cpu_reference
// .cpp:14-25), so this restates the default decode path of DecodeSession
// (src/runtime/vk_session.cpp:2658-3370, 3516-3563) shader by shader:
//   rms_norm.comp:31-70        lane-local sums of 4 squares, stride-128..1 tree,
//                              x * (1/sqrt(mean+eps)) * (1+w) -> fp16
//   matvec.comp:28-41          sequential fp32 dot per row -> fp16
//   split_q_gate / rms_norm_per_head / rope_apply / kv_cache_store /
//   attention_decode.comp:64-143 / sigmoid_gate / residual_add / silu_gate
//   deltanet_conv_l2_qk + deltanet_recurrent_gbeta_norm_gate (decode_ops.cpp)
//   lm_head (tied embedding) -> fp16 logits, argmax.comp (lowest index on ties)
// The RoPE cos/sin table is built with the same host formula as the reference
// (vk_session.cpp:333-346). Weights are referenced, not copied.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <immintrin.h>

#include <algorithm>
#include <map>
#include <string>
#include <thread>
#include <vector>

#include "half.h"
#include "oracle.h"

using oracle::f2h;
using oracle::h2f;

namespace {
constexpr int HID = 1024, INTER = 3584, DNH = 16, DND = 128, CONV = 6144;
constexpr int QH = 8, KVH = 2, HD = 256, ROT = 64, ATT_IN = QH * HD * 2 + 2 * KVH * HD;

struct Seq {
  std::vector<float> dn_state;      // [n_dn][16][128][128]
  std::vector<uint16_t> conv;       // [n_dn][6144][4]
  std::vector<uint16_t> kv;         // [n_attn][max_seq][2][2][256]
  int pos = 0;
};

template <class F>
void par(int n, int threads, F f) {
  if (threads <= 1) {
    for (int i = 0; i < n; ++i) f(i);
    return;
  }
  std::vector<std::thread> th;
  for (int t = 0; t < threads; ++t)
    th.emplace_back([&, t] {
      const int lo = (int)((int64_t)n * t / threads), hi = (int)((int64_t)n * (t + 1) / threads);
      for (int i = lo; i < hi; ++i) f(i);
    });
  for (auto& x : th) x.join();
}

// Each row's dot is sequential over j (matvec.comp:28-41); 8 rows advance
// together only so the independent chains overlap in the CPU's pipeline.
// fp16 -> fp32 of every bit pattern (exact; the same values h2f returns).
const float* h2f_table() {
  static const std::vector<float> t = [] {
    std::vector<float> v(65536);
    for (int i = 0; i < 65536; ++i) v[i] = h2f((uint16_t)i);
    return v;
  }();
  return t.data();
}

// 8 rows x 8 columns of fp16 weights -> fp32, transposed (t[c] holds column c
// of the 8 rows) with AVX2/F16C; the conversions are exact.
__attribute__((target("avx2,f16c"))) inline void load8x8_t(const uint16_t* const* w, int j, __m256 t[8]) {
  __m256 r[8];
  for (int i = 0; i < 8; ++i) r[i] = _mm256_cvtph_ps(_mm_loadu_si128(reinterpret_cast<const __m128i*>(w[i] + j)));
  const __m256 a0 = _mm256_unpacklo_ps(r[0], r[1]), a1 = _mm256_unpackhi_ps(r[0], r[1]);
  const __m256 a2 = _mm256_unpacklo_ps(r[2], r[3]), a3 = _mm256_unpackhi_ps(r[2], r[3]);
  const __m256 a4 = _mm256_unpacklo_ps(r[4], r[5]), a5 = _mm256_unpackhi_ps(r[4], r[5]);
  const __m256 a6 = _mm256_unpacklo_ps(r[6], r[7]), a7 = _mm256_unpackhi_ps(r[6], r[7]);
  const __m256 b0 = _mm256_shuffle_ps(a0, a2, 0x44), b1 = _mm256_shuffle_ps(a0, a2, 0xEE);
  const __m256 b2 = _mm256_shuffle_ps(a1, a3, 0x44), b3 = _mm256_shuffle_ps(a1, a3, 0xEE);
  const __m256 b4 = _mm256_shuffle_ps(a4, a6, 0x44), b5 = _mm256_shuffle_ps(a4, a6, 0xEE);
  const __m256 b6 = _mm256_shuffle_ps(a5, a7, 0x44), b7 = _mm256_shuffle_ps(a5, a7, 0xEE);
  t[0] = _mm256_permute2f128_ps(b0, b4, 0x20);
  t[1] = _mm256_permute2f128_ps(b1, b5, 0x20);
  t[2] = _mm256_permute2f128_ps(b2, b6, 0x20);
  t[3] = _mm256_permute2f128_ps(b3, b7, 0x20);
  t[4] = _mm256_permute2f128_ps(b0, b4, 0x31);
  t[5] = _mm256_permute2f128_ps(b1, b5, 0x31);
  t[6] = _mm256_permute2f128_ps(b2, b6, 0x31);
  t[7] = _mm256_permute2f128_ps(b3, b7, 0x31);
}

// 8 rows' dots, each sequential over j with a separate multiply and add per
// term (lane i of the vectors is row i).
__attribute__((target("avx2,f16c"))) void dot8_rows(const uint16_t* const* w, const float* xf, int in, float* out8) {
  __m256 s = _mm256_setzero_ps();
  __m256 t[8];
  for (int j = 0; j < in; j += 8) {
    load8x8_t(w, j, t);
    for (int c = 0; c < 8; ++c) s = _mm256_add_ps(s, _mm256_mul_ps(t[c], _mm256_set1_ps(xf[j + c])));
  }
  _mm256_storeu_ps(out8, s);
}

void matvec(const uint16_t* W, const uint16_t* x, int out, int in, uint16_t* y, int threads) {
  const float* H = h2f_table();
  std::vector<float> xf(in);
  for (int j = 0; j < in; ++j) xf[j] = h2f(x[j]);
  constexpr int RB = 8;
  par((out + RB - 1) / RB, threads, [&](int blk) {
    const int r0 = blk * RB, nr = std::min(RB, out - r0);
    float s[RB] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    const uint16_t* w[RB];
    for (int i = 0; i < RB; ++i) w[i] = W + (size_t)(r0 + (i < nr ? i : 0)) * in;
    if (in % 8 == 0) {
      dot8_rows(w, xf.data(), in, s);
    } else {
      for (int j = 0; j < in; ++j)
        for (int i = 0; i < RB; ++i) s[i] += H[w[i][j]] * xf[j];
    }
    for (int i = 0; i < nr; ++i) y[r0 + i] = f2h(s[i]);
  });
}

void rmsnorm(const uint16_t* x, const uint16_t* w, float eps, uint16_t* y) {
  float s[256];
  for (int l = 0; l < 256; ++l) {
    float a = 0.f;
    for (int i = 0; i < 4; ++i) {
      const float v = h2f(x[l * 4 + i]);
      a += v * v;
    }
    s[l] = a;
  }
  for (int st = 128; st > 0; st >>= 1)
    for (int l = 0; l < st; ++l) s[l] += s[l + st];
  const float nf = 1.0f / std::sqrt(s[0] / (float)HID + eps);
  for (int i = 0; i < HID; ++i) y[i] = f2h(h2f(x[i]) * nf * (1.0f + h2f(w[i])));
}

void rmsnorm_head(const uint16_t* x, const uint16_t* w, float eps, uint16_t* y) {
  float s[256];
  for (int l = 0; l < 256; ++l) {
    const float v = h2f(x[l]);
    s[l] = v * v;
  }
  for (int st = 128; st > 0; st >>= 1)
    for (int l = 0; l < st; ++l) s[l] += s[l + st];
  const float nf = 1.0f / std::sqrt(s[0] / (float)HD + eps);
  for (int d = 0; d < HD; ++d) y[d] = f2h(h2f(x[d]) * nf * (1.0f + h2f(w[d])));
}

void rope(uint16_t* x, int heads, const float* cs /*[64] of this position*/) {
  for (int h = 0; h < heads; ++h) {
    uint16_t* b = x + h * HD;
    for (int i = 0; i < 32; ++i) {
      const float c = cs[2 * i], s = cs[2 * i + 1];
      const float v0 = h2f(b[i]), v1 = h2f(b[i + 32]);
      b[i] = f2h(v0 * c - v1 * s);
      b[i + 32] = f2h(v1 * c + v0 * s);
    }
  }
}
// One token of gated full attention for one sequence, from the projected row
// proj = [q0 | gate0 | ... | q7 | gate7 | k0 k1 | v0 v1] (5120 fp16): the
// reference's split_q_gate, rms_norm_per_head (q, k), rope_apply (cs: this
// position's 32 (cos, sin) pairs), kv_cache_store (cache: [max_seq][K|V][2][256]
// of this layer, row `pos`), attention_decode.comp:64-143 over positions
// 0..pos (scale 1/16) and sigmoid_gate -> gated [8*256].
void attention_token(const uint16_t* proj, const uint16_t* qn_w, const uint16_t* kn_w, float eps, const float* cs,
                     uint16_t* cache, int pos, uint16_t* gated) {
  std::vector<uint16_t> q(QH * HD), gate(QH * HD), k(KVH * HD), att(QH * HD);
  for (int hh = 0; hh < QH; ++hh)
    for (int d = 0; d < HD; ++d) {
      q[hh * HD + d] = proj[hh * 2 * HD + d];
      gate[hh * HD + d] = proj[hh * 2 * HD + HD + d];
    }
  std::memcpy(k.data(), proj + QH * HD * 2, KVH * HD * 2);
  const uint16_t* v = proj + QH * HD * 2 + KVH * HD;
  for (int hh = 0; hh < QH; ++hh) rmsnorm_head(q.data() + hh * HD, qn_w, eps, q.data() + hh * HD);
  for (int hh = 0; hh < KVH; ++hh) rmsnorm_head(k.data() + hh * HD, kn_w, eps, k.data() + hh * HD);
  rope(q.data(), QH, cs);
  rope(k.data(), KVH, cs);
  std::memcpy(cache + (size_t)pos * 2 * KVH * HD, k.data(), KVH * HD * 2);
  std::memcpy(cache + (size_t)pos * 2 * KVH * HD + KVH * HD, v, KVH * HD * 2);
  const int L = pos + 1;
  const float scale = 1.0f / 16.0f;
  for (int hh = 0; hh < QH; ++hh) {
    const int kvh = hh / (QH / KVH);
    std::vector<float> sc(L);
    float mx = -1e30f;
    for (int p = 0; p < L; ++p) {
      float dot = 0.f;
      const uint16_t* kr = cache + (size_t)p * 2 * KVH * HD + kvh * HD;
      for (int d = 0; d < HD; ++d) dot += h2f(q[hh * HD + d]) * h2f(kr[d]);
      sc[p] = dot * scale;
      mx = std::max(mx, sc[p]);
    }
    float sum = 0.f;
    std::vector<float> acc(HD, 0.f);
    for (int p = 0; p < L; ++p) {
      const float w = oracle::exp_d(sc[p] - mx);
      sum += w;
      const uint16_t* vr = cache + (size_t)p * 2 * KVH * HD + KVH * HD + kvh * HD;
      for (int d = 0; d < HD; ++d) acc[d] += w * h2f(vr[d]);
    }
    const float inv = 1.0f / (sum + 1e-30f);
    for (int d = 0; d < HD; ++d) att[hh * HD + d] = f2h(acc[d] * inv);
  }
  for (int i = 0; i < QH * HD; ++i) {
    const float g = h2f(gate[i]);
    gated[i] = f2h(h2f(att[i]) * (1.0f / (1.0f + oracle::exp_d(-g))));
  }
}

// argmax.comp:27-62 over fp16 logits: the strictly greater value wins, so the
// lowest index wins among equal maxima.
int argmax16(const uint16_t* logits, int n, float* margin) {
  int best = 0;
  float bv = -3.402823466e+38f, second = -3.402823466e+38f;
  for (int i = 0; i < n; ++i) {
    const float v = h2f(logits[i]);
    if (v > bv) {
      second = bv;
      bv = v;
      best = i;
    } else if (v > second) {
      second = v;
    }
  }
  if (margin) *margin = bv - second;
  return best;
}
}  // namespace

struct oracle_model {
  int layers, vocab, max_seq;
  float eps, theta;
  std::map<std::string, const void*> w;
  std::vector<float> rope;  // [max_seq][64]
  std::vector<Seq> seqs;
  const uint16_t* W(const std::string& r) const {
    auto it = w.find(r);
    return it == w.end() ? nullptr : static_cast<const uint16_t*>(it->second);
  }
  const float* F(const std::string& r) const {
    auto it = w.find(r);
    return it == w.end() ? nullptr : static_cast<const float*>(it->second);
  }
};

extern "C" oracle_model* oracle_model_create(int layers, int vocab, int max_seq, float eps, float theta) {
  auto* m = new oracle_model();
  m->layers = layers;
  m->vocab = vocab;
  m->max_seq = max_seq;
  m->eps = eps;
  m->theta = theta;
  m->rope.resize((size_t)max_seq * ROT);
  for (int p = 0; p < max_seq; ++p)
    for (int i = 0; i < 32; ++i) {
      const float inv_freq = 1.0f / std::pow(theta, 2.0f * (float)i / (float)ROT);
      const float ang = (float)p * inv_freq;
      m->rope[(size_t)p * ROT + 2 * i] = std::cos(ang);
      m->rope[(size_t)p * ROT + 2 * i + 1] = std::sin(ang);
    }
  return m;
}

extern "C" void oracle_model_destroy(oracle_model* m) { delete m; }

extern "C" void oracle_model_set(oracle_model* m, const char* role, const void* ptr) { m->w[role] = ptr; }

extern "C" void oracle_model_reset(oracle_model* m, int batch) {
  const int ndn = m->layers - m->layers / 4, nat = m->layers / 4;
  m->seqs.assign(batch, Seq());
  for (auto& s : m->seqs) {
    s.dn_state.assign((size_t)ndn * DNH * DND * DND, 0.f);
    s.conv.assign((size_t)ndn * CONV * 4, 0);
    s.kv.assign((size_t)nat * m->max_seq * 2 * KVH * HD, 0);
    s.pos = 0;
  }
}

// tokens [batch] -> out_tokens [batch]; hidden_out (nullable) [batch][1024]
// final-normed hidden; margin (nullable) [batch] = top1 - top2 fp16 logit.
extern "C" int oracle_model_step(oracle_model* m, const int* tokens, int* out_tokens, uint16_t* hidden_out,
                                 float* margin, int threads) {
  const float eps = m->eps;
  const uint16_t* emb = m->W("embedding");
  for (size_t b = 0; b < m->seqs.size(); ++b) {
    Seq& sq = m->seqs[b];
    if (sq.pos >= m->max_seq) return -1;
    std::vector<uint16_t> h(emb + (size_t)tokens[b] * HID, emb + (size_t)(tokens[b] + 1) * HID);
    std::vector<uint16_t> x(HID), y(HID);
    int di = 0, ai = 0;
    for (int li = 0; li < m->layers; ++li) {
      const std::string P = "layer." + std::to_string(li) + ".";
      rmsnorm(h.data(), m->W(P + "input_norm"), eps, x.data());
      if (li % 4 != 3) {  // DeltaNet
        std::vector<uint16_t> qkv(CONV), z(2048), a(DNH), bb(DNH), out(2048);
        matvec(m->W(P + "delta_in_proj_qkv"), x.data(), CONV, HID, qkv.data(), threads);
        matvec(m->W(P + "delta_in_proj_z"), x.data(), 2048, HID, z.data(), threads);
        matvec(m->W(P + "delta_in_proj_a"), x.data(), DNH, HID, a.data(), 1);
        matvec(m->W(P + "delta_in_proj_b"), x.data(), DNH, HID, bb.data(), 1);
        uint16_t* conv = sq.conv.data() + (size_t)di * CONV * 4;
        oracle_conv_l2_qk(1, CONV, 4, DNH * DND, DNH, qkv.data(), conv, m->W(P + "delta_conv"), 1);
        float alb[DNH * 2];
        const float* alog = m->F(P + "delta_a_log");
        const uint16_t* dtb = m->W(P + "delta_dt_bias");
        for (int hh = 0; hh < DNH; ++hh) {
          alb[hh * 2] = alog[hh];
          alb[hh * 2 + 1] = h2f(dtb[hh]);
        }
        oracle_rec_norm_gate(1, DNH, DND, DND, 1.0f / std::sqrt((float)DND), eps, a.data(), bb.data(), alb,
                             qkv.data(), sq.dn_state.data() + (size_t)di * DNH * DND * DND, z.data(),
                             m->F(P + "delta_norm"), out.data(), 1);
        matvec(m->W(P + "delta_out_proj"), out.data(), HID, 2048, y.data(), threads);
        ++di;
      } else {  // gated full attention
        std::vector<uint16_t> proj(ATT_IN), gated(QH * HD);
        matvec(m->W(P + "attn_q"), x.data(), QH * HD * 2, HID, proj.data(), threads);
        matvec(m->W(P + "attn_k"), x.data(), KVH * HD, HID, proj.data() + QH * HD * 2, threads);
        matvec(m->W(P + "attn_v"), x.data(), KVH * HD, HID, proj.data() + QH * HD * 2 + KVH * HD, threads);
        uint16_t* cache = sq.kv.data() + (size_t)ai * m->max_seq * 2 * KVH * HD;
        attention_token(proj.data(), m->W(P + "attn_q_norm"), m->W(P + "attn_k_norm"), eps,
                        m->rope.data() + (size_t)sq.pos * ROT, cache, sq.pos, gated.data());
        matvec(m->W(P + "attn_o"), gated.data(), HID, QH * HD, y.data(), threads);
        ++ai;
      }
      oracle_residual_add(HID, h.data(), y.data(), h.data());
      rmsnorm(h.data(), m->W(P + "post_norm"), eps, x.data());
      std::vector<uint16_t> g(INTER), u(INTER), mm(INTER);
      matvec(m->W(P + "mlp_gate"), x.data(), INTER, HID, g.data(), threads);
      matvec(m->W(P + "mlp_up"), x.data(), INTER, HID, u.data(), threads);
      oracle_silu_gate(INTER, g.data(), u.data(), mm.data());
      matvec(m->W(P + "mlp_down"), mm.data(), HID, INTER, y.data(), threads);
      oracle_residual_add(HID, h.data(), y.data(), h.data());
    }
    rmsnorm(h.data(), m->W("final_norm"), eps, x.data());
    if (hidden_out) std::memcpy(hidden_out + b * HID, x.data(), HID * 2);
    std::vector<uint16_t> logits(m->vocab);
    matvec(emb, x.data(), m->vocab, HID, logits.data(), threads);
    out_tokens[b] = argmax16(logits.data(), m->vocab, margin ? margin + b : nullptr);
    sq.pos += 1;
  }
  return 0;
}

// matvec.comp on its own (per-op parity tests): y[out] = fp16(W[out][in] . x).
extern "C" void oracle_matvec(const uint16_t* W, const uint16_t* x, int out, int in, uint16_t* y, int threads) {
  matvec(W, x, out, in, y, threads);
}

// rms_norm.comp on one 1024-wide row: y = fp16(x * (1/sqrt(mean(x^2) + eps)) * (1 + w)).
extern "C" void oracle_rms_norm(const uint16_t* x, const uint16_t* w, float eps, uint16_t* y) { rmsnorm(x, w, eps, y); }

// argmax.comp on fp16 logits [n].
extern "C" int oracle_argmax(const uint16_t* logits, int n) { return argmax16(logits, n, nullptr); }

// One attention token of one sequence (attention_token above); the RoPE row is
// built here from theta with the reference's host formula.
extern "C" void oracle_attention_decode(const uint16_t* proj, const uint16_t* qn_w, const uint16_t* kn_w, float eps,
                                        float theta, uint16_t* cache, int pos, uint16_t* gated) {
  float cs[ROT];
  for (int i = 0; i < 32; ++i) {
    const float inv_freq = 1.0f / std::pow(theta, 2.0f * (float)i / (float)ROT);
    const float ang = (float)pos * inv_freq;
    cs[2 * i] = std::cos(ang);
    cs[2 * i + 1] = std::sin(ang);
  }
  attention_token(proj, qn_w, kn_w, eps, cs, cache, pos, gated);
}
