// Decode glue around the DeltaNet mixer for the Qwen3.5-0.8B layout, batched
// over independent sequences (one row per sequence). Each kernel restates a
// reference shader's arithmetic, including its fp16 storage points:
//   embed_kernel       shaders/embedding_lookup.comp
//   rmsnorm_kernel     shaders/rms_norm.comp:31-70 (x * rsqrt(mean(x^2)+eps) * (1+w);
//                      4 consecutive elements per lane, then a stride-128..1 tree)
//   attn_prep_kernel   split_q_gate.comp + rms_norm_per_head.comp (q_norm, k_norm)
//                      + rope_apply.comp (rotary 64 of 256, pairs d / d+32, host
//                      cos/sin table) + kv_cache_store.comp, fused per head
//   attn_decode_kernel attention_decode.comp (GQA 8 q / 2 kv heads, head 256,
//                      softmax over positions 0..pos) + sigmoid_gate.comp, fused
#include <mutex>

#include "common.cuh"

namespace spock {
namespace {

constexpr int HID = 1024;
constexpr int HD = 256;       // attention head dim
constexpr int QH = 8, KVH = 2;
constexpr int ROT = 64;

__global__ void embed_kernel(const int* __restrict__ tokens, const uint4* __restrict__ emb, uint4* __restrict__ h,
                             int batch) {
  const int b = blockIdx.x;
  pdl_wait();
  pdl_launch();
  if (b >= batch) return;
  const int tok = tokens[b];
  for (int i = threadIdx.x; i < HID / 8; i += blockDim.x) h[(size_t)b * (HID / 8) + i] = emb[(size_t)tok * (HID / 8) + i];
}

// One CTA (256 threads) per row.
__global__ void __launch_bounds__(256) rmsnorm_kernel(const __half* __restrict__ x, const __half* __restrict__ w,
                                                      __half* __restrict__ y, float eps, int batch) {
  const int b = blockIdx.x, t = threadIdx.x;
  pdl_wait();
  pdl_launch();
  if (b >= batch) return;
  __shared__ float s[256];
  const __half* xr = x + (size_t)b * HID;
  float v[4], acc = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[i] = __half2float(xr[t * 4 + i]);
    acc = __fadd_rn(acc, __fmul_rn(v[i], v[i]));
  }
  s[t] = acc;
  __syncthreads();
  for (int stride = 128; stride > 0; stride >>= 1) {
    if (t < stride) s[t] = __fadd_rn(s[t], s[t + stride]);
    __syncthreads();
  }
  const float nf = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s[0], (float)HID), eps)));
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float wv = __fadd_rn(1.0f, __half2float(w[t * 4 + i]));
    y[(size_t)b * HID + t * 4 + i] = __float2half_rn(__fmul_rn(__fmul_rn(v[i], nf), wv));
  }
}

// grid (rows, QH + KVH), 256 threads (thread d = head dimension d). Row r is
// token r % T of sequence r / T (T = rows_per_seq: 1 in decode, the prompt
// length in prefill), at position pos[seq] + r % T.
// qkv: [rows][ld] with [q0 (256) | gate0 (256) | q1 | gate1 | ... | k (2x256) | v (2x256)].
__global__ void __launch_bounds__(256)
    attn_prep_kernel(const __half* __restrict__ qkv, int ld, const __half* __restrict__ qn_w,
                     const __half* __restrict__ kn_w, const float* __restrict__ rope /*[max_seq][64] cos,sin*/,
                     const int* __restrict__ pos, __half* __restrict__ q_out /*[batch][QH][HD]*/,
                     __half* __restrict__ gate_out, __half* __restrict__ kv /*[batch][layers][max_seq][2][KVH][HD]*/,
                     int64_t kv_seq_stride /*elements per sequence*/, int64_t kv_layer_off, float eps, int rows_per_seq) {
  const int hh = blockIdx.y, b = blockIdx.x, d = threadIdx.x;  // b: row
  const int seq = b / rows_per_seq;
  pdl_wait();
  pdl_launch();
  const __half* row = qkv + (size_t)b * ld;
  __shared__ float s[256];
  __shared__ float sn[256];
  const bool is_q = hh < QH;
  const int kvh = hh - QH;
  const float x = __half2float(is_q ? row[hh * 2 * HD + d] : row[QH * 2 * HD + kvh * HD + d]);
  if (is_q) gate_out[((size_t)b * QH + hh) * HD + d] = row[hh * 2 * HD + HD + d];
  // per-head RMSNorm (rms_norm_per_head.comp: one element per lane, stride-128..1 tree)
  s[d] = __fmul_rn(x, x);
  __syncthreads();
  for (int stride = 128; stride > 0; stride >>= 1) {
    if (d < stride) s[d] = __fadd_rn(s[d], s[d + stride]);
    __syncthreads();
  }
  const float nf = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s[0], (float)HD), eps)));
  const float wv = __fadd_rn(1.0f, __half2float(is_q ? qn_w[d] : kn_w[d]));
  const float xn = __half2float(__float2half_rn(__fmul_rn(__fmul_rn(x, nf), wv)));
  sn[d] = xn;
  __syncthreads();
  // partial RoPE: pairs (d, d+32) for d < 32 of the first 64 dims
  float o = xn;
  const int p = pos[seq] + b % rows_per_seq;
  if (d < ROT) {
    const int i = d & 31;
    const float c = rope[(size_t)p * ROT + 2 * i], sn_ = rope[(size_t)p * ROT + 2 * i + 1];
    if (d < 32) o = __fsub_rn(__fmul_rn(xn, c), __fmul_rn(sn[d + 32], sn_));
    else o = __fadd_rn(__fmul_rn(xn, c), __fmul_rn(sn[d - 32], sn_));
  }
  const __half oh = __float2half_rn(o);
  if (is_q) {
    q_out[((size_t)b * QH + hh) * HD + d] = oh;
  } else {
    __half* base = kv + (size_t)seq * kv_seq_stride + kv_layer_off + (size_t)p * (2 * KVH * HD);
    base[kvh * HD + d] = oh;                                          // K
    base[KVH * HD + kvh * HD + d] = row[QH * 2 * HD + KVH * HD + kvh * HD + d];  // V (no norm, no rope)
  }
}

// grid (rows, KVH), 256 threads = 8 warps; rows as in attn_prep_kernel, each
// query row attends causally to positions 0 .. pos[seq] + row % T.
// Warp w takes positions w, w+8, ...;
// lane l owns dims 8l..8l+7 of the 4 query heads of this kv head (GQA group).
// Online softmax per warp, merged across warps in shared memory; the output is
// fp16(acc / (sum + 1e-30)) and then fp16(out * sigmoid(gate)).
__global__ void __launch_bounds__(256)
    attn_decode_kernel(const __half* __restrict__ q /*[batch][QH][HD]*/, const __half* __restrict__ gate,
                       const __half* __restrict__ kv, int64_t kv_seq_stride, int64_t kv_layer_off,
                       const int* __restrict__ pos, float scale, __half* __restrict__ out /*[rows][QH*HD]*/,
                       int rows_per_seq) {
  const int kvh = blockIdx.y, b = blockIdx.x;  // b: row
  const int seq = b / rows_per_seq;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int G = QH / KVH;  // 4
  pdl_wait();
  pdl_launch();
  const int L = pos[seq] + b % rows_per_seq + 1;
  float qv[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const uint4 u = *reinterpret_cast<const uint4*>(q + ((size_t)b * QH + kvh * G + g) * HD + lane * 8);
    const __half2* h2 = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = __half22float2(h2[k]);
      qv[g][2 * k] = f.x;
      qv[g][2 * k + 1] = f.y;
    }
  }
  float m[G], l[G], acc[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[g][k] = 0.f;
  }
  const __half* base = kv + (size_t)seq * kv_seq_stride + kv_layer_off;
  for (int p = warp; p < L; p += 8) {
    const __half* kr = base + (size_t)p * (2 * KVH * HD) + kvh * HD + lane * 8;
    const __half* vr = base + (size_t)p * (2 * KVH * HD) + KVH * HD + kvh * HD + lane * 8;
    const uint4 ku = *reinterpret_cast<const uint4*>(kr);
    const uint4 vu = *reinterpret_cast<const uint4*>(vr);
    float kf[8], vf[8];
    const __half2* k2 = reinterpret_cast<const __half2*>(&ku);
    const __half2* v2 = reinterpret_cast<const __half2*>(&vu);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 a = __half22float2(k2[k]), c = __half22float2(v2[k]);
      kf[2 * k] = a.x;
      kf[2 * k + 1] = a.y;
      vf[2 * k] = c.x;
      vf[2 * k + 1] = c.y;
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float dot = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k) dot = fmaf(qv[g][k], kf[k], dot);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
      const float sc = dot * scale;
      const float mn = fmaxf(m[g], sc);
      const float corr = expf(m[g] - mn), w = expf(sc - mn);
      l[g] = l[g] * corr + w;
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[g][k] = fmaf(w, vf[k], acc[g][k] * corr);
      m[g] = mn;
    }
  }
  __shared__ float sm_m[8][G], sm_l[8][G];
  __shared__ float sm_acc[8][G][HD];
  if (lane == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      sm_m[warp][g] = m[g];
      sm_l[warp][g] = l[g];
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int k = 0; k < 8; ++k) sm_acc[warp][g][lane * 8 + k] = acc[g][k];
  __syncthreads();
  // thread t -> (g = t / 64, dims 4*(t%64)..+3)
  const int g = threadIdx.x >> 6, d0 = (threadIdx.x & 63) * 4;
  float mt = -INFINITY;
  for (int w = 0; w < 8; ++w) mt = fmaxf(mt, sm_m[w][g]);
  float lt = 0.f, at[4] = {0.f, 0.f, 0.f, 0.f};
  for (int w = 0; w < 8; ++w) {
    if (sm_m[w][g] == -INFINITY) continue;
    const float c = expf(sm_m[w][g] - mt);
    lt += sm_l[w][g] * c;
#pragma unroll
    for (int k = 0; k < 4; ++k) at[k] += sm_acc[w][g][d0 + k] * c;
  }
  const float inv = 1.0f / (lt + 1e-30f);
  const int qh = kvh * G + g;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float a16 = __half2float(__float2half_rn(at[k] * inv));
    const float gt = __half2float(gate[((size_t)b * QH + qh) * HD + d0 + k]);
    const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-gt)));
    out[((size_t)b * QH + qh) * HD + d0 + k] = __float2half_rn(__fmul_rn(a16, sig));
  }
}

// ---- prefill attention: query tiles on the tensor cores ---------------------
// The layer-major prefill's causal attention, tiled: a CTA takes 16 prompt rows
// of one sequence and one kv head, i.e. 64 query vectors (warp w = q head
// kvh*4 + w, 16 rows each), and walks the KV cache in 64-position tiles.
// S = Q Kᵀ and O += P V run as mma.sync m16n8k16 (fp16 operands, fp32
// accumulation; P is rounded to fp16), with the online softmax of
// attention_decode.comp per row in registers. The output is
// fp16(O / (l + 1e-30)) gated by sigmoid, as in attn_decode_kernel.
constexpr int kAR = 16, kAP = 64, kLDH = HD + 8;  // rows per CTA, positions per tile, padded smem row
constexpr int kAttnPrefillSmem = 3 * 64 * kLDH * 2;

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const __half* p) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const __half* p) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// grid (ceil(T / 16) * batch, KVH), 128 threads; q, gate, out rows r = seq*T + t.
__global__ void __launch_bounds__(128, 1)
    attn_prefill_kernel(const __half* __restrict__ q, const __half* __restrict__ gate, const __half* __restrict__ kv,
                        int64_t kv_seq_stride, int64_t kv_layer_off, const int* __restrict__ pos, float scale,
                        __half* __restrict__ out, int T) {
  extern __shared__ __align__(16) uint8_t attn_smem[];
  __half* Qs = reinterpret_cast<__half*>(attn_smem);
  __half* Ks = Qs + 64 * kLDH;
  __half* Vs = Ks + kAP * kLDH;
  constexpr int G = QH / KVH;  // 4 q heads per kv head
  const int tiles = (T + kAR - 1) / kAR;
  const int seq = blockIdx.x / tiles, t0 = (blockIdx.x % tiles) * kAR, kvh = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, tq = lane & 3;
  pdl_wait();
  pdl_launch();
  const int p_base = pos[seq];
  const int rows_here = min(kAR, T - t0);
  const int Lmax = p_base + t0 + rows_here;  // positions 0 .. Lmax-1 are read
  for (int c = tid; c < 64 * (HD / 8); c += 128) {  // Q tile: row i = w*16 + r
    const int i = c / (HD / 8), d8 = c % (HD / 8), w = i / kAR, r = i % kAR;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < rows_here) v = *reinterpret_cast<const uint4*>(q + ((size_t)(seq * T + t0 + r) * QH + kvh * G + w) * HD + d8 * 8);
    *reinterpret_cast<uint4*>(Qs + i * kLDH + d8 * 8) = v;
  }
  float o[HD / 8][4];
#pragma unroll
  for (int nd = 0; nd < HD / 8; ++nd) o[nd][0] = o[nd][1] = o[nd][2] = o[nd][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const int lim0 = p_base + t0 + g, lim1 = p_base + t0 + g + 8;  // last position rows g, g+8 attend to
  const __half* base = kv + (size_t)seq * kv_seq_stride + kv_layer_off;
  for (int p0 = 0; p0 < Lmax; p0 += kAP) {
    __syncthreads();  // the previous tile's K/V reads are done
    for (int c = tid; c < kAP * (HD / 8); c += 128) {
      const int j = c / (HD / 8), d8 = c % (HD / 8), p = p0 + j;
      uint4 kk = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
      if (p < Lmax) {
        const __half* row = base + (size_t)p * (2 * KVH * HD) + kvh * HD + d8 * 8;
        kk = *reinterpret_cast<const uint4*>(row);
        vv = *reinterpret_cast<const uint4*>(row + KVH * HD);
      }
      *reinterpret_cast<uint4*>(Ks + j * kLDH + d8 * 8) = kk;
      *reinterpret_cast<uint4*>(Vs + j * kLDH + d8 * 8) = vv;
    }
    __syncthreads();
    float sc[kAP / 8][4];
#pragma unroll
    for (int nt = 0; nt < kAP / 8; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll 4
    for (int ks = 0; ks < HD / 16; ++ks) {
      uint32_t a[4];
      ldsm_x4(a, Qs + (warp * 16 + (lane & 15)) * kLDH + ks * 16 + (lane >> 4) * 8);
#pragma unroll
      for (int nt = 0; nt < kAP / 8; nt += 2) {
        uint32_t b[4];
        ldsm_x4(b, Ks + (nt * 8 + ((lane >> 4) & 1) * 8 + (lane & 7)) * kLDH + ks * 16 + ((lane >> 3) & 1) * 8);
        mma16816(sc[nt], a, b[0], b[1]);
        mma16816(sc[nt + 1], a, b[2], b[3]);
      }
    }
    // scale, causal mask, online softmax (rows g and g+8 of this warp's 16)
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < kAP / 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int p = p0 + nt * 8 + 2 * tq + (e & 1);
        float v = sc[nt][e] * scale;
        if (p > (e < 2 ? lim0 : lim1)) v = -INFINITY;
        sc[nt][e] = v;
      }
      mx0 = fmaxf(mx0, fmaxf(sc[nt][0], sc[nt][1]));
      mx1 = fmaxf(mx1, fmaxf(sc[nt][2], sc[nt][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);  // finite: position 0 is in every row's first tile
    const float c0 = expf(m0 - mn0), c1 = expf(m1 - mn1);
    m0 = mn0;
    m1 = mn1;
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int nt = 0; nt < kAP / 8; ++nt) {
      // P is rounded to fp16 here, where the P.V mma will see it, so the
      // denominators sum exactly the weights the numerators use
      sc[nt][0] = __half2float(__float2half_rn(expf(sc[nt][0] - mn0)));
      sc[nt][1] = __half2float(__float2half_rn(expf(sc[nt][1] - mn0)));
      sc[nt][2] = __half2float(__float2half_rn(expf(sc[nt][2] - mn1)));
      sc[nt][3] = __half2float(__float2half_rn(expf(sc[nt][3] - mn1)));
      s0 += sc[nt][0] + sc[nt][1];
      s1 += sc[nt][2] + sc[nt][3];
    }
    l0 = l0 * c0 + s0;
    l1 = l1 * c1 + s1;
#pragma unroll
    for (int nd = 0; nd < HD / 8; ++nd) {
      o[nd][0] *= c0;
      o[nd][1] *= c0;
      o[nd][2] *= c1;
      o[nd][3] *= c1;
    }
    // O += P V: P's accumulator tiles (2j, 2j+1) are the A operand of k step j
#pragma unroll
    for (int j = 0; j < kAP / 16; ++j) {
      const uint32_t a[4] = {pack_h2(sc[2 * j][0], sc[2 * j][1]), pack_h2(sc[2 * j][2], sc[2 * j][3]),
                             pack_h2(sc[2 * j + 1][0], sc[2 * j + 1][1]), pack_h2(sc[2 * j + 1][2], sc[2 * j + 1][3])};
#pragma unroll
      for (int nd = 0; nd < HD / 8; nd += 2) {
        uint32_t b[4];
        ldsm_x4_t(b, Vs + (16 * j + ((lane >> 3) & 1) * 8 + (lane & 7)) * kLDH + nd * 8 + (lane >> 4) * 8);
        mma16816(o[nd], a, b[0], b[1]);
        mma16816(o[nd + 1], a, b[2], b[3]);
      }
    }
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = 1.0f / (l0 + 1e-30f), inv1 = 1.0f / (l1 + 1e-30f);
  const int qh = kvh * G + warp;
#pragma unroll
  for (int half_row = 0; half_row < 2; ++half_row) {
    const int r = g + 8 * half_row;
    if (r >= rows_here) continue;
    const float inv = half_row ? inv1 : inv0;
    const size_t off = ((size_t)(seq * T + t0 + r) * QH + qh) * HD + 2 * tq;
#pragma unroll
    for (int nd = 0; nd < HD / 8; ++nd) {
      const __half2 gt2 = *reinterpret_cast<const __half2*>(gate + off + nd * 8);
      const float2 gt = __half22float2(gt2);
      float res[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float a16 = __half2float(__float2half_rn(o[nd][2 * half_row + e] * inv));
        const float gv = e ? gt.y : gt.x;
        const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-gv)));
        res[e] = __fmul_rn(a16, sig);
      }
      *reinterpret_cast<__half2*>(out + off + nd * 8) = __floats2half2_rn(res[0], res[1]);
    }
  }
}

}  // namespace

Status launch_attn_prefill(const void* q, const void* gate, const void* kv, int64_t kv_seq_stride,
                           int64_t kv_layer_off, const int* pos, float scale, void* out, int batch, int T,
                           cudaStream_t st) {
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [] {
    attr = cudaFuncSetAttribute(attn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnPrefillSmem);
  });
  if (attr != cudaSuccess) return cuda_status(attr, "attn_prefill_kernel attribute");
  const int tiles = (T + kAR - 1) / kAR;
  launch_k(attn_prefill_kernel, dim3(tiles * batch, KVH), dim3(128), kAttnPrefillSmem, st, (const __half*)q,
           (const __half*)gate, (const __half*)kv, kv_seq_stride, kv_layer_off, pos, scale, (__half*)out, T);
  SPOCK_LAUNCH_CHECK("attn_prefill_kernel");
  return Status::ok();
}

Status launch_embed(const int* tokens, const void* emb, void* h, int batch, cudaStream_t st) {
  launch_k(embed_kernel, dim3(batch), dim3(128), 0, st, tokens, (const uint4*)emb, (uint4*)h, batch);
  SPOCK_LAUNCH_CHECK("embed_kernel");
  return Status::ok();
}

Status launch_rmsnorm(const void* x, const void* w, void* y, float eps, int batch, cudaStream_t st) {
  launch_k(rmsnorm_kernel, dim3(batch), dim3(256), 0, st, (const __half*)x, (const __half*)w, (__half*)y, eps, batch);
  SPOCK_LAUNCH_CHECK("rmsnorm_kernel");
  return Status::ok();
}

Status launch_attn_prep(const void* qkv, int ld, const void* qn_w, const void* kn_w, const float* rope,
                        const int* pos, void* q_out, void* gate_out, void* kv, int64_t kv_seq_stride,
                        int64_t kv_layer_off, float eps, int rows, cudaStream_t st, int rows_per_seq) {
  launch_k(attn_prep_kernel, dim3(rows, QH + KVH), dim3(256), 0, st, (const __half*)qkv, ld, (const __half*)qn_w,
           (const __half*)kn_w, rope, pos, (__half*)q_out, (__half*)gate_out, (__half*)kv, kv_seq_stride,
           kv_layer_off, eps, rows_per_seq);
  SPOCK_LAUNCH_CHECK("attn_prep_kernel");
  return Status::ok();
}

Status launch_attn_decode(const void* q, const void* gate, const void* kv, int64_t kv_seq_stride,
                          int64_t kv_layer_off, const int* pos, float scale, void* out, int rows,
                          cudaStream_t st, int rows_per_seq) {
  launch_k(attn_decode_kernel, dim3(rows, KVH), dim3(256), 0, st, (const __half*)q, (const __half*)gate,
           (const __half*)kv, kv_seq_stride, kv_layer_off, pos, scale, (__half*)out, rows_per_seq);
  SPOCK_LAUNCH_CHECK("attn_decode_kernel");
  return Status::ok();
}

}  // namespace spock
