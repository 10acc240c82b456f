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
// (the layer-major prefill's attention is attn_tc.cu)
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

// One warp per row, 8 rows per 256-thread CTA. The shader's order is kept:
// slot t (0..255) sums x[4t..4t+3]^2 in order, then a stride-128..1 tree over
// the slots. Slot t = lane + 32 j lives in lane `lane`, so strides 128, 64
// and 32 combine inside a lane and 16..1 go by shfl_down (bit-identical).
__global__ void __launch_bounds__(256) rmsnorm_kernel(const __half* __restrict__ x, const __half* __restrict__ w,
                                                      __half* __restrict__ y, float eps, int batch) {
  const int lane = threadIdx.x & 31, b = blockIdx.x * 8 + (threadIdx.x >> 5);
  pdl_wait();
  pdl_launch();
  if (b >= batch) return;
  const uint2* xr = reinterpret_cast<const uint2*>(x + (size_t)b * HID);
  const uint2* wr = reinterpret_cast<const uint2*>(w);
  float v[8][4], acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint2 u = xr[lane + 32 * j];
    const __half2* h = reinterpret_cast<const __half2*>(&u);
    const float2 f0 = __half22float2(h[0]), f1 = __half22float2(h[1]);
    v[j][0] = f0.x;
    v[j][1] = f0.y;
    v[j][2] = f1.x;
    v[j][3] = f1.y;
    acc[j] = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[j] = __fadd_rn(acc[j], __fmul_rn(v[j][i], v[j][i]));
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) acc[j] = __fadd_rn(acc[j], acc[j + 4]);
#pragma unroll
  for (int j = 0; j < 2; ++j) acc[j] = __fadd_rn(acc[j], acc[j + 2]);
  acc[0] = __fadd_rn(acc[0], acc[1]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc[0] = __fadd_rn(acc[0], __shfl_down_sync(0xffffffffu, acc[0], o));
  const float tot = __shfl_sync(0xffffffffu, acc[0], 0);
  const float nf = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)HID), eps)));
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint2 wu = wr[lane + 32 * j];
    const __half* wh = reinterpret_cast<const __half*>(&wu);
    uint2 o;
    __half* oh = reinterpret_cast<__half*>(&o);
#pragma unroll
    for (int i = 0; i < 4; ++i)
      oh[i] = __float2half_rn(__fmul_rn(__fmul_rn(v[j][i], nf), __fadd_rn(1.0f, __half2float(wh[i]))));
    reinterpret_cast<uint2*>(y + (size_t)b * HID)[lane + 32 * j] = o;
  }
}

// One warp per (row, head), 8 per 256-thread CTA: item = row * (QH + KVH) + head.
// Row r is token r % T of sequence r / T (T = rows_per_seq: 1 in decode, the
// prompt length in prefill), at position pos[seq] + r % T. Lane l holds head
// dims d = l + 32 j; the per-head RMSNorm keeps rms_norm_per_head.comp's
// one-element-per-slot stride-128..1 tree (strides 128..32 in-lane, 16..1 by
// shuffle), and the RoPE pair (d, d + 32), d < 32, sits in one lane.
// qkv: [rows][ld] with [q0 (256) | gate0 (256) | q1 | gate1 | ... | k (2x256) | v (2x256)].
__global__ void __launch_bounds__(256)
    attn_prep_kernel(const __half* __restrict__ qkv, int ld, const __half* __restrict__ qn_w,
                     const __half* __restrict__ kn_w, const float* __restrict__ rope /*[max_seq][64] cos,sin*/,
                     const int* __restrict__ pos, __half* __restrict__ q_out /*[batch][QH][HD]*/,
                     __half* __restrict__ gate_out, __half* __restrict__ kv /*[batch][layers][max_seq][2][KVH][HD]*/,
                     int64_t kv_seq_stride /*elements per sequence*/, int64_t kv_layer_off, float eps, int rows_per_seq,
                     int rows) {
  const int lane = threadIdx.x & 31, item = blockIdx.x * 8 + (threadIdx.x >> 5);
  pdl_wait();
  pdl_launch();
  if (item >= rows * (QH + KVH)) return;
  const int b = item / (QH + KVH), hh = item % (QH + KVH);
  const int seq = b / rows_per_seq;
  const __half* row = qkv + (size_t)b * ld;
  const bool is_q = hh < QH;
  const int kvh = hh - QH;
  const __half* src = is_q ? row + hh * 2 * HD : row + QH * 2 * HD + kvh * HD;
  const __half* nw = is_q ? qn_w : kn_w;
  float x[8], s[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    x[j] = __half2float(src[lane + 32 * j]);
    s[j] = __fmul_rn(x[j], x[j]);
  }
  if (is_q)  // gate: 16-byte segments
    reinterpret_cast<uint4*>(gate_out + ((size_t)b * QH + hh) * HD)[lane] =
        reinterpret_cast<const uint4*>(row + hh * 2 * HD + HD)[lane];
#pragma unroll
  for (int j = 0; j < 4; ++j) s[j] = __fadd_rn(s[j], s[j + 4]);
#pragma unroll
  for (int j = 0; j < 2; ++j) s[j] = __fadd_rn(s[j], s[j + 2]);
  s[0] = __fadd_rn(s[0], s[1]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s[0] = __fadd_rn(s[0], __shfl_down_sync(0xffffffffu, s[0], o));
  const float tot = __shfl_sync(0xffffffffu, s[0], 0);
  const float nf = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)HD), eps)));
  float xn[8];
#pragma unroll
  for (int j = 0; j < 8; ++j)
    xn[j] = __half2float(__float2half_rn(__fmul_rn(__fmul_rn(x[j], nf), __fadd_rn(1.0f, __half2float(nw[lane + 32 * j])))));
  // partial RoPE on the first 64 dims: pair i = lane rotates (d = lane, d = lane + 32)
  const int p = pos[seq] + b % rows_per_seq;
  const float c = rope[(size_t)p * ROT + 2 * lane], sn = rope[(size_t)p * ROT + 2 * lane + 1];
  const float r0 = __fsub_rn(__fmul_rn(xn[0], c), __fmul_rn(xn[1], sn));
  const float r1 = __fadd_rn(__fmul_rn(xn[1], c), __fmul_rn(xn[0], sn));
  xn[0] = r0;
  xn[1] = r1;
  __half* dst = is_q ? q_out + ((size_t)b * QH + hh) * HD
                     : kv + (size_t)seq * kv_seq_stride + kv_layer_off + (size_t)p * (2 * KVH * HD) + kvh * HD;
#pragma unroll
  for (int j = 0; j < 8; ++j) dst[lane + 32 * j] = __float2half_rn(xn[j]);
  if (!is_q) {  // V (no norm, no rope), 16-byte segments
    __half* vbase = kv + (size_t)seq * kv_seq_stride + kv_layer_off + (size_t)p * (2 * KVH * HD) + KVH * HD + kvh * HD;
    reinterpret_cast<uint4*>(vbase)[lane] = reinterpret_cast<const uint4*>(row + QH * 2 * HD + KVH * HD + kvh * HD)[lane];
  }
}

// grid (rows, KVH, ns), 256 threads = 8 warps; rows as in attn_prep_kernel,
// each query row attends causally to positions 0 .. pos[seq] + row % T.
// With ns > 1 (few rows) the positions are split into ns contiguous ranges,
// one per CTA; each CTA leaves its partial (max, sum, weighted V) in ws and
// the last of a row's ns CTAs (atomic ticket, reset for the next launch)
// merges them in range order. Within a CTA, warp w takes positions w, w+8, ...,
// two per round with the next round's K/V rows already loading; lane l owns
// dims 8l..8l+7 of the 4 query heads of this kv head (GQA group).
// Online softmax per warp, merged across warps in shared memory; the output is
// fp16(acc / (sum + 1e-30)) and then fp16(out * sigmoid(gate)).
__global__ void __launch_bounds__(256)
    attn_decode_kernel(const __half* __restrict__ q /*[batch][QH][HD]*/, const __half* __restrict__ gate,
                       const __half* __restrict__ kv, int64_t kv_seq_stride, int64_t kv_layer_off,
                       const int* __restrict__ pos, float scale, __half* __restrict__ out /*[rows][QH*HD]*/,
                       int rows_per_seq, int ns, float* __restrict__ ws, int* __restrict__ tickets) {
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
  const int span = (L + ns - 1) / ns, p_lo = blockIdx.z * span, p_hi = min(L, p_lo + span);
  // K and V rows of position p (zeros past the range; the update skips them)
  auto load = [&](int p, uint4& ku, uint4& vu) {
    if (p < p_hi) {
      const __half* row = base + (size_t)p * (2 * KVH * HD) + kvh * HD + lane * 8;
      ku = *reinterpret_cast<const uint4*>(row);
      vu = *reinterpret_cast<const uint4*>(row + KVH * HD);
    } else {
      ku = vu = make_uint4(0, 0, 0, 0);
    }
  };
  // online softmax update of this warp's state with one position
  auto update = [&](const uint4& ku, const uint4& vu) {
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
    float dot[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      dot[g] = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k) dot[g] = fmaf(qv[g][k], kf[k], dot[g]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int g = 0; g < G; ++g) dot[g] += __shfl_xor_sync(0xffffffffu, dot[g], o);
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float sc = dot[g] * scale;
      const float mn = fmaxf(m[g], sc);
      const float corr = __expf(m[g] - mn), w = __expf(sc - mn);
      l[g] = l[g] * corr + w;
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[g][k] = fmaf(w, vf[k], acc[g][k] * corr);
      m[g] = mn;
    }
  };
  // two positions per round (p, p + 8); the next round's rows are loaded
  // before this round's arithmetic
  int p = p_lo + warp;
  uint4 k0, v0, k1, v1;
  load(p, k0, v0);
  load(p + 8, k1, v1);
  for (; p < p_hi; p += 16) {
    uint4 nk0, nv0, nk1, nv1;
    load(p + 16, nk0, nv0);
    load(p + 24, nk1, nv1);
    update(k0, v0);
    if (p + 8 < p_hi) update(k1, v1);
    k0 = nk0;
    v0 = nv0;
    k1 = nk1;
    v1 = nv1;
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
  if (ns > 1) {
    // this range's partial -> ws[row][kvh][range]: m[4] | l[4] | acc[4][256]
    float* part = ws + (((size_t)b * KVH + kvh) * ns + blockIdx.z) * (2 * G + G * HD);
    if ((threadIdx.x & 63) == 0) {
      part[g] = mt;
      part[G + g] = lt;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) part[2 * G + g * HD + d0 + k] = at[k];
    __threadfence();
    __syncthreads();
    __shared__ int s_last;
    if (threadIdx.x == 0) {
      int* tk = tickets + (size_t)b * KVH + kvh;
      const int n = atomicAdd(tk, 1);
      s_last = n == ns - 1;
      if (s_last) *tk = 0;  // ready for the next launch
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const float* parts = ws + ((size_t)b * KVH + kvh) * ns * (2 * G + G * HD);
    mt = -INFINITY;
    for (int z = 0; z < ns; ++z) mt = fmaxf(mt, __ldcg(parts + z * (2 * G + G * HD) + g));
    lt = 0.f;
    at[0] = at[1] = at[2] = at[3] = 0.f;
    for (int z = 0; z < ns; ++z) {
      const float* pz = parts + z * (2 * G + G * HD);
      const float mz = __ldcg(pz + g);
      if (mz == -INFINITY) continue;
      const float c = expf(mz - mt);
      lt += __ldcg(pz + G + g) * c;
#pragma unroll
      for (int k = 0; k < 4; ++k) at[k] += __ldcg(pz + 2 * G + g * HD + d0 + k) * c;
    }
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

}  // namespace

Status launch_embed(const int* tokens, const void* emb, void* h, int batch, cudaStream_t st) {
  launch_k(embed_kernel, dim3(batch), dim3(128), 0, st, tokens, (const uint4*)emb, (uint4*)h, batch);
  SPOCK_LAUNCH_CHECK("embed_kernel");
  return Status::ok();
}

Status launch_rmsnorm(const void* x, const void* w, void* y, float eps, int batch, cudaStream_t st) {
  launch_k(rmsnorm_kernel, dim3((batch + 7) / 8), dim3(256), 0, st, (const __half*)x, (const __half*)w, (__half*)y, eps,
           batch);
  SPOCK_LAUNCH_CHECK("rmsnorm_kernel");
  return Status::ok();
}

Status launch_attn_prep(const void* qkv, int ld, const void* qn_w, const void* kn_w, const float* rope,
                        const int* pos, void* q_out, void* gate_out, void* kv, int64_t kv_seq_stride,
                        int64_t kv_layer_off, float eps, int rows, cudaStream_t st, int rows_per_seq) {
  launch_k(attn_prep_kernel, dim3((rows * (QH + KVH) + 7) / 8), dim3(256), 0, st, (const __half*)qkv, ld,
           (const __half*)qn_w, (const __half*)kn_w, rope, pos, (__half*)q_out, (__half*)gate_out, (__half*)kv,
           kv_seq_stride, kv_layer_off, eps, rows_per_seq, rows);
  SPOCK_LAUNCH_CHECK("attn_prep_kernel");
  return Status::ok();
}

// Position ranges per row for the split decode attention: enough CTAs to
// occupy the SMs when there are few rows (the partials need ws/tickets).
int attn_decode_splits(int rows) { return rows <= 4 ? 16 : (rows <= 16 ? 4 : 1); }

Status launch_attn_decode(const void* q, const void* gate, const void* kv, int64_t kv_seq_stride,
                          int64_t kv_layer_off, const int* pos, float scale, void* out, int rows,
                          cudaStream_t st, int rows_per_seq, float* ws, int* tickets) {
  const int ns = (ws && tickets) ? attn_decode_splits(rows) : 1;
  launch_k(attn_decode_kernel, dim3(rows, KVH, ns), dim3(256), 0, st, (const __half*)q, (const __half*)gate,
           (const __half*)kv, kv_seq_stride, kv_layer_off, pos, scale, (__half*)out, rows_per_seq, ns, ws, tickets);
  SPOCK_LAUNCH_CHECK("attn_decode_kernel");
  return Status::ok();
}

}  // namespace spock
