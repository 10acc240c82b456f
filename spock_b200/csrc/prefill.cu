// Layer-major prefill of a DeltaNet layer (the batched form of the reference's
// layer_major_prefill, src/runtime/vk_session.cpp:1003-2018): the per-token
// causal conv + SiLU + L2 of deltanet_conv_l2_qk.comp:41-110 over a whole
// prompt, the g/beta of deltanet_recurrent_gbeta_norm_gate.comp:101-115, a
// head-major hand-off to the tcgen05 chunk rule (this replaces the collect
// shader deltanet_prefill_collect.comp:75-107), and the gated RMSNorm of
// deltanet_recurrent_gbeta_norm_gate.comp:300-335 on the chunk outputs.
// Every per-token formula, rounding point and reduction order is the decode
// step's (decode_step.cu), so prefill and token-serial decode agree up to the
// chunk rule's own regrouping.
#include "common.cuh"

namespace spock {
namespace {

constexpr int kDim = 128;
constexpr int kTokTile = 16;  // tokens per CTA of the conv kernel (many CTAs: each thread walks its tokens in order)

// The shaders' stride-64..1 tree over s[0..127] by one warp (decode_step.cu).
__device__ __forceinline__ float warp_tree128(const float* s, int lane) {
  float v0 = s[lane], v1 = s[lane + 32];
  v0 += s[lane + 64];
  v1 += s[lane + 96];
  v0 += v1;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v0 += __shfl_down_sync(0xffffffffu, v0, o);
  return v0;
}

// grid (3 * H channel blocks [q heads | k heads | v heads], batch, ceil(T / kTokTile)),
// 128 threads (thread c = channel c of the block).
// proj: [rows = b * T + t][ld] fp16 token rows [qkv 3*H*128 | z H*128 | a H | b H].
// conv_old: [batch][3*H*128][4] fp16 (slots = the last four inputs, oldest
// first), a snapshot of the state before the prompt; conv_new (the live state)
// receives the prompt's last four inputs. Separate buffers, because the CTA of
// the last tile may finish before the CTA of the first tile reads the old state. Outputs q, k (L2-normalised) and v
// head-major [batch][H][T][128] fp16; g, beta [batch][H][T] fp32.
__global__ void __launch_bounds__(kDim)
    dn_prefill_conv_kernel(const __half* __restrict__ proj, int ld, int T, int H, const uint16_t* __restrict__ conv_w,
                           const uint16_t* __restrict__ conv_old, uint16_t* __restrict__ conv_new,
                           const float* __restrict__ a_log_bias,
                           __half* __restrict__ q_out, __half* __restrict__ k_out, __half* __restrict__ v_out,
                           float* __restrict__ g_out, float* __restrict__ beta_out) {
  const int blk = blockIdx.x / H, h = blockIdx.x % H, b = blockIdx.y, c = threadIdx.x;
  const int t0 = blockIdx.z * kTokTile, t1 = min(T, t0 + kTokTile);
  const int conv_dim = 3 * H * kDim;
  const int ch = blk * H * kDim + h * kDim + c;
  __shared__ float sq[kTokTile][kDim];
  __shared__ float inv_s[kTokTile];
  pdl_wait();
  pdl_launch();
  const __half* xrow = proj + (size_t)b * T * ld + ch;
  const uint16_t* cs = conv_old + ((size_t)b * conv_dim + ch) * 4;
  uint16_t* cn = conv_new + ((size_t)b * conv_dim + ch) * 4;
  const uint2 wv = *reinterpret_cast<const uint2*>(conv_w + (size_t)ch * 4);
  const float w0 = h2f((uint16_t)(wv.x & 0xffff)), w1 = h2f((uint16_t)(wv.x >> 16)),
              w2 = h2f((uint16_t)(wv.y & 0xffff)), w3 = h2f((uint16_t)(wv.y >> 16));
  const uint2 st = *reinterpret_cast<const uint2*>(cs);  // x_{-4} x_{-3} x_{-2} x_{-1}
  const uint16_t sv[4] = {(uint16_t)(st.x & 0xffff), (uint16_t)(st.x >> 16), (uint16_t)(st.y & 0xffff),
                          (uint16_t)(st.y >> 16)};
  auto xin = [&](int t) -> uint16_t {  // input of token t (t >= -4)
    return t >= 0 ? __half_as_ushort(xrow[(size_t)t * ld]) : sv[4 + t];
  };
  // the tile's inputs, all loads in flight at once
  uint16_t xs[kTokTile];
#pragma unroll
  for (int u = 0; u < kTokTile; ++u) xs[u] = t0 + u < t1 ? __half_as_ushort(xrow[(size_t)(t0 + u) * ld]) : 0;
  uint16_t s1 = xin(t0 - 3), s2 = xin(t0 - 2), s3 = xin(t0 - 1);
  __half* dst = (blk == 0 ? q_out : blk == 1 ? k_out : v_out) + (((size_t)b * H + h) * T) * kDim + c;
  float yf[kTokTile];
#pragma unroll
  for (int u = 0; u < kTokTile; ++u) {
    yf[u] = 0.f;
    if (t0 + u < t1) {
      const uint16_t x = xs[u];
      float sum = 0.f;
      sum = add_rn(sum, mul_rn(h2f(s1), w0));
      sum = add_rn(sum, mul_rn(h2f(s2), w1));
      sum = add_rn(sum, mul_rn(h2f(s3), w2));
      sum = add_rn(sum, mul_rn(h2f(x), w3));
      const float silu = __fdiv_rn(sum, add_rn(1.0f, expf(-sum)));
      yf[u] = h2f(f2h(silu));
      s1 = s2;
      s2 = s3;
      s3 = x;
    }
    if (blk < 2) sq[u][c] = mul_rn(yf[u], yf[u]);
  }
  if (blk < 2) {  // L2 of this head's q or k for each token of the tile
    __syncthreads();
    const int warp = c >> 5, lane = c & 31;
    for (int u = warp; u < kTokTile; u += kDim / 32) {
      const float tot = warp_tree128(sq[u], lane);
      if (lane == 0) inv_s[u] = __fdiv_rn(1.0f, __fsqrt_rn(add_rn(tot, 1e-6f)));
    }
    __syncthreads();
  }
#pragma unroll
  for (int u = 0; u < kTokTile; ++u) {
    if (t0 + u >= t1) break;
    dst[(size_t)(t0 + u) * kDim] = blk < 2 ? __float2half_rn(mul_rn(yf[u], inv_s[u])) : __float2half_rn(yf[u]);
  }
  // the CTA holding the last token leaves the conv state at the prompt's last four inputs
  if (t1 == T) {
    const uint16_t n0 = xin(T - 4), n1 = xin(T - 3), n2 = xin(T - 2), n3 = xin(T - 1);
    *reinterpret_cast<uint2*>(cn) = make_uint2((uint32_t)n0 | ((uint32_t)n1 << 16), (uint32_t)n2 | ((uint32_t)n3 << 16));
  }
  // g and beta of this head for the tile's tokens (q-block CTAs)
  if (blk == 0) {
    for (int t = t0 + c; t < t1; t += kDim) {
      const __half* row = proj + ((size_t)b * T + t) * ld;
      const float a_val = __half2float(row[conv_dim + H * kDim + h]);
      const float b_val = __half2float(row[conv_dim + H * kDim + H + h]);
      const float a_log = a_log_bias[h * 2 + 0], dt_bias = a_log_bias[h * 2 + 1];
      const float sp = logf(add_rn(1.0f, expf(add_rn(a_val, dt_bias))));
      g_out[((size_t)b * H + h) * T + t] = mul_rn(-expf(a_log), sp);
      beta_out[((size_t)b * H + h) * T + t] = __fdiv_rn(1.0f, add_rn(1.0f, expf(-b_val)));
    }
  }
}

// One warp per (row, head), 8 per 256-thread CTA: gated RMSNorm of the chunk
// rule's output. Lane l holds channels l + 32 j; the sum of squares is
// warp_tree128's order (the shader's stride-64..1 tree).
// core: [batch][H][T][128] fp32; z from proj row [.. | z (H*128) | ..] at column z_off;
// out: [rows][H*128] fp16 (token rows for the output projection).
__global__ void __launch_bounds__(256)
    dn_prefill_gate_kernel(const float* __restrict__ core, const __half* __restrict__ proj, int ld, int z_off,
                           const float* __restrict__ norm_w, float eps, int T, int H, int rows,
                           __half* __restrict__ out) {
  const int lane = threadIdx.x & 31, item = blockIdx.x * 8 + (threadIdx.x >> 5);
  pdl_wait();
  pdl_launch();
  if (item >= rows * H) return;
  const int row = item / H, h = item % H, b = row / T, t = row % T;
  const float* cr = core + (((size_t)b * H + h) * T + t) * kDim;
  const __half* zr = proj + (size_t)row * ld + z_off + h * kDim;
  float o[4], zz[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    o[j] = cr[lane + 32 * j];
    zz[j] = __half2float(zr[lane + 32 * j]);
  }
  float v0 = mul_rn(o[0], o[0]), v1 = mul_rn(o[1], o[1]);
  v0 = add_rn(v0, mul_rn(o[2], o[2]));
  v1 = add_rn(v1, mul_rn(o[3], o[3]));
  v0 = add_rn(v0, v1);
#pragma unroll
  for (int k = 16; k > 0; k >>= 1) v0 += __shfl_down_sync(0xffffffffu, v0, k);
  const float ss = __shfl_sync(0xffffffffu, v0, 0);
  const float nf = __fdiv_rn(1.0f, __fsqrt_rn(add_rn(__fdiv_rn(ss, (float)kDim), eps)));
  __half* dst = out + (size_t)row * (H * kDim) + h * kDim;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float normed = mul_rn(o[j], nf);
    const float silu = __fdiv_rn(zz[j], add_rn(1.0f, expf(-zz[j])));
    const float weighted = h2f(f2h(mul_rn(norm_w[lane + 32 * j], normed)));
    dst[lane + 32 * j] = __float2half_rn(mul_rn(weighted, silu));
  }
}

// dst[b] = src[b * T + T - 1] (rows of `width` halves): the last prompt token of each sequence.
__global__ void last_rows_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst, int T, int width8) {
  const int b = blockIdx.x;
  pdl_wait();
  pdl_launch();
  for (int i = threadIdx.x; i < width8; i += blockDim.x)
    dst[(size_t)b * width8 + i] = src[((size_t)b * T + T - 1) * width8 + i];
}

// pos[b] += T
__global__ void advance_pos_kernel(int* pos, int batch, int T) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  pdl_wait();
  pdl_launch();
  if (b < batch) pos[b] += T;
}

}  // namespace

Status launch_dn_prefill_conv(const void* proj, int ld, int batch, int T, int H, const void* conv_w,
                              const void* conv_old, void* conv_new, const float* a_log_bias, void* q, void* k, void* v,
                              float* g, float* beta, cudaStream_t st) {
  const dim3 grid(3 * H, batch, (T + kTokTile - 1) / kTokTile);
  launch_k(dn_prefill_conv_kernel, grid, dim3(kDim), 0, st, (const __half*)proj, ld, T, H, (const uint16_t*)conv_w,
           (const uint16_t*)conv_old, (uint16_t*)conv_new, a_log_bias, (__half*)q, (__half*)k, (__half*)v, g, beta);
  SPOCK_LAUNCH_CHECK("dn_prefill_conv_kernel");
  return Status::ok();
}

Status launch_dn_prefill_gate(const float* core, const void* proj, int ld, int z_off, const float* norm_w, float eps,
                              int batch, int T, int H, void* out, cudaStream_t st) {
  launch_k(dn_prefill_gate_kernel, dim3((batch * T * H + 7) / 8), dim3(256), 0, st, core, (const __half*)proj, ld,
           z_off, norm_w, eps, T, H, batch * T, (__half*)out);
  SPOCK_LAUNCH_CHECK("dn_prefill_gate_kernel");
  return Status::ok();
}

Status launch_last_rows(const void* src, void* dst, int batch, int T, int width, cudaStream_t st) {
  launch_k(last_rows_kernel, dim3(batch), dim3(128), 0, st, (const uint4*)src, (uint4*)dst, T, width / 8);
  SPOCK_LAUNCH_CHECK("last_rows_kernel");
  return Status::ok();
}

Status launch_advance_pos(int* pos, int batch, int T, cudaStream_t st) {
  launch_k(advance_pos_kernel, dim3((batch + 127) / 128), dim3(128), 0, st, pos, batch, T);
  SPOCK_LAUNCH_CHECK("advance_pos_kernel");
  return Status::ok();
}

}  // namespace spock
