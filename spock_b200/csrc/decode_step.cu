// Fused single-token Gated DeltaNet decode step for sm_100a.
//
// One CTA per (sequence, head); 256 threads = 8 warps. The head's 128x128 fp32
// state (64 KiB) is streamed HBM -> registers once with coalesced 128-bit
// loads (warp w owns rows 16w..16w+15, lane l owns columns 4l..4l+3), updated
// in registers and streamed back once: 2 x 64 KiB of HBM traffic per head per
// token, the algorithmic minimum. The reference shader reads the state 3x and
// writes it 2x (deltanet_recurrent_gbeta_norm_gate.comp:243-291).
//
// The state loads are issued first, so the causal-conv + SiLU + L2 prologue
// (deltanet_conv_l2_qk.comp:48-110), restricted to this head's 3x128
// channels, and the g/beta computation (deltanet_recurrent_gbeta_norm_gate
// .comp:212-227) overlap the loads in flight.
//
// Numerics follow the shaders: fp16 storage of the conv output before the L2
// pass, the shaders' stride-64..1 tree for 128-wide sums of squares, per-
// element state updates as a separate rounded multiply and add
// (S*=e^g; S+=k*delta), RMSNorm as x*(1/sqrt(mean+eps)), w*norm rounded to fp16
// before the SiLU gate. Reductions over the key dimension are split 16 rows
// per warp and then summed over the 8 warps (the shader sums rows in order).
#include "common.cuh"

namespace spock {
namespace {

constexpr int kDim = 128;      // key_dim == value_dim on this path
constexpr int kThreads = 256;  // 8 warps x 16 state rows
constexpr int kRowsPerWarp = 16;

// Pairwise tree over s[0..127] (the shaders' stride 64..1 loop); all 256
// threads call it; returns the total to every thread.
__device__ __forceinline__ float tree128(float* s) {
  for (int stride = 64; stride > 0; stride >>= 1) {
    if (threadIdx.x < stride) s[threadIdx.x] += s[threadIdx.x + stride];
    __syncthreads();
  }
  return s[0];
}

template <bool kFused>
__global__ void __launch_bounds__(kThreads, 2)
    dn_decode_kernel(int H, float q_scale, float eps, uint16_t* __restrict__ qkv,
                     uint16_t* __restrict__ conv_state, const uint16_t* __restrict__ conv_w,
                     const float* __restrict__ a_log_bias, const float* __restrict__ norm_w,
                     const uint16_t* __restrict__ a_in, const uint16_t* __restrict__ b_in,
                     const uint16_t* __restrict__ z_in, const uint16_t* __restrict__ q_raw,
                     const uint16_t* __restrict__ k_raw, const uint16_t* __restrict__ v_raw,
                     const float* __restrict__ g_in, const float* __restrict__ beta_in,
                     float* __restrict__ state, uint16_t* __restrict__ out,
                     uint16_t* __restrict__ core_raw, int qkv_ld, int ab_ld, int z_ld, int out_ld) {
  const int h = blockIdx.x;
  const int s = blockIdx.y;
  const int t = threadIdx.x;
  const int warp = t >> 5, lane = t & 31;

  __shared__ float sq[kDim], sk[kDim], sv[kDim];
  __shared__ float red[kThreads / 32][kDim];
  __shared__ float tq[kDim], tk[kDim];
  __shared__ float sdelta[kDim];
  __shared__ float s_g, s_beta;

  // 1. Issue the state loads (16 x 16 B per thread) before anything else.
  float4* S4 = reinterpret_cast<float4*>(state + ((size_t)s * H + h) * kDim * kDim);
  float4 S[kRowsPerWarp];
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) S[r] = S4[(warp * kRowsPerWarp + r) * (kDim / 4) + lane];

  // 2. Prologue: q, k, v for this head, g and beta.
  if constexpr (kFused) {
    const int conv_dim = H * 3 * kDim;
    uint16_t* x = qkv + (size_t)s * qkv_ld;
    uint16_t* cs = conv_state + (size_t)s * conv_dim * 4;
    for (int c = t; c < 3 * kDim; c += kThreads) {
      const int blk = c / kDim, off = c % kDim;
      const int ch = blk * H * kDim + h * kDim + off;
      uint2 st = *reinterpret_cast<const uint2*>(cs + (size_t)ch * 4);
      const uint2 wv = *reinterpret_cast<const uint2*>(conv_w + (size_t)ch * 4);
      const uint16_t xin = x[ch];
      // shift left by one slot, insert the new value at the end
      const uint16_t s0 = (uint16_t)(st.x >> 16), s1 = (uint16_t)(st.y & 0xffff),
                     s2 = (uint16_t)(st.y >> 16), s3 = xin;
      st.x = (uint32_t)s0 | ((uint32_t)s1 << 16);
      st.y = (uint32_t)s2 | ((uint32_t)s3 << 16);
      *reinterpret_cast<uint2*>(cs + (size_t)ch * 4) = st;
      float sum = 0.f;
      sum = add_rn(sum, mul_rn(h2f(s0), h2f((uint16_t)(wv.x & 0xffff))));
      sum = add_rn(sum, mul_rn(h2f(s1), h2f((uint16_t)(wv.x >> 16))));
      sum = add_rn(sum, mul_rn(h2f(s2), h2f((uint16_t)(wv.y & 0xffff))));
      sum = add_rn(sum, mul_rn(h2f(s3), h2f((uint16_t)(wv.y >> 16))));
      const float silu = __fdiv_rn(sum, add_rn(1.0f, expf(-sum)));
      const uint16_t y = f2h(silu);
      const float yf = h2f(y);
      if (blk == 0) {
        sq[off] = yf;
        tq[off] = mul_rn(yf, yf);
      } else if (blk == 1) {
        sk[off] = yf;
        tk[off] = mul_rn(yf, yf);
      } else {
        sv[off] = yf;
        x[ch] = y;
      }
    }
    if (t == 0) {
      const float a_val = h2f(a_in[(size_t)s * ab_ld + h]);
      const float b_val = h2f(b_in[(size_t)s * ab_ld + h]);
      const float a_log = a_log_bias[h * 2 + 0], dt_bias = a_log_bias[h * 2 + 1];
      const float sp = logf(add_rn(1.0f, expf(add_rn(a_val, dt_bias))));
      s_g = mul_rn(-expf(a_log), sp);
      s_beta = __fdiv_rn(1.0f, add_rn(1.0f, expf(-b_val)));
    }
    __syncthreads();
    // L2 of the Q and K blocks (two trees side by side)
    for (int stride = 64; stride > 0; stride >>= 1) {
      if (t < stride) tq[t] += tq[t + stride];
      else if (t >= 128 && t - 128 < stride) tk[t - 128] += tk[t - 128 + stride];
      __syncthreads();
    }
    if (t < kDim) {
      const float inv = __fdiv_rn(1.0f, __fsqrt_rn(add_rn(tq[0], 1e-6f)));
      const uint16_t qn = f2h(mul_rn(sq[t], inv));
      x[h * kDim + t] = qn;
      sq[t] = mul_rn(h2f(qn), q_scale);
    } else {
      const int j = t - kDim;
      const float inv = __fdiv_rn(1.0f, __fsqrt_rn(add_rn(tk[0], 1e-6f)));
      const uint16_t kn = f2h(mul_rn(sk[j], inv));
      x[H * kDim + h * kDim + j] = kn;
      sk[j] = h2f(kn);
    }
  } else {
    if (t < kDim) {
      const size_t base = ((size_t)s * H + h) * kDim + t;
      sq[t] = mul_rn(h2f(q_raw[base]), q_scale);
      sk[t] = h2f(k_raw[base]);
      sv[t] = h2f(v_raw[base]);
    }
    if (t == 0) {
      s_g = g_in[(size_t)s * H + h];
      s_beta = beta_in[(size_t)s * H + h];
    }
  }
  __syncthreads();

  // 3. Recurrent update in registers.
  const float eg = expf(s_g);
  const float beta = s_beta;
  float4 kv = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) {
    const float ki = sk[warp * kRowsPerWarp + r];
    S[r].x = mul_rn(S[r].x, eg);
    S[r].y = mul_rn(S[r].y, eg);
    S[r].z = mul_rn(S[r].z, eg);
    S[r].w = mul_rn(S[r].w, eg);
    kv.x = fmaf(S[r].x, ki, kv.x);
    kv.y = fmaf(S[r].y, ki, kv.y);
    kv.z = fmaf(S[r].z, ki, kv.z);
    kv.w = fmaf(S[r].w, ki, kv.w);
  }
  *reinterpret_cast<float4*>(&red[warp][lane * 4]) = kv;
  __syncthreads();
  if (t < kDim) {
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) acc += red[w][t];
    sdelta[t] = mul_rn(sv[t] - acc, beta);
  }
  __syncthreads();
  const float4 d4 = *reinterpret_cast<const float4*>(&sdelta[lane * 4]);
  float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) {
    const float ki = sk[warp * kRowsPerWarp + r];
    const float qi = sq[warp * kRowsPerWarp + r];
    S[r].x = add_rn(S[r].x, mul_rn(ki, d4.x));
    S[r].y = add_rn(S[r].y, mul_rn(ki, d4.y));
    S[r].z = add_rn(S[r].z, mul_rn(ki, d4.z));
    S[r].w = add_rn(S[r].w, mul_rn(ki, d4.w));
    o.x = fmaf(S[r].x, qi, o.x);
    o.y = fmaf(S[r].y, qi, o.y);
    o.z = fmaf(S[r].z, qi, o.z);
    o.w = fmaf(S[r].w, qi, o.w);
    S4[(warp * kRowsPerWarp + r) * (kDim / 4) + lane] = S[r];
  }
  *reinterpret_cast<float4*>(&red[warp][lane * 4]) = o;
  __syncthreads();
  float ov = 0.f;
  if (t < kDim) {
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) ov += red[w][t];
    tq[t] = mul_rn(ov, ov);
    if (core_raw) core_raw[((size_t)s * H + h) * kDim + t] = f2h(ov);
  }
  __syncthreads();
  if constexpr (!kFused) return;

  // 4. Gated RMSNorm: fp16(w * norm(o)) * SiLU(z) -> fp16.
  const float ss = tree128(tq);
  if (t < kDim) {
    const float nf = __fdiv_rn(1.0f, __fsqrt_rn(add_rn(__fdiv_rn(ss, (float)kDim), eps)));
    const float normed = mul_rn(ov, nf);
    const float zz = h2f(z_in[(size_t)s * z_ld + h * kDim + t]);
    const float silu = __fdiv_rn(zz, add_rn(1.0f, expf(-zz)));
    const float weighted = h2f(f2h(mul_rn(norm_w[t], normed)));
    out[(size_t)s * out_ld + h * kDim + t] = f2h(mul_rn(weighted, silu));
  }
}

}  // namespace

Status launch_decode_step_strided(const spock_dn_layer& L, int64_t batch, void* qkv, int qkv_ld,
                                  void* conv_state, float* state, const void* a, const void* b, int ab_ld,
                                  const void* z, int z_ld, void* out, int out_ld, void* core_raw,
                                  cudaStream_t stream) {
  if (L.key_dim != kDim || L.value_dim != kDim || L.conv_kernel != 4)
    return Status::err(SPOCK_ERR_UNSUPPORTED,
                       "decode step: CUDA path implements key_dim=value_dim=128, conv_kernel=4");
  if (L.num_heads <= 0 || L.num_heads > 65535 || batch <= 0 || batch > 65535)
    return Status::err(SPOCK_ERR_INVALID, "decode step: num_heads and batch must be in [1, 65535]");
  if (((uintptr_t)state & 15) || ((uintptr_t)conv_state & 7) || ((uintptr_t)L.conv_weight & 7))
    return Status::err(SPOCK_ERR_INVALID,
                       "decode step: state must be 16-byte aligned, conv_state/conv_weight 8-byte aligned");
  dim3 grid((unsigned)L.num_heads, (unsigned)batch);
  dn_decode_kernel<true><<<grid, kThreads, 0, stream>>>(
      L.num_heads, 1.0f / sqrtf((float)kDim), L.eps, (uint16_t*)qkv, (uint16_t*)conv_state,
      (const uint16_t*)L.conv_weight, L.a_log_bias, L.norm_weight, (const uint16_t*)a,
      (const uint16_t*)b, (const uint16_t*)z, nullptr, nullptr, nullptr, nullptr, nullptr, state,
      (uint16_t*)out, (uint16_t*)core_raw, qkv_ld, ab_ld, z_ld, out_ld);
  SPOCK_LAUNCH_CHECK("dn_decode_kernel<fused>");
  return Status::ok();
}

Status launch_decode_step(const spock_dn_layer& L, int64_t batch, void* qkv, void* conv_state,
                          float* state, const void* a, const void* b, const void* z, void* out,
                          void* core_raw, cudaStream_t stream) {
  const int conv_dim = L.num_heads * (L.key_dim * 2 + L.value_dim);
  return launch_decode_step_strided(L, batch, qkv, conv_dim, conv_state, state, a, b, L.num_heads, z,
                                    L.num_heads * L.value_dim, out, L.num_heads * L.value_dim, core_raw,
                                    stream);
}

Status launch_recurrent(int64_t batch, int H, int kd, int vd, const void* q, const void* k,
                        const void* v, const float* g, const float* beta, float* state, void* out,
                        cudaStream_t stream) {
  if (kd != kDim || vd != kDim)
    return Status::err(SPOCK_ERR_UNSUPPORTED, "recurrent: CUDA path implements key_dim=value_dim=128");
  if (H <= 0 || H > 65535 || batch <= 0 || batch > 65535)
    return Status::err(SPOCK_ERR_INVALID, "recurrent: num_heads and batch must be in [1, 65535]");
  if ((uintptr_t)state & 15) return Status::err(SPOCK_ERR_INVALID, "recurrent: state must be 16-byte aligned");
  dim3 grid((unsigned)H, (unsigned)batch);
  dn_decode_kernel<false><<<grid, kThreads, 0, stream>>>(
      H, 1.0f / sqrtf((float)kDim), 0.f, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
      nullptr, nullptr, (const uint16_t*)q, (const uint16_t*)k, (const uint16_t*)v, g, beta, state,
      nullptr, (uint16_t*)out, 0, 0, 0, 0);
  SPOCK_LAUNCH_CHECK("dn_decode_kernel<raw>");
  return Status::ok();
}

}  // namespace spock
