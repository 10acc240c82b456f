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
#include "tc.cuh"

namespace spock {
namespace {

constexpr int kDim = 128;      // key_dim == value_dim on this path
constexpr int kThreads = 256;  // 8 warps x 16 state rows
constexpr int kRowsPerWarp = 16;
constexpr int kStages = 3;                   // state ring of the streaming kernel
constexpr uint32_t kStateBytes = kDim * kDim * 4;
constexpr uint32_t kWaitLimit = 1u << 22;    // polls of a ~µs-scale try_wait: seconds

struct Args {
  int H;
  float q_scale, eps;
  uint16_t* qkv;
  uint16_t* conv_state;
  const uint16_t* conv_w;
  const float* a_log_bias;
  const float* norm_w;
  const uint16_t *a_in, *b_in, *z_in, *q_raw, *k_raw, *v_raw;
  const float *g_in, *beta_in;
  float* state;
  uint16_t* out;
  uint16_t* core_raw;
  int qkv_ld, ab_ld, z_ld, out_ld;
};

struct __align__(16) Smem {  // float4 access to red and sdelta
  float sq[kDim], sk[kDim], sv[kDim];
  float red[kThreads / 32][kDim];
  float tq[kDim], tk[kDim];
  float sdelta[kDim];
  float g, beta;
  float qss, kss, oss;  // sums of squares of q, k (L2) and of the output (RMSNorm)
};

// The shaders' pairwise tree over s[0..127] (s[i] += s[i + stride] for
// stride 64, 32, ..., 1) by one warp with the same additions in the same
// order: lane l holds s[l], s[l+32], s[l+64], s[l+96]. Total in lane 0.
__device__ __forceinline__ float warp_tree128(const float* s, int lane) {
  float v0 = s[lane], v1 = s[lane + 32];
  v0 += s[lane + 64];
  v1 += s[lane + 96];
  v0 += v1;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v0 += __shfl_down_sync(0xffffffffu, v0, o);
  return v0;
}

// Global inputs of the fused prologue for one thread: its conv channels
// c = t and c = t + 256 (threads 0..127 have two), and a, b for the last thread.
constexpr int kPer = (3 * kDim + kThreads - 1) / kThreads;
struct PIn {
  uint2 st[kPer], wv[kPer];
  uint16_t xin[kPer];
  float a_val, b_val;
};

template <bool kFused>
__device__ __forceinline__ PIn prologue_load(const Args& A, int s, int h, int t) {
  PIn in{};
  if constexpr (kFused) {
    const int H = A.H;
    const uint16_t* x = A.qkv + (size_t)s * A.qkv_ld;
    const uint16_t* cs = A.conv_state + (size_t)s * H * 3 * kDim * 4;
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      const int c = t + u * kThreads;
      if (c < 3 * kDim) {
        const int ch = (c / kDim) * H * kDim + h * kDim + c % kDim;
        in.st[u] = *reinterpret_cast<const uint2*>(cs + (size_t)ch * 4);
        in.wv[u] = *reinterpret_cast<const uint2*>(A.conv_w + (size_t)ch * 4);
        in.xin[u] = x[ch];
      }
    }
    if (t == kThreads - 1) {  // a thread with a single conv channel
      in.a_val = h2f(A.a_in[(size_t)s * A.ab_ld + h]);
      in.b_val = h2f(A.b_in[(size_t)s * A.ab_ld + h]);
    }
  }
  return in;
}

// q, k, v of head h of sequence s (scaled q in sq), g and beta -> shared memory.
// Fused: causal conv + SiLU + L2 from the raw qkv token and the conv cache
// (their global inputs already in `in`).
template <bool kFused, class Sync>
__device__ __forceinline__ void prologue(const Args& A, Smem& m, int s, int h, int t, Sync sync, const PIn& in) {
  const int H = A.H;
  if constexpr (kFused) {
    const int conv_dim = H * 3 * kDim;
    uint16_t* x = A.qkv + (size_t)s * A.qkv_ld;
    uint16_t* cs = A.conv_state + (size_t)s * conv_dim * 4;
    if (t == kThreads - 1) {
      const float a_log = A.a_log_bias[h * 2 + 0], dt_bias = A.a_log_bias[h * 2 + 1];
      const float sp = logf(add_rn(1.0f, expf(add_rn(in.a_val, dt_bias))));
      m.g = mul_rn(-expf(a_log), sp);
      m.beta = __fdiv_rn(1.0f, add_rn(1.0f, expf(-in.b_val)));
    }
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      const int c = t + u * kThreads;
      if (c >= 3 * kDim) continue;
      const int blk = c / kDim, off = c % kDim;
      const int ch = blk * H * kDim + h * kDim + off;
      uint2 st = in.st[u];
      const uint2 wv = in.wv[u];
      const uint16_t xin = in.xin[u];
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
        m.sq[off] = yf;
        m.tq[off] = mul_rn(yf, yf);
      } else if (blk == 1) {
        m.sk[off] = yf;
        m.tk[off] = mul_rn(yf, yf);
      } else {
        m.sv[off] = yf;
        x[ch] = y;
      }
    }
    sync();
    // L2 of the Q and K blocks: warp 0 and warp 1 run the two trees
    if (t < 64) {
      const float tot = warp_tree128(t < 32 ? m.tq : m.tk, t & 31);
      if (t == 0) m.qss = tot;
      if (t == 32) m.kss = tot;
    }
    sync();
    if (t < kDim) {
      const float inv = __fdiv_rn(1.0f, __fsqrt_rn(add_rn(m.qss, 1e-6f)));
      const uint16_t qn = f2h(mul_rn(m.sq[t], inv));
      x[h * kDim + t] = qn;
      m.sq[t] = mul_rn(h2f(qn), A.q_scale);
    } else {
      const int j = t - kDim;
      const float inv = __fdiv_rn(1.0f, __fsqrt_rn(add_rn(m.kss, 1e-6f)));
      const uint16_t kn = f2h(mul_rn(m.sk[j], inv));
      x[H * kDim + h * kDim + j] = kn;
      m.sk[j] = h2f(kn);
    }
  } else {
    if (t < kDim) {
      const size_t base = ((size_t)s * H + h) * kDim + t;
      m.sq[t] = mul_rn(h2f(A.q_raw[base]), A.q_scale);
      m.sk[t] = h2f(A.k_raw[base]);
      m.sv[t] = h2f(A.v_raw[base]);
    }
    if (t == 0) {
      m.g = A.g_in[(size_t)s * H + h];
      m.beta = A.beta_in[(size_t)s * H + h];
    }
  }
  sync();
}

// Recurrent update of the head's state held in registers (warp w: rows
// 16w..16w+15, lane l: columns 4l..4l+3), streamed back to S4; then the
// gated RMSNorm output. All 256 threads.
template <bool kFused, class Sync>
__device__ __forceinline__ void update_and_output(const Args& A, Smem& m, float4 (&S)[kRowsPerWarp],
                                                  float4* __restrict__ S4, int s, int h, int t, Sync sync) {
  const int warp = t >> 5, lane = t & 31, H = A.H;
  float zz = 0.f;  // gate input, loaded early so its latency hides behind the update
  if (kFused && t < kDim) zz = h2f(A.z_in[(size_t)s * A.z_ld + h * kDim + t]);
  const float eg = expf(m.g);
  const float beta = m.beta;
  float4 kv = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) {
    const float ki = m.sk[warp * kRowsPerWarp + r];
    S[r].x = mul_rn(S[r].x, eg);
    S[r].y = mul_rn(S[r].y, eg);
    S[r].z = mul_rn(S[r].z, eg);
    S[r].w = mul_rn(S[r].w, eg);
    kv.x = fmaf(S[r].x, ki, kv.x);
    kv.y = fmaf(S[r].y, ki, kv.y);
    kv.z = fmaf(S[r].z, ki, kv.z);
    kv.w = fmaf(S[r].w, ki, kv.w);
  }
  *reinterpret_cast<float4*>(&m.red[warp][lane * 4]) = kv;
  sync();
  if (t < kDim) {
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) acc += m.red[w][t];
    m.sdelta[t] = mul_rn(m.sv[t] - acc, beta);
  }
  sync();
  const float4 d4 = *reinterpret_cast<const float4*>(&m.sdelta[lane * 4]);
  float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) {
    const float ki = m.sk[warp * kRowsPerWarp + r];
    const float qi = m.sq[warp * kRowsPerWarp + r];
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
  *reinterpret_cast<float4*>(&m.red[warp][lane * 4]) = o;
  sync();
  float ov = 0.f;
  if (t < kDim) {
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) ov += m.red[w][t];
    m.tq[t] = mul_rn(ov, ov);
    if (A.core_raw) A.core_raw[((size_t)s * H + h) * kDim + t] = f2h(ov);
  }
  sync();
  if constexpr (kFused) {
    // Gated RMSNorm: fp16(w * norm(o)) * SiLU(z) -> fp16.
    if (t < 32) {
      const float tot = warp_tree128(m.tq, t);
      if (t == 0) m.oss = tot;
    }
    sync();
    if (t < kDim) {
      const float nf = __fdiv_rn(1.0f, __fsqrt_rn(add_rn(__fdiv_rn(m.oss, (float)kDim), A.eps)));
      const float normed = mul_rn(ov, nf);
      const float silu = __fdiv_rn(zz, add_rn(1.0f, expf(-zz)));
      const float weighted = h2f(f2h(mul_rn(A.norm_w[t], normed)));
      A.out[(size_t)s * A.out_ld + h * kDim + t] = f2h(mul_rn(weighted, silu));
    }
  }
}

// One CTA per (head, sequence): the state loads are issued first, so the
// conv/L2 prologue overlaps them. Used when there are too few heads to keep
// every SM streaming.
template <bool kFused>
__global__ void __launch_bounds__(kThreads, 2) dn_decode_kernel(const __grid_constant__ Args A) {
  __shared__ Smem m;
  const int h = blockIdx.x, s = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float4* S4 = reinterpret_cast<float4*>(A.state + ((size_t)s * A.H + h) * kDim * kDim);
  float4 S[kRowsPerWarp];
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) S[r] = S4[(warp * kRowsPerWarp + r) * (kDim / 4) + lane];
  pdl_wait();  // the state was last written by an earlier step; the token's inputs come from the predecessor
  pdl_launch();
  auto sync = [] { __syncthreads(); };
  prologue<kFused>(A, m, s, h, threadIdx.x, sync, prologue_load<kFused>(A, s, h, threadIdx.x));
  update_and_output<kFused>(A, m, S, S4, s, h, threadIdx.x, sync);
}

// Persistent streaming variant, one CTA (two 256-thread groups) per SM. The
// CTA walks its (sequence, head) items j = 0, 1, 2, ... (global index
// blockIdx.x + j*gridDim.x); group j&1 runs item j exactly as dn_decode_kernel
// does, so the two groups' prologues, barriers and stores overlap. Each item's
// 64 KiB state arrives in a 3-slot shared-memory ring by bulk copies issued
// three items ahead, so HBM keeps streaming. A ring wait that gives up sets
// *err; the group then lets the copies it issued land (bounded) and leaves.
template <bool kFused>
__global__ void __launch_bounds__(2 * kThreads, 1)
    dn_decode_stream_kernel(const __grid_constant__ Args A, int items, int* __restrict__ err) {
  extern __shared__ __align__(128) uint8_t ring_raw[];
  float* ring = reinterpret_cast<float*>(ring_raw);
  __shared__ Smem msm[2];
  __shared__ uint64_t full[kStages];
  const int grp = threadIdx.x >> 8, t = threadIdx.x & (kThreads - 1), warp = t >> 5, lane = t & 31;
  Smem& m = msm[grp];
  const int G = gridDim.x;
  const int mine = items > (int)blockIdx.x ? (items - 1 - (int)blockIdx.x) / G + 1 : 0;
  auto src = [&](int j) {  // items are (sequence, head) in memory order
    return A.state + (size_t)((int)blockIdx.x + j * G) * kDim * kDim;
  };
  auto issue = [&](int j) {
    const int b = j % kStages;
    tc::mbar_arrive_expect_tx(&full[b], kStateBytes);
#pragma unroll
    for (int q = 0; q < 4; ++q)
      tc::bulk_load(ring + b * kDim * kDim + q * 4096, src(j) + q * 4096, kStateBytes / 4, &full[b]);
  };
  if (threadIdx.x == 0) {
    for (int b = 0; b < kStages; ++b) tc::mbar_init(&full[b], 1);
    tc::fence_mbar_init();
    for (int j = 0; j < kStages && j < mine; ++j) issue(j);
  }
  pdl_wait();  // the states were last written by an earlier step: their copies start before this
  pdl_launch();
  __syncthreads();
  const int bar_id = 1 + grp;
  auto sync = [bar_id] { asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(kThreads) : "memory"); };
  auto coord = [&](int j, int& s, int& h) {
    const int it = (int)blockIdx.x + j * G;
    s = it / A.H;
    h = it % A.H;
  };
  PIn nxt{};
  if (grp < mine) {
    int s0, h0;
    coord(grp, s0, h0);
    nxt = prologue_load<kFused>(A, s0, h0, t);
  }
  for (int j = grp; j < mine; j += 2) {
    int s, h;
    coord(j, s, h);
    const int b = j % kStages;
    const PIn cur = nxt;
    if (j + 2 < mine) {  // the group's next item: its loads fly during this item
      int s2, h2;
      coord(j + 2, s2, h2);
      nxt = prologue_load<kFused>(A, s2, h2, t);
    }
    prologue<kFused>(A, m, s, h, t, sync, cur);
    const bool ok = tc::mbar_wait_bounded(&full[b], (uint32_t)(j / kStages) & 1u, kWaitLimit);
    uint32_t any;
    asm volatile("{\n .reg .pred p, q;\n setp.ne.u32 q, %1, 0;\n bar.red.or.pred p, %2, %3, q;\n selp.u32 %0, 1, 0, p;\n}"
                 : "=r"(any) : "r"((uint32_t)!ok), "r"(bar_id), "r"(kThreads) : "memory");
    if (any) {
      if (t == 0) {
        atomicExch(err, 2);
        // this group issued the copies of items j+1 .. j+kStages-1 (at most)
        for (int k = j + 1; k < j + kStages && k < mine; ++k)
          tc::mbar_wait_bounded(&full[k % kStages], (uint32_t)(k / kStages) & 1u, kWaitLimit);
      }
      return;
    }
    const float4* R = reinterpret_cast<const float4*>(ring + b * kDim * kDim);
    float4 S[kRowsPerWarp];
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r) S[r] = R[(warp * kRowsPerWarp + r) * (kDim / 4) + lane];
    sync();  // the group has read slot b: it may be refilled
    if (t == 0 && j + kStages < mine) {
      tc::fence_async_smem();
      issue(j + kStages);
    }
    update_and_output<kFused>(A, m, S, reinterpret_cast<float4*>(src(j)), s, h, t, sync);
  }
}

// Failure-detection self-test: the bounded mbarrier wait of the kernels above
// on a barrier that never completes. It gives up after `polls` polls, records
// code 5 in *err and returns; nothing faults.
__global__ void wait_timeout_selftest_kernel(uint32_t polls, int* err) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, 1);
    tc::fence_mbar_init();
  }
  __syncthreads();
  const bool ok = tc::mbar_wait_bounded(&bar, 0, polls);
  if (__syncthreads_or(!ok) && threadIdx.x == 0) atomicExch(err, 5);
}

Args make_args(int H, float eps) {
  Args a{};
  a.H = H;
  a.q_scale = 1.0f / sqrtf((float)kDim);
  a.eps = eps;
  return a;
}

// Streams when there are at least two items per SM; below that one CTA per
// item issues all of its loads at once.
template <bool kFused>
Status launch(const Args& A, int64_t batch, int* err, cudaStream_t stream) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t items = batch * A.H;
  if (err && items >= 2 * (int64_t)sms && items <= 0x7fffffff) {
    const int smem = kStages * (int)kStateBytes;
    auto kern = dn_decode_stream_kernel<kFused>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return cuda_status(e, "dn_decode_stream_kernel smem attribute");
    launch_k(kern, dim3((unsigned)sms), dim3(2 * kThreads), smem, stream, A, (int)items, err);
    SPOCK_LAUNCH_CHECK(kFused ? "dn_decode_stream_kernel<fused>" : "dn_decode_stream_kernel<raw>");
    return Status::ok();
  }
  dim3 grid((unsigned)A.H, (unsigned)batch);
  launch_k(dn_decode_kernel<kFused>, grid, dim3(kThreads), 0, stream, A);
  SPOCK_LAUNCH_CHECK(kFused ? "dn_decode_kernel<fused>" : "dn_decode_kernel<raw>");
  return Status::ok();
}

}  // namespace

Status launch_wait_timeout_selftest(uint32_t polls, int* err, cudaStream_t stream) {
  wait_timeout_selftest_kernel<<<1, 32, 0, stream>>>(polls, err);
  SPOCK_LAUNCH_CHECK("wait_timeout_selftest_kernel");
  return Status::ok();
}

Status launch_decode_step_strided(const spock_dn_layer& L, int64_t batch, void* qkv, int qkv_ld,
                                  void* conv_state, float* state, const void* a, const void* b, int ab_ld,
                                  const void* z, int z_ld, void* out, int out_ld, void* core_raw, int* err,
                                  cudaStream_t stream) {
  if (L.key_dim != kDim || L.value_dim != kDim || L.conv_kernel != 4)
    return Status::err(SPOCK_ERR_UNSUPPORTED,
                       "decode step: CUDA path implements key_dim=value_dim=128, conv_kernel=4");
  if (L.num_heads <= 0 || L.num_heads > 65535 || batch <= 0 || batch > 65535)
    return Status::err(SPOCK_ERR_INVALID, "decode step: num_heads and batch must be in [1, 65535]");
  if (((uintptr_t)state & 15) || ((uintptr_t)conv_state & 7) || ((uintptr_t)L.conv_weight & 7))
    return Status::err(SPOCK_ERR_INVALID,
                       "decode step: state must be 16-byte aligned, conv_state/conv_weight 8-byte aligned");
  Args A = make_args(L.num_heads, L.eps);
  A.qkv = (uint16_t*)qkv;
  A.conv_state = (uint16_t*)conv_state;
  A.conv_w = (const uint16_t*)L.conv_weight;
  A.a_log_bias = L.a_log_bias;
  A.norm_w = L.norm_weight;
  A.a_in = (const uint16_t*)a;
  A.b_in = (const uint16_t*)b;
  A.z_in = (const uint16_t*)z;
  A.state = state;
  A.out = (uint16_t*)out;
  A.core_raw = (uint16_t*)core_raw;
  A.qkv_ld = qkv_ld;
  A.ab_ld = ab_ld;
  A.z_ld = z_ld;
  A.out_ld = out_ld;
  return launch<true>(A, batch, err, stream);
}

Status launch_decode_step(const spock_dn_layer& L, int64_t batch, void* qkv, void* conv_state,
                          float* state, const void* a, const void* b, const void* z, void* out,
                          void* core_raw, int* err, cudaStream_t stream) {
  const int conv_dim = L.num_heads * (L.key_dim * 2 + L.value_dim);
  return launch_decode_step_strided(L, batch, qkv, conv_dim, conv_state, state, a, b, L.num_heads, z,
                                    L.num_heads * L.value_dim, out, L.num_heads * L.value_dim, core_raw, err,
                                    stream);
}

Status launch_recurrent(int64_t batch, int H, int kd, int vd, const void* q, const void* k,
                        const void* v, const float* g, const float* beta, float* state, void* out, int* err,
                        cudaStream_t stream) {
  if (kd != kDim || vd != kDim)
    return Status::err(SPOCK_ERR_UNSUPPORTED, "recurrent: CUDA path implements key_dim=value_dim=128");
  if (H <= 0 || H > 65535 || batch <= 0 || batch > 65535)
    return Status::err(SPOCK_ERR_INVALID, "recurrent: num_heads and batch must be in [1, 65535]");
  if ((uintptr_t)state & 15) return Status::err(SPOCK_ERR_INVALID, "recurrent: state must be 16-byte aligned");
  Args A = make_args(H, 0.f);
  A.q_raw = (const uint16_t*)q;
  A.k_raw = (const uint16_t*)k;
  A.v_raw = (const uint16_t*)v;
  A.g_in = g;
  A.beta_in = beta;
  A.state = state;
  A.core_raw = (uint16_t*)out;
  return launch<false>(A, batch, err, stream);
}

}  // namespace spock
