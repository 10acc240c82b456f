// Exact-order kernels of the full-model path (spock_model_desc.exact = 1).
//
// Greedy decoding is chaotic: one fp16 rounding that differs from the
// reference's changes later logits, and an argmax over 248320 fp16 logits
// meets near-ties often. These kernels therefore evaluate every reduction in
// the reference shaders' own order, so each fp16 storage point rounds exactly
// as the CPU restatement of those shaders does:
//   projections      matvec.comp:28-41: one sequential fp32 dot per output
//                    row over k = 0..K-1. The products of two fp16 values are
//                    exact in fp32, so fma(w, x, s) rounds exactly like the
//                    shader's separate multiply and add.
//   attention        attention_decode.comp:64-143 in two passes: scores
//                    (sequential over the head dim), max, exp, the sum and the
//                    weighted V accumulation each sequential over positions,
//                    then the sigmoid gate (sigmoid_gate.comp).
//   DeltaNet         deltanet_conv_l2_qk.comp:48-110 and
//                    deltanet_recurrent_gbeta_norm_gate.comp:91-224: one
//                    thread per value column with the column of the state in
//                    registers, sums over the key dim sequential, the
//                    shared-memory trees of the shaders for the norms.
// This file is compiled without floating-point contraction (--fmad=false):
// every a*b+c outside an explicit fmaf rounds twice, as in the shaders; the
// explicit fmaf calls are on exact fp16 x fp16 products only. exp and log are
// evaluated in double precision and rounded once to float (the definition
// the CPU restatement uses; GLSL leaves their precision to the
// implementation).
//
// Prefill runs layer-major like the fast path, but each DeltaNet layer walks
// its prompt tokens through the recurrence one by one (token-serial decode
// semantics), with the state resident in registers.
#include "common.cuh"
#include "gemm.h"

namespace spock {
namespace xk {
namespace {

constexpr int HID = 1024, DNH = 16, DND = 128, CONV = 6144;
constexpr int QH = 8, KVH = 2, HD = 256, G = QH / KVH;

__device__ __forceinline__ float exp_d(float x) { return (float)exp((double)x); }
__device__ __forceinline__ float log_d(float x) { return (float)log((double)x); }

__device__ __forceinline__ void h8_to_f(const uint4& u, float* f) {
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __half22float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

// ---- epilogues shared by both projection kernels ---------------------------
// value(s) of output row n for batch row b -> memory. EPI_SWIGLU gets the gate
// and up accumulators of one output pair p.
struct Epi {
  __half* y;
  int ldy;
  const __half* res;
};

__device__ __forceinline__ void store_f16(const Epi& e, int b, int n, float acc) {
  e.y[(size_t)b * e.ldy + n] = __float2half_rn(acc);
}
__device__ __forceinline__ void store_res(const Epi& e, int b, int n, float acc) {
  // residual_add.comp after the matvec's fp16 store: fp16(h + fp16(y))
  const float yv = __half2float(__float2half_rn(acc));
  const float hv = __half2float(e.res[(size_t)b * e.ldy + n]);
  e.y[(size_t)b * e.ldy + n] = __float2half_rn(hv + yv);
}
__device__ __forceinline__ void store_swiglu(const Epi& e, int b, int p, float ag, float au) {
  // silu_gate.comp on the two fp16 matvec outputs
  const float g = __half2float(__float2half_rn(ag));
  const float u = __half2float(__float2half_rn(au));
  e.y[(size_t)b * e.ldy + p] = __float2half_rn((g / (1.0f + exp_d(-g))) * u);
}

// ---- small-batch projection: one thread per weight row ----------------------
// x [R][K] fp16 (row stride ldx), W [N][K] fp16. Thread t of CTA c owns weight
// row c*128 + t (EPI_SWIGLU: output pair c*128 + t, i.e. gate row and up row of
// the 16-row interleave) and accumulates its R batch rows sequentially over k,
// streaming the row from HBM 32 bytes at a time, two steps ahead.
constexpr int kXC = 512;  // k chunk of x staged in shared memory (fp32)

template <int EPI, int R>
__global__ void __launch_bounds__(128) xgemv_kernel(const __half* __restrict__ x, int ldx,
                                                    const __half* __restrict__ W, int K, int N, int batch, Epi e,
                                                    float* __restrict__ amax_val, int* __restrict__ amax_idx) {
  constexpr int NR = EPI == EPI_SWIGLU ? 2 : 1;  // weight rows per thread
  __shared__ __align__(16) float xs[R][kXC];
  const int t = threadIdx.x;
  const int unit = blockIdx.x * 128 + t;  // output row, or output pair for SWIGLU
  const int n_units = EPI == EPI_SWIGLU ? N / 2 : N;
  const bool live = unit < n_units;
  int rows[NR];
  if constexpr (EPI == EPI_SWIGLU) {
    rows[0] = (unit >> 4) * 32 + (unit & 15);
    rows[NR - 1] = rows[0] + 16;
  } else {
    rows[0] = unit;
  }
  const uint4* wp[NR];
#pragma unroll
  for (int i = 0; i < NR; ++i) wp[i] = reinterpret_cast<const uint4*>(W + (size_t)(live ? rows[i] : 0) * K);
  const int steps = K / 16;  // 16 k per step: two 16-byte loads per row
  // three register stages (current, +1, +2): loads run two steps ahead.
  // Weights do not depend on the previous kernel: start streaming before the wait.
  uint4 cur[NR][2], nx1[NR][2], nx2[NR][2];
#pragma unroll
  for (int i = 0; i < NR; ++i) {
    cur[i][0] = __ldg(wp[i]);
    cur[i][1] = __ldg(wp[i] + 1);
    nx1[i][0] = __ldg(wp[i] + 2);
    nx1[i][1] = __ldg(wp[i] + 3);
  }
  pdl_wait();
  pdl_launch();
  float acc[NR][R];
#pragma unroll
  for (int i = 0; i < NR; ++i)
#pragma unroll
    for (int r = 0; r < R; ++r) acc[i][r] = 0.f;
  for (int s = 0; s < steps; ++s) {
    const int k0 = s * 16;
    if ((k0 % kXC) == 0) {
      __syncthreads();
      for (int j = t; j < R * kXC; j += 128) {
        const int r = j / kXC, kk = j % kXC;
        xs[r][kk] = (r < batch && k0 + kk < K) ? __half2float(x[(size_t)r * ldx + k0 + kk]) : 0.f;
      }
      __syncthreads();
    }
    if (s + 2 < steps) {
#pragma unroll
      for (int i = 0; i < NR; ++i) {
        nx2[i][0] = __ldg(wp[i] + 2 * (s + 2));
        nx2[i][1] = __ldg(wp[i] + 2 * (s + 2) + 1);
      }
    }
    const int kx = k0 % kXC;
#pragma unroll
    for (int i = 0; i < NR; ++i) {
      float w[16];
      h8_to_f(cur[i][0], w);
      h8_to_f(cur[i][1], w + 8);
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const float4* xr = reinterpret_cast<const float4*>(&xs[r][kx]);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 xv = xr[q];
          acc[i][r] = fmaf(w[4 * q], xv.x, acc[i][r]);
          acc[i][r] = fmaf(w[4 * q + 1], xv.y, acc[i][r]);
          acc[i][r] = fmaf(w[4 * q + 2], xv.z, acc[i][r]);
          acc[i][r] = fmaf(w[4 * q + 3], xv.w, acc[i][r]);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < NR; ++i) {
      cur[i][0] = nx1[i][0];
      cur[i][1] = nx1[i][1];
      nx1[i][0] = nx2[i][0];
      nx1[i][1] = nx2[i][1];
    }
  }
  if constexpr (EPI == EPI_ARGMAX) {
    // per batch row: fp16 logits of this CTA's 128 rows -> (max, lowest index)
    __shared__ float sv[4][R];
    __shared__ int si[4][R];
    const int warp = t >> 5, lane = t & 31;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float v = live ? __half2float(__float2half_rn(acc[0][r])) : -INFINITY;
      int idx = live ? unit : 0x7fffffff;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (ov > v || (ov == v && oi < idx)) {
          v = ov;
          idx = oi;
        }
      }
      if (lane == 0) {
        sv[warp][r] = v;
        si[warp][r] = idx;
      }
    }
    __syncthreads();
    if (t < R && t < batch) {
      float v = sv[0][t];
      int idx = si[0][t];
      for (int w = 1; w < 4; ++w)
        if (sv[w][t] > v || (sv[w][t] == v && si[w][t] < idx)) {
          v = sv[w][t];
          idx = si[w][t];
        }
      amax_val[(size_t)blockIdx.x * batch + t] = v;
      amax_idx[(size_t)blockIdx.x * batch + t] = idx;
    }
    return;
  }
  if (!live) return;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    if (r >= batch) break;
    if constexpr (EPI == EPI_F16) store_f16(e, r, unit, acc[0][r]);
    if constexpr (EPI == EPI_RESIDUAL) store_res(e, r, unit, acc[0][r]);
    if constexpr (EPI == EPI_SWIGLU) store_swiglu(e, r, unit, acc[0][r], acc[NR - 1][r]);
  }
}

// ---- small-batch projection, staged: one thread per weight row --------------
// The same per-row order as xgemv_kernel, but the weights reach shared memory
// through a ring of cp.async stages (kSt stages of 64 k for the CTA's rows,
// each 16-byte chunk loaded by consecutive threads, so every row's 128 bytes
// per stage arrive coalesced) and 64 threads per CTA keep twice as many CTAs
// per projection. Thread t still accumulates its row's dot over k in order;
// the row stride in shared memory (144 bytes) keeps the per-thread 16-byte
// reads of 8 consecutive rows on distinct banks.
constexpr int kRowB = 144;  // 128 bytes of a row's 64 k, padded

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <int EPI, int R, int kSt>
__global__ void __launch_bounds__(64) xgemv2_kernel(const __half* __restrict__ x, int ldx,
                                                    const __half* __restrict__ W, int K, int N, int batch, Epi e,
                                                    float* __restrict__ amax_val, int* __restrict__ amax_idx) {
  constexpr int NR = EPI == EPI_SWIGLU ? 2 : 1;
  constexpr int ROWS = 64 * NR;          // weight rows of this CTA
  constexpr int STAGE = ROWS * kRowB;    // bytes per ring stage
  extern __shared__ __align__(16) uint8_t xg_sm[];
  uint8_t* ring = xg_sm;
  float* xs = reinterpret_cast<float*>(xg_sm + kSt * STAGE);  // [R][kXC]
  const int t = threadIdx.x;
  const int unit = blockIdx.x * 64 + t;
  const int n_units = EPI == EPI_SWIGLU ? N / 2 : N;
  const bool live = unit < n_units;
  // weight row of CTA-local row r (SWIGLU: rows 0..63 gate, 64..127 up)
  auto wrow = [&](int r) {
    int u = blockIdx.x * 64 + (r & 63);
    if (u >= n_units) u = n_units - 1;  // clamped: loads stay in bounds, results unused
    if constexpr (EPI == EPI_SWIGLU) return (u >> 4) * 32 + (u & 15) + (r >= 64 ? 16 : 0);
    return u;
  };
  const int nst = K / 64;
  auto issue = [&](int s) {
    if (s < nst) {
      uint8_t* dst = ring + (s % kSt) * STAGE;
#pragma unroll
      for (int i = 0; i < ROWS * 8 / 64; ++i) {
        const int c = t + 64 * i, r = c >> 3, col = c & 7;
        cp_async16(dst + r * kRowB + col * 16, W + (size_t)wrow(r) * K + s * 64 + col * 8);
      }
    }
    cp_commit();
  };
#pragma unroll
  for (int s = 0; s < kSt - 1; ++s) issue(s);  // weights: before the dependency wait
  pdl_wait();
  pdl_launch();
  float acc[NR][R];
#pragma unroll
  for (int i = 0; i < NR; ++i)
#pragma unroll
    for (int r = 0; r < R; ++r) acc[i][r] = 0.f;
  for (int s = 0; s < nst; ++s) {
    cp_wait<kSt - 2>();
    __syncthreads();  // stage s landed for every thread; stage s-1 is no longer read
    issue(s + kSt - 1);
    const int k0 = s * 64;
    if ((k0 % kXC) == 0) {
      for (int j = t; j < R * kXC; j += 64) {
        const int r = j / kXC, kk = j % kXC;
        xs[r * kXC + kk] = (r < batch && k0 + kk < K) ? __half2float(x[(size_t)r * ldx + k0 + kk]) : 0.f;
      }
      __syncthreads();
    }
    const uint8_t* st = ring + (s % kSt) * STAGE;
    const int kx = k0 % kXC;
#pragma unroll
    for (int i = 0; i < NR; ++i) {
      const uint4* wr = reinterpret_cast<const uint4*>(st + (t + 64 * i) * kRowB);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        float w[8];
        h8_to_f(wr[c], w);
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const float4* xr = reinterpret_cast<const float4*>(xs + r * kXC + kx + c * 8);
          const float4 x0 = xr[0], x1 = xr[1];
          acc[i][r] = fmaf(w[0], x0.x, acc[i][r]);
          acc[i][r] = fmaf(w[1], x0.y, acc[i][r]);
          acc[i][r] = fmaf(w[2], x0.z, acc[i][r]);
          acc[i][r] = fmaf(w[3], x0.w, acc[i][r]);
          acc[i][r] = fmaf(w[4], x1.x, acc[i][r]);
          acc[i][r] = fmaf(w[5], x1.y, acc[i][r]);
          acc[i][r] = fmaf(w[6], x1.z, acc[i][r]);
          acc[i][r] = fmaf(w[7], x1.w, acc[i][r]);
        }
      }
    }
  }
  cp_wait<0>();
  static_assert(EPI != EPI_ARGMAX, "the LM head keeps xgemv_kernel: one argmax partial per 128-row tile");
  if (!live) return;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    if (r >= batch) break;
    if constexpr (EPI == EPI_F16) store_f16(e, r, unit, acc[0][r]);
    if constexpr (EPI == EPI_RESIDUAL) store_res(e, r, unit, acc[0][r]);
    if constexpr (EPI == EPI_SWIGLU) store_swiglu(e, r, unit, acc[0][r], acc[NR - 1][r]);
  }
}

// ---- batched projection: register-tiled, sequential k per output ------------
// CTA tile TN weight rows x (16*TB) batch rows, (TN/8) x 16 threads, each with
// 8 rows x TB batch columns. Thread (ty, tx) owns rows base..base+3 and
// base+16..base+19 with base = (ty/4)*32 + (ty%4)*4 (so the gate and up rows
// of one SWIGLU output pair sit in the same thread) and batch columns
// tx*TB..tx*TB+TB-1. k advances 16 at a time through double-buffered shared
// tiles (fp32, transposed: [k][row]); every output accumulates k in order
// 0..K-1. TN = 64 doubles the CTAs of the narrow (1024-output) projections.
constexpr int kTK = 16, kLDS = 132;

template <int EPI, int TN, int TB>
__global__ void __launch_bounds__(TN * 2) xgemm_kernel(const __half* __restrict__ x, int ldx,
                                                       const __half* __restrict__ W, int K, int N, int batch, Epi e,
                                                       float* __restrict__ amax_val, int* __restrict__ amax_idx) {
  constexpr int BT = 16 * TB;     // batch rows per CTA
  constexpr int NT = TN * 2;      // threads
  __shared__ __align__(16) float Ws[2][kTK][kLDS];
  __shared__ __align__(16) float Xs[2][kTK][kLDS];
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  const int n0 = blockIdx.x * TN, b0 = blockIdx.y * BT;
  const int base = (ty >> 2) * 32 + (ty & 3) * 4;
  // global -> register staging: W tile TN rows x 16 k (thread: row tid/2, k half tid%2);
  // X tile BT rows x 16 k in NT-thread passes
  constexpr int XP = (BT * 2 + NT - 1) / NT;
  const int lr = tid >> 1, lk = (tid & 1) * 8;
  const bool wl = n0 + lr < N;
  const __half* wsrc = W + (size_t)(wl ? n0 + lr : 0) * K + lk;
  const uint4 zero = make_uint4(0, 0, 0, 0);
  uint4 wr = wl ? __ldg(reinterpret_cast<const uint4*>(wsrc)) : zero;
  pdl_wait();
  pdl_launch();
  uint4 xr[XP];
  auto xload = [&](int kt) {
#pragma unroll
    for (int i = 0; i < XP; ++i) {
      const int c = tid + NT * i, row = c >> 1;
      const bool ok = c < BT * 2 && b0 + row < batch;
      xr[i] = ok ? *reinterpret_cast<const uint4*>(x + (size_t)(b0 + row) * ldx + kt * kTK + (c & 1) * 8) : zero;
    }
  };
  xload(0);
  auto stage = [&](int buf) {
    float f[8];
    h8_to_f(wr, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) Ws[buf][lk + i][lr] = f[i];
#pragma unroll
    for (int i = 0; i < XP; ++i) {
      const int c = tid + NT * i;
      if (c < BT * 2) {
        h8_to_f(xr[i], f);
#pragma unroll
        for (int q = 0; q < 8; ++q) Xs[buf][(c & 1) * 8 + q][c >> 1] = f[q];
      }
    }
  };
  stage(0);
  __syncthreads();
  float acc[8][TB];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < TB; ++j) acc[i][j] = 0.f;
  const int kt_n = K / kTK;
  for (int kt = 0; kt < kt_n; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < kt_n) {
      wr = wl ? __ldg(reinterpret_cast<const uint4*>(wsrc + (kt + 1) * kTK)) : zero;
      xload(kt + 1);
    }
#pragma unroll
    for (int kk = 0; kk < kTK; ++kk) {
      float a[8], bv[TB];
      const float4 a0 = *reinterpret_cast<const float4*>(&Ws[buf][kk][base]);
      const float4 a1 = *reinterpret_cast<const float4*>(&Ws[buf][kk][base + 16]);
      a[0] = a0.x, a[1] = a0.y, a[2] = a0.z, a[3] = a0.w;
      a[4] = a1.x, a[5] = a1.y, a[6] = a1.z, a[7] = a1.w;
#pragma unroll
      for (int j4 = 0; j4 < TB; j4 += 4) {
        const float4 b4 = *reinterpret_cast<const float4*>(&Xs[buf][kk][tx * TB + j4]);
        bv[j4] = b4.x, bv[j4 + 1] = b4.y, bv[j4 + 2] = b4.z, bv[j4 + 3] = b4.w;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < TB; ++j) acc[i][j] = fmaf(a[i], bv[j], acc[i][j]);
    }
    if (kt + 1 < kt_n) {
      stage(buf ^ 1);
      __syncthreads();
    }
  }
  auto row_of = [&](int i) { return n0 + base + (i < 4 ? i : 12 + i); };  // i>=4: base+16+(i-4)
  if constexpr (EPI == EPI_ARGMAX) {
    static_assert(TN == 128, "argmax partials are per 128-row tile");
    __syncthreads();  // the tiles are free: reuse them for the reduction
    float* rv = &Ws[0][0][0];                              // [16 ty][BT]
    int* ri = reinterpret_cast<int*>(&Xs[0][0][0]);        // [16 ty][BT]
#pragma unroll
    for (int j = 0; j < TB; ++j) {
      float v = -INFINITY;
      int idx = 0x7fffffff;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int n = row_of(i);
        if (n < N) {
          const float f = __half2float(__float2half_rn(acc[i][j]));
          if (f > v || (f == v && n < idx)) {
            v = f;
            idx = n;
          }
        }
      }
      rv[ty * BT + tx * TB + j] = v;
      ri[ty * BT + tx * TB + j] = idx;
    }
    __syncthreads();
    if (tid < BT && b0 + tid < batch) {
      float v = -INFINITY;
      int idx = 0x7fffffff;
      for (int y = 0; y < 16; ++y) {
        const float f = rv[y * BT + tid];
        const int n = ri[y * BT + tid];
        if (f > v || (f == v && n < idx)) {
          v = f;
          idx = n;
        }
      }
      amax_val[(size_t)blockIdx.x * batch + b0 + tid] = v;
      amax_idx[(size_t)blockIdx.x * batch + b0 + tid] = idx;
    }
    return;
  }
#pragma unroll
  for (int j = 0; j < TB; ++j) {
    const int b = b0 + tx * TB + j;
    if (b >= batch) break;
    if constexpr (EPI == EPI_SWIGLU) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int p = (n0 >> 1) + (ty >> 2) * 16 + (ty & 3) * 4 + i;
        if (p < N / 2) store_swiglu(e, b, p, acc[i][j], acc[i + 4][j]);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int n = row_of(i);
        if (n >= N) continue;
        if constexpr (EPI == EPI_F16) store_f16(e, b, n, acc[i][j]);
        if constexpr (EPI == EPI_RESIDUAL) store_res(e, b, n, acc[i][j]);
      }
    }
  }
}

// ---- attention (decode and prefill rows) -------------------------------------
// grid (rows, KVH), 256 threads; the 4 query heads of one kv head. Row r is
// token r % T of sequence r / T at position pos[seq] + r % T, and attends to
// positions 0 .. that position. Pass 1: thread -> positions (scores, each a
// sequential dot over 256 dims). Pass 2: thread d -> head dim d (weighted V
// sums, sequential over positions); threads 0..3 also form the 4 softmax sums.
__global__ void __launch_bounds__(256)
    xattn_kernel(const __half* __restrict__ q /*[rows][QH][HD]*/, const __half* __restrict__ gate,
                 const __half* __restrict__ kv, int64_t kv_seq_stride, int64_t kv_layer_off,
                 const int* __restrict__ pos, float scale, __half* __restrict__ out /*[rows][QH*HD]*/,
                 int rows_per_seq) {
  extern __shared__ float xa_sm[];  // [G][L] scores, then weights
  __shared__ __align__(16) float qs[G][HD];
  __shared__ float red[8][G];
  const int kvh = blockIdx.y, row = blockIdx.x, t = threadIdx.x;
  const int warp = t >> 5, lane = t & 31;
  const int seq = row / rows_per_seq;
  pdl_wait();
  pdl_launch();
  const int L = pos[seq] + row % rows_per_seq + 1;
#pragma unroll
  for (int g = 0; g < G; ++g) qs[g][t] = __half2float(q[((size_t)row * QH + kvh * G + g) * HD + t]);
  __syncthreads();
  const __half* base = kv + (size_t)seq * kv_seq_stride + kv_layer_off;
  float mx[G];
#pragma unroll
  for (int g = 0; g < G; ++g) mx[g] = -INFINITY;
  for (int p = t; p < L; p += 256) {
    const uint4* kr = reinterpret_cast<const uint4*>(base + (size_t)p * (2 * KVH * HD) + kvh * HD);
    float dot[G] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 8
    for (int d8 = 0; d8 < HD / 8; ++d8) {
      float kf[8];
      h8_to_f(kr[d8], kf);
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int g = 0; g < G; ++g) dot[g] = fmaf(qs[g][d8 * 8 + i], kf[i], dot[g]);  // exact fp16 products
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float sc = dot[g] * scale;
      xa_sm[g * L + p] = sc;
      mx[g] = fmaxf(mx[g], sc);
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx[g] = fmaxf(mx[g], __shfl_xor_sync(0xffffffffu, mx[g], o));
    if (lane == 0) red[warp][g] = mx[g];
  }
  __syncthreads();
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float m = red[0][g];
    for (int w = 1; w < 8; ++w) m = fmaxf(m, red[w][g]);
    mx[g] = m;
  }
  for (int p = t; p < L; p += 256)
#pragma unroll
    for (int g = 0; g < G; ++g) xa_sm[g * L + p] = exp_d(xa_sm[g * L + p] - mx[g]);
  __syncthreads();
  float acc[G] = {0.f, 0.f, 0.f, 0.f};
  float sum = 0.f;
  const __half* vb = base + KVH * HD + kvh * HD + t;
  // positions in blocks of 8: the 8 value loads are issued before the
  // sequential accumulation uses them (the order over positions is unchanged)
  int p = 0;
  for (; p + 8 <= L; p += 8) {
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = __half2float(vb[(size_t)(p + j) * (2 * KVH * HD)]);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int g = 0; g < G; ++g) acc[g] = acc[g] + xa_sm[g * L + p + j] * v[j];  // separate multiply and add
      if (t < G) sum = sum + xa_sm[t * L + p + j];
    }
  }
  for (; p < L; ++p) {
    const float v = __half2float(vb[(size_t)p * (2 * KVH * HD)]);
#pragma unroll
    for (int g = 0; g < G; ++g) acc[g] = acc[g] + xa_sm[g * L + p] * v;
    if (t < G) sum = sum + xa_sm[t * L + p];
  }
  __syncthreads();
  if (t < G) red[0][t] = sum;
  __syncthreads();
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const float inv = 1.0f / (red[0][g] + 1e-30f);
    const int qh = kvh * G + g;
    const float a16 = __half2float(__float2half_rn(acc[g] * inv));
    const float gt = __half2float(gate[((size_t)row * QH + qh) * HD + t]);
    out[((size_t)row * QH + qh) * HD + t] = __float2half_rn(a16 * (1.0f / (1.0f + exp_d(-gt))));
  }
}

// ---- DeltaNet ---------------------------------------------------------------
// 128-wide sum of squares in the shaders' tree order (strides 64..1). The
// strides 64 and 32 pair lanes of different warps (shared memory); strides
// 16..1 run in warp 0 with shfl_down, which adds exactly the same pairs
// (lane i takes lane i + stride), so the result is the shared-memory tree's.
__device__ __forceinline__ float tree128(float* s, int t) {
  __syncthreads();
  if (t < 64) s[t] = s[t] + s[t + 64];
  __syncthreads();
  if (t < 32) {
    float v = s[t] + s[t + 32];
#pragma unroll
    for (int stride = 16; stride > 0; stride >>= 1) v = v + __shfl_down_sync(0xffffffffu, v, stride);
    if (t == 0) s[0] = v;
  }
  __syncthreads();
  const float r = s[0];
  __syncthreads();
  return r;
}

// conv + SiLU (fp16) of one channel: window w[0..3] oldest first.
__device__ __forceinline__ float conv_silu(const float* win, const __half* cw) {
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) sum = fmaf(win[i], __half2float(cw[i]), sum);  // exact fp16 products
  const float silu = sum / (1.0f + exp_d(-sum));
  return __half2float(__float2half_rn(silu));
}

struct GBeta {
  float g, beta;
};
__device__ __forceinline__ GBeta gbeta(float a, float b, const float* alb /*[2]*/) {
  const float sp = log_d(1.0f + exp_d(a + alb[1]));
  GBeta r;
  r.g = -exp_d(alb[0]) * sp;
  r.beta = 1.0f / (1.0f + exp_d(-b));
  return r;
}

// The recurrence of one token for value column j (thread j) with the column
// S[:, j] in registers; sk, sq: this token's k and q * q_scale (fp32, shared).
// Returns the raw output o_j = S^T q.
__device__ __forceinline__ float rec_column(float* S, const float* sk, const float* sq, float vj, float eg,
                                            float beta) {
  float kv = 0.f;
#pragma unroll
  for (int i = 0; i < DND; ++i) {
    S[i] = S[i] * eg;
    kv = kv + S[i] * sk[i];
  }
  const float delta = (vj - kv) * beta;
  float o = 0.f;
#pragma unroll
  for (int i = 0; i < DND; ++i) {
    S[i] = S[i] + sk[i] * delta;
    o = o + S[i] * sq[i];
  }
  return o;
}

// RMSNorm of the 128 outputs (tree), weight, fp16 round, SiLU(z) gate.
__device__ __forceinline__ __half norm_gate(float o, float* red, int j, float w, float z, float eps) {
  red[j] = o * o;
  const float nf = 1.0f / sqrtf(tree128(red, j) / (float)DND + eps);
  const float normed = o * nf;
  const float silu = z / (1.0f + exp_d(-z));
  const float weighted = __half2float(__float2half_rn(w * normed));
  return __float2half_rn(weighted * silu);
}

// One decode token: grid (batch * 16), 128 threads (thread j: channel j of the
// head's q, k and v blocks, and value column j). qkv: [batch][ld] raw
// projection [q 2048 | k 2048 | v 2048 | z 2048 | a 16 | b 16] (ld = 8224);
// conv [batch][6144][4]; state [batch][16][128][128]; out [batch][ldo].
__global__ void __launch_bounds__(128, 2)
    xdn_decode_kernel(__half* __restrict__ qkv, int ld, __half* __restrict__ conv, const __half* __restrict__ conv_w,
                      const float* __restrict__ alb, const float* __restrict__ norm_w, float eps,
                      float* __restrict__ state, __half* __restrict__ out, int ldo) {
  const int item = blockIdx.x, b = item / DNH, h = item % DNH, j = threadIdx.x;
  __shared__ float sk[DND], sq[DND], red[DND];
  __shared__ GBeta gb;
  float* Sg = state + (size_t)item * DND * DND;
  // the state does not depend on the predecessor's output: pull it into L2
  // now (thread j: the four 128-byte lines of state row j), load it later
#pragma unroll
  for (int l = 0; l < 4; ++l) asm volatile("prefetch.global.L2 [%0];" ::"l"(Sg + j * DND + l * 32));
  pdl_wait();
  pdl_launch();
  __half* row = qkv + (size_t)b * ld;
  float val[3];
#pragma unroll
  for (int c = 0; c < 3; ++c) {  // conv state shift + insert, conv, SiLU (deltanet_conv_l2_qk.comp:48-75)
    const int ch = c * 2048 + h * DND + j;
    __half* cs = conv + ((size_t)b * CONV + ch) * 4;
    float win[4];
#pragma unroll
    for (int i = 0; i < 3; ++i) win[i] = __half2float(cs[i + 1]);
    win[3] = __half2float(row[ch]);
#pragma unroll
    for (int i = 0; i < 3; ++i) cs[i] = cs[i + 1];
    cs[3] = row[ch];
    val[c] = conv_silu(win, conv_w + (size_t)ch * 4);
  }
  // L2 of the q and k blocks (:79-110), stored as fp16 (the in-place contract)
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    red[j] = val[c] * val[c];
    const float inv = 1.0f / sqrtf(tree128(red, j) + 1e-6f);
    const __half r16 = __float2half_rn(val[c] * inv);
    row[c * 2048 + h * DND + j] = r16;
    if (c == 0) sq[j] = __half2float(r16) * (1.0f / sqrtf((float)DND));  // q * q_scale
    else sk[j] = __half2float(r16);
  }
  const __half v16 = __float2half_rn(val[2]);
  row[4096 + h * DND + j] = v16;
  if (j == 0) gb = gbeta(__half2float(row[8192 + h]), __half2float(row[8192 + DNH + h]), alb + 2 * h);
  float S[DND];
#pragma unroll
  for (int i = 0; i < DND; ++i) S[i] = Sg[i * DND + j];
  __syncthreads();
  const float o = rec_column(S, sk, sq, __half2float(v16), exp_d(gb.g), gb.beta);
#pragma unroll
  for (int i = 0; i < DND; ++i) Sg[i * DND + j] = S[i];
  out[(size_t)b * ldo + h * DND + j] = norm_gate(o, red, j, norm_w[j], __half2float(row[6144 + h * DND + j]), eps);
}

// Prefill, part 1 (every prompt token at once): conv + SiLU + L2 and g/beta.
// grid (rows = batch*T, 16), 128 threads. proj [rows][ld] as in the decode
// kernel; conv_old [batch][6144][4] is the conv state before the prompt;
// rows t == T-1 write the new conv state. Outputs token-major fp16 q, k, v
// [rows][2048] (q pre-scaled by q_scale in fp32 happens in part 2) and fp32
// g, beta [rows][16].
__global__ void __launch_bounds__(128)
    xdn_prefill_conv_kernel(const __half* __restrict__ proj, int ld, int T, const __half* __restrict__ conv_w,
                            const __half* __restrict__ conv_old, __half* __restrict__ conv_new,
                            const float* __restrict__ alb, __half* __restrict__ qo, __half* __restrict__ ko,
                            __half* __restrict__ vo, float* __restrict__ go, float* __restrict__ bo) {
  const int r = blockIdx.x, h = blockIdx.y, j = threadIdx.x;
  const int b = r / T, t = r % T;
  __shared__ float red[DND];
  pdl_wait();
  pdl_launch();
  float val[3];
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    const int ch = c * 2048 + h * DND + j;
    float win[4];  // x_{t-3} .. x_t; before the prompt: the conv state's newest slots
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int tt = t - 3 + i;
      win[i] = tt >= 0 ? __half2float(proj[(size_t)(b * T + tt) * ld + ch])
                       : __half2float(conv_old[((size_t)b * CONV + ch) * 4 + 4 + tt]);
    }
    val[c] = conv_silu(win, conv_w + (size_t)ch * 4);
    if (t == T - 1) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int tt = T - 4 + i;
        conv_new[((size_t)b * CONV + ch) * 4 + i] =
            tt >= 0 ? proj[(size_t)(b * T + tt) * ld + ch] : conv_old[((size_t)b * CONV + ch) * 4 + 4 + tt];
      }
    }
  }
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    red[j] = val[c] * val[c];
    const float inv = 1.0f / sqrtf(tree128(red, j) + 1e-6f);
    (c == 0 ? qo : ko)[(size_t)r * 2048 + h * DND + j] = __float2half_rn(val[c] * inv);
  }
  vo[(size_t)r * 2048 + h * DND + j] = __float2half_rn(val[2]);
  if (j == 0) {
    const GBeta gbv = gbeta(__half2float(proj[(size_t)r * ld + 8192 + h]),
                            __half2float(proj[(size_t)r * ld + 8192 + DNH + h]), alb + 2 * h);
    go[(size_t)r * DNH + h] = gbv.g;
    bo[(size_t)r * DNH + h] = gbv.beta;
  }
}

// Prefill, part 2: the recurrence over the prompt, token by token. Value
// columns are independent in the recurrence, so a head's 128 columns are
// split over 4 CTAs of one warp each (thread = column, its column of the
// state in registers); the next token's inputs are loaded while the current
// one is computed. Writes the raw outputs o = S^T (q * q_scale) as fp32
// core [rows][2048]; part 3 applies the gated norm.
constexpr int kRecCols = 32;
__global__ void __launch_bounds__(kRecCols)
    xdn_prefill_rec_kernel(const __half* __restrict__ qi, const __half* __restrict__ ki,
                           const __half* __restrict__ vi, const float* __restrict__ gi,
                           const float* __restrict__ bi, int T, float* __restrict__ state,
                           float* __restrict__ core /*[rows][2048]*/) {
  constexpr int SPLIT = DND / kRecCols;
  const int item = blockIdx.x / SPLIT, part = blockIdx.x % SPLIT, b = item / DNH, h = item % DNH;
  const int lane = threadIdx.x, j = part * kRecCols + lane;
  __shared__ __align__(16) float sk[2][DND], sq[2][DND];
  float* Sg = state + (size_t)item * DND * DND;
  float S[DND];
#pragma unroll
  for (int i = 0; i < DND; ++i) S[i] = Sg[i * DND + j];
  pdl_wait();
  pdl_launch();
  const float q_scale = 1.0f / sqrtf((float)DND);
  // this token's inputs: q, k (4 of the 128 per lane), v_j, g, beta
  uint2 nq, nk;
  float nv, ng, nb;
  auto load = [&](int t) {
    const size_t r = (size_t)b * T + t;
    nq = *reinterpret_cast<const uint2*>(qi + r * 2048 + h * DND + lane * 4);
    nk = *reinterpret_cast<const uint2*>(ki + r * 2048 + h * DND + lane * 4);
    nv = __half2float(vi[r * 2048 + h * DND + j]);
    ng = gi[r * DNH + h];
    nb = bi[r * DNH + h];
  };
  load(0);
  for (int t = 0; t < T; ++t) {
    const int s = t & 1;
    {
      const __half2* q2 = reinterpret_cast<const __half2*>(&nq);
      const __half2* k2 = reinterpret_cast<const __half2*>(&nk);
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float2 qf = __half22float2(q2[e]), kf = __half22float2(k2[e]);
        sq[s][lane * 4 + 2 * e] = qf.x * q_scale;
        sq[s][lane * 4 + 2 * e + 1] = qf.y * q_scale;
        sk[s][lane * 4 + 2 * e] = kf.x;
        sk[s][lane * 4 + 2 * e + 1] = kf.y;
      }
    }
    const float vj = nv, eg = exp_d(ng), beta = nb;
    __syncwarp();
    if (t + 1 < T) load(t + 1);
    core[((size_t)b * T + t) * 2048 + h * DND + j] = rec_column(S, sk[s], sq[s], vj, eg, beta);
  }
#pragma unroll
  for (int i = 0; i < DND; ++i) Sg[i * DND + j] = S[i];
}

// Prefill, part 3: the gated RMSNorm of every (token, head), all at once.
// grid (rows, 16), 128 threads.
__global__ void __launch_bounds__(128)
    xdn_prefill_gate_kernel(const float* __restrict__ core, const __half* __restrict__ proj, int ld,
                            const float* __restrict__ norm_w, float eps, __half* __restrict__ out) {
  const int r = blockIdx.x, h = blockIdx.y, j = threadIdx.x;
  __shared__ float red[DND];
  pdl_wait();
  pdl_launch();
  const float o = core[(size_t)r * 2048 + h * DND + j];
  const float z = __half2float(proj[(size_t)r * ld + 6144 + h * DND + j]);
  out[(size_t)r * 2048 + h * DND + j] = norm_gate(o, red, j, norm_w[j], z, eps);
}

template <int EPI, int R>
Status gemv_launch(const __half* x, int ldx, const __half* w, int K, int N, int batch, Epi e, float* av, int* ai,
                   cudaStream_t st) {
  const int units = EPI == EPI_SWIGLU ? N / 2 : N;
  cudaError_t err = launch_k(xgemv_kernel<EPI, R>, dim3((units + 127) / 128), dim3(128), 0, st, x, ldx, w, K, N,
                             batch, e, av, ai);
  if (err != cudaSuccess) return cuda_status(err, "xgemv_kernel");
  SPOCK_LAUNCH_CHECK("xgemv_kernel");
  return Status::ok();
}

template <int EPI, int R>
Status gemv2_launch(const __half* x, int ldx, const __half* w, int K, int N, int batch, Epi e, float* av, int* ai,
                    cudaStream_t st) {
  constexpr int kSt = EPI == EPI_SWIGLU ? 4 : 6;
  constexpr int NR = EPI == EPI_SWIGLU ? 2 : 1;
  const size_t smem = (size_t)kSt * 64 * NR * kRowB + (size_t)R * kXC * 4;
  // per device, once (the first call of a shape is eager, before any capture)
  static std::atomic<uint64_t> configured{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  if (!(configured.load() & bit)) {
    cudaError_t a = cudaFuncSetAttribute(xgemv2_kernel<EPI, R, kSt>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (a != cudaSuccess) return cuda_status(a, "xgemv2_kernel smem attribute");
    configured.fetch_or(bit);
  }
  const int units = EPI == EPI_SWIGLU ? N / 2 : N;
  cudaError_t err = launch_k(xgemv2_kernel<EPI, R, kSt>, dim3((units + 63) / 64), dim3(64), smem, st, x, ldx, w, K,
                             N, batch, e, av, ai);
  if (err != cudaSuccess) return cuda_status(err, "xgemv2_kernel");
  SPOCK_LAUNCH_CHECK("xgemv2_kernel");
  return Status::ok();
}

template <int EPI, int TN, int TB>
Status gemm_launch(const __half* x, int ldx, const __half* w, int K, int N, int batch, Epi e, float* av, int* ai,
                   cudaStream_t st) {
  const int bt = 16 * TB;
  cudaError_t err = launch_k(xgemm_kernel<EPI, TN, TB>, dim3((N + TN - 1) / TN, (batch + bt - 1) / bt), dim3(TN * 2),
                             0, st, x, ldx, w, K, N, batch, e, av, ai);
  if (err != cudaSuccess) return cuda_status(err, "xgemm_kernel");
  SPOCK_LAUNCH_CHECK("xgemm_kernel");
  return Status::ok();
}

// The largest tile that still gives every SM two CTAs (fewer, larger tiles
// re-read less but leave SMs idle on the narrow projections).
template <int EPI>
Status gemm_pick(const __half* x, int ldx, const __half* w, int K, int N, int batch, Epi e, float* av, int* ai,
                 cudaStream_t st) {
  auto ctas = [&](int tn, int tb) { return (int64_t)((N + tn - 1) / tn) * ((batch + 16 * tb - 1) / (16 * tb)); };
  const int64_t want = 2 * 148;
  if (EPI == EPI_ARGMAX || ctas(128, 8) >= want)
    return batch > 64 ? gemm_launch<EPI, 128, 8>(x, ldx, w, K, N, batch, e, av, ai, st)
                      : gemm_launch<EPI, 128, 4>(x, ldx, w, K, N, batch, e, av, ai, st);
  if constexpr (EPI != EPI_ARGMAX) {
    if (batch > 64 && ctas(64, 8) >= want) return gemm_launch<EPI, 64, 8>(x, ldx, w, K, N, batch, e, av, ai, st);
    if (ctas(128, 4) >= want) return gemm_launch<EPI, 128, 4>(x, ldx, w, K, N, batch, e, av, ai, st);
    return gemm_launch<EPI, 64, 4>(x, ldx, w, K, N, batch, e, av, ai, st);
  }
  return Status::ok();
}

template <int EPI>
Status proj_epi(const __half* x, int ldx, const __half* w, int K, int N, int batch, Epi e, float* av, int* ai,
                cudaStream_t st) {
  if constexpr (EPI != EPI_ARGMAX) {
    if (batch == 1) return gemv2_launch<EPI, 1>(x, ldx, w, K, N, batch, e, av, ai, st);
    if (batch == 2) return gemv2_launch<EPI, 2>(x, ldx, w, K, N, batch, e, av, ai, st);
  }
  switch (batch) {
    case 1: return gemv_launch<EPI, 1>(x, ldx, w, K, N, batch, e, av, ai, st);
    case 2: return gemv_launch<EPI, 2>(x, ldx, w, K, N, batch, e, av, ai, st);
    case 3:
    case 4: return gemv_launch<EPI, 4>(x, ldx, w, K, N, batch, e, av, ai, st);
    case 5: case 6: case 7: case 8: return gemv_launch<EPI, 8>(x, ldx, w, K, N, batch, e, av, ai, st);
    default: break;
  }
  return gemm_pick<EPI>(x, ldx, w, K, N, batch, e, av, ai, st);
}

}  // namespace
}  // namespace xk

// y[b][n] = fp16(sum_k W[n][k] x[b][k]) in matvec.comp's order, with the
// epilogue `epi` (EPI_F16, EPI_RESIDUAL: y = fp16(res + fp16(.)), EPI_SWIGLU on
// 16-row-interleaved gate/up weights: y[b][p] = fp16(silu(g) u), EPI_ARGMAX:
// per 128-row tile partials for launch_argmax_finish).
Status launch_exact_proj(int epi, const void* x, int ldx, const void* w, int K, int N, int batch, void* y, int ldy,
                         const void* res, float* amax_val, int* amax_idx, cudaStream_t st) {
  if (K % 16 || ldx % 8 || ((uintptr_t)x & 15) || ((uintptr_t)w & 15))
    return Status::err(SPOCK_ERR_UNSUPPORTED, "exact projection: K and ldx multiples of 16 / 8, 16-byte aligned");
  if (epi == EPI_SWIGLU && N % 32) return Status::err(SPOCK_ERR_UNSUPPORTED, "exact projection: SWIGLU needs N % 32 == 0");
  xk::Epi e{(__half*)y, ldy, (const __half*)res};
  const __half *xh = (const __half*)x, *wh = (const __half*)w;
  switch (epi) {
    case EPI_F16: return xk::proj_epi<EPI_F16>(xh, ldx, wh, K, N, batch, e, amax_val, amax_idx, st);
    case EPI_RESIDUAL: return xk::proj_epi<EPI_RESIDUAL>(xh, ldx, wh, K, N, batch, e, amax_val, amax_idx, st);
    case EPI_SWIGLU: return xk::proj_epi<EPI_SWIGLU>(xh, ldx, wh, K, N, batch, e, amax_val, amax_idx, st);
    case EPI_ARGMAX: return xk::proj_epi<EPI_ARGMAX>(xh, ldx, wh, K, N, batch, e, amax_val, amax_idx, st);
    default: return Status::err(SPOCK_ERR_INVALID, "exact projection: unknown epilogue");
  }
}

Status launch_exact_attn(const void* q, const void* gate, const void* kv, int64_t kv_seq_stride, int64_t kv_layer_off,
                         const int* pos, int max_seq, float scale, void* out, int rows, int rows_per_seq,
                         cudaStream_t st) {
  const size_t smem = (size_t)xk::G * max_seq * sizeof(float);
  static thread_local size_t configured = 0;
  if (smem > configured) {
    cudaError_t e = cudaFuncSetAttribute(xk::xattn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return cuda_status(e, "xattn_kernel smem attribute");
    configured = smem;
  }
  cudaError_t e = launch_k(xk::xattn_kernel, dim3(rows, xk::KVH), dim3(256), smem, st, (const __half*)q,
                           (const __half*)gate, (const __half*)kv, kv_seq_stride, kv_layer_off, pos, scale,
                           (__half*)out, rows_per_seq);
  if (e != cudaSuccess) return cuda_status(e, "xattn_kernel");
  SPOCK_LAUNCH_CHECK("xattn_kernel");
  return Status::ok();
}

Status launch_exact_dn_decode(void* proj, int ld, void* conv, const void* conv_w, const float* alb, const float* norm_w,
                              float eps, float* state, void* out, int ldo, int batch, cudaStream_t st) {
  cudaError_t e = launch_k(xk::xdn_decode_kernel, dim3(batch * xk::DNH), dim3(128), 0, st, (__half*)proj, ld,
                           (__half*)conv, (const __half*)conv_w, alb, norm_w, eps, state, (__half*)out, ldo);
  if (e != cudaSuccess) return cuda_status(e, "xdn_decode_kernel");
  SPOCK_LAUNCH_CHECK("xdn_decode_kernel");
  return Status::ok();
}

Status launch_exact_dn_prefill(const void* proj, int ld, int batch, int T, const void* conv_w, const void* conv_old,
                               void* conv_new, const float* alb, const float* norm_w, float eps, void* q, void* k,
                               void* v, float* g, float* beta, float* core, float* state, void* out, cudaStream_t st) {
  cudaError_t e = launch_k(xk::xdn_prefill_conv_kernel, dim3(batch * T, xk::DNH), dim3(128), 0, st,
                           (const __half*)proj, ld, T, (const __half*)conv_w, (const __half*)conv_old,
                           (__half*)conv_new, alb, (__half*)q, (__half*)k, (__half*)v, g, beta);
  if (e != cudaSuccess) return cuda_status(e, "xdn_prefill_conv_kernel");
  SPOCK_LAUNCH_CHECK("xdn_prefill_conv_kernel");
  e = launch_k(xk::xdn_prefill_rec_kernel, dim3(batch * xk::DNH * (xk::DND / xk::kRecCols)), dim3(xk::kRecCols), 0,
               st, (const __half*)q, (const __half*)k, (const __half*)v, (const float*)g, (const float*)beta, T, state,
               core);
  if (e != cudaSuccess) return cuda_status(e, "xdn_prefill_rec_kernel");
  SPOCK_LAUNCH_CHECK("xdn_prefill_rec_kernel");
  e = launch_k(xk::xdn_prefill_gate_kernel, dim3(batch * T, xk::DNH), dim3(128), 0, st, (const float*)core,
               (const __half*)proj, ld, norm_w, eps, (__half*)out);
  if (e != cudaSuccess) return cuda_status(e, "xdn_prefill_gate_kernel");
  SPOCK_LAUNCH_CHECK("xdn_prefill_gate_kernel");
  return Status::ok();
}

}  // namespace spock
