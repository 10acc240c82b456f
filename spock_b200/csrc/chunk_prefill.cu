// Chunked gated delta rule on sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// Semantics: spock's run_deltanet_chunk_rule (src/runtime/deltanet_chunk.cpp:
// 53-284), i.e. the chunked form of HF torch_chunk_gated_delta_rule. One CTA
// owns one (sequence, head) pair and walks its chunks of C=64 tokens in order;
// the 128x128 fp32 recurrent state S lives in TMEM for the whole walk and is
// written to HBM once at the end.
//
// Per chunk (s = 1/sqrt(128); gc = cumulative g in the chunk;
// Dec[i][j] = exp(gc_i - gc_j) for j <= i):
//   G1  = [Q;K] K^T                         tcgen05, M=128 N=64  K=128
//   P   = s * (Q K^T) o Dec (lower incl. diag)              CUDA cores
//   N   = -(beta_i K K^T) o Dec (strictly lower)            CUDA cores
//   T   = (I - N)^-1  (unit lower, fp32 blocked inverse)    CUDA cores
//   D1  = [T diag(beta) ; 0] V           = [U ; 0]          tcgen05, M=128 N=128 K=64
//   Wt  = K^T (T diag(beta e^gc))^T      = W^T              tcgen05, M=128 N=64  K=64
//   D1 += [-W ; diag(s e^gc) Q] S16      = [v_new ; Q'S]    tcgen05, M=128 N=128 K=128
//   S  <- e^{gc_63} S + K^T diag(e^{gc_63-gc}) v_new        tcgen05 into TMEM, M=128 N=128 K=64
//   D1 += [0 ; P] v_new                  -> rows 64..127 = core_attn_out of the chunk
// This is the reference's steps (deltanet_chunk.cpp:137-268) regrouped: the
// reference's k_cumdecay = A (k beta e^g) is W, solved_value = A (v beta) is U,
// v_prime = W S, attn_inter = (q e^g) S and local_attn = P.
//
// Operands are fp16 with fp32 accumulation; S is rounded to fp16 only as an
// MMA operand while its fp32 master copy stays in TMEM. Inputs arrive as fp16
// or bf16 tiles by TMA (bf16 is converted to fp16 in shared memory). The
// precise variant (fp32 inputs) carries the operands whose rounding reaches
// the results as fp16 hi/lo pairs (x = hi + lo, about 22 bits): Q and K in
// G1, T diag(beta) and V in U, P and v_new in the output, K and the decayed
// v_new in the state update (hi*hi + hi*lo + lo*hi). A numpy model of these
// rounding points singled them out: fp16 K in the state update alone gave the
// 2e-4 state error, P / v_new / G1 the output error at large |v|.
//
// TMEM (512 columns): [0,128) S, [128,256) D1, [256,320) G1, [320,384) W^T.
// Every wait on an mbarrier is bounded; on timeout the kernel records an error
// code in *err_flag, releases TMEM and returns.
#include <cuda.h>

#include <cstdlib>
#include <mutex>

#include "chunk_scratch.h"
#include "common.cuh"
#include "tc.cuh"
#include "chunk_common.cuh"

namespace spock {
namespace {

using chunk::C;
using chunk::D;
using chunk::LDN;
using chunk::sw128;
using chunk::pack_h2;
using chunk::pack8;
using chunk::unpack8;
using chunk::store_row32;
constexpr int kThreads = 128;
constexpr uint32_t kWaitLimit = 1u << 22;

// Shared memory carve-up (offsets from a 1024-aligned base).
constexpr int OFF_QK = 0;                  // [Q;K] K-major, 2 column halves x (Q 8K | K 8K)
constexpr int OFF_V = 32 * 1024;           // V, 2 column halves x 8K
constexpr int OFF_TB = 48 * 1024;          // [T diag(beta) 8K | zero 8K | P 8K]
constexpr int OFF_TBE = 72 * 1024;         // T diag(beta e^gc), K-major 64x64
constexpr int OFF_AW = 80 * 1024;          // [-W ; Q'] K-major 128x128
constexpr int OFF_SB = 112 * 1024;         // S16, MN-major [kd][v] (aliased by VN/VS)
constexpr int OFF_VN = OFF_SB;             // v_new16, MN-major [token][v]
constexpr int OFF_VS = OFF_SB + 16 * 1024; // v_new16 * e^{gL-gc}
constexpr int OFF_NM = 144 * 1024;
constexpr int OFF_TM = OFF_NM + C * LDN * 4;
constexpr int OFF_YM = OFF_TM + C * LDN * 4;
constexpr int OFF_SMALL = OFF_YM + 3 * 256 * 4;
constexpr int SMEM_BYTES = OFF_SMALL + 2048 + 1024;  // + alignment slack
// Extra regions of the precise (fp32-input) variant: the low fp16 halves of V
// and K, and [T diag(beta)]_lo with its own zero block, followed by P_lo.
// Q_lo / K_lo for G1 and v_new_lo for the output borrow the AW region while
// it is idle. The low half of
// diag(e^{gL-gc}) v_new reuses the AW region, which is dead after step 7.
constexpr int OFF_VLO = 182 * 1024;
constexpr int OFF_KLO = OFF_NM;  // low fp16 half of K, 2 x 8K, between the solve and the next G1
static_assert(C * LDN * 4 >= 16 * 1024, "K_lo fits in the N matrix's region");
constexpr int OFF_TBL = OFF_VLO + 16 * 1024;
constexpr int OFF_PLO = OFF_TBL + 16 * 1024;  // P_lo: with TBL's zero block before it, [0 ; P_lo]
constexpr int SMEM_BYTES_PRECISE = OFF_PLO + 8 * 1024 + 1024;
static_assert(SMEM_BYTES_PRECISE <= 232448, "shared memory per CTA");
static_assert(OFF_VLO >= OFF_SMALL + 2048, "smem regions overlap");

template <bool kBf16In, int kOut, bool kPrecise>
__global__ void __launch_bounds__(kThreads, 1)
    chunk_rule_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                      const __grid_constant__ CUtensorMap tmv, const __grid_constant__ CUtensorMap tmvlo,
                      const __grid_constant__ CUtensorMap tmklo, const __grid_constant__ CUtensorMap tmqlo,
                      const float* __restrict__ g,
                      const float* __restrict__ beta, const float* __restrict__ init,
                      void* __restrict__ out, float* __restrict__ final_state, int S,
                      int* __restrict__ err_flag) {
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment by pointer arithmetic on the __shared__ array keeps the
  // shared address space visible to the compiler (LDS/STS, not generic loads).
  uint8_t* sm = smem_raw + ((1024u - (tc::smem_u32(smem_raw) & 1023u)) & 1023u);
  float* NM = reinterpret_cast<float*>(sm + OFF_NM);
  float* TM = reinterpret_cast<float*>(sm + OFF_TM);
  float* YM = reinterpret_cast<float*>(sm + OFF_YM);
  float* s_g = reinterpret_cast<float*>(sm + OFF_SMALL);  // raw g, then cumulative
  float* s_beta = s_g + 64;
  float* s_eg = s_beta + 64;
  uint64_t* bar_tma = reinterpret_cast<uint64_t*>(s_eg + 64);
  uint64_t* bar_mma = bar_tma + 1;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bar_mma + 1);

  const int t = threadIdx.x, warp = t >> 5;
  const int p = blockIdx.x;  // (sequence, head) pair
  const float scale = 0.08838834764831845f;  // 1/sqrt(128)
  const uint32_t sbase = tc::smem_u32(sm);

  if (t == 0) {
    tc::mbar_init(bar_tma, 1);
    tc::mbar_init(bar_mma, 1);
    tc::fence_mbar_init();
    tc::prefetch_tmap(&tmq);
    tc::prefetch_tmap(&tmk);
    tc::prefetch_tmap(&tmv);
    if constexpr (kPrecise) {
      tc::prefetch_tmap(&tmvlo);
      tc::prefetch_tmap(&tmklo);
      tc::prefetch_tmap(&tmqlo);
    }
  }
  if (warp == 0) {
    tc::tmem_alloc(s_tmem, 512);
    tc::tmem_relinquish();
  }
  // zero block between T diag(beta) and P (and after [T diag(beta)]_lo)
  for (int i = t; i < 8 * 1024 / 16; i += kThreads) {
    reinterpret_cast<uint4*>(sm + OFF_TB + 8 * 1024)[i] = make_uint4(0, 0, 0, 0);
    if constexpr (kPrecise) reinterpret_cast<uint4*>(sm + OFF_TBL + 8 * 1024)[i] = make_uint4(0, 0, 0, 0);
  }
  tc::fence_async_smem();
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tb = *s_tmem;
  const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
  const uint32_t tS = tb + lane_base, tD1 = tb + 128 + lane_base, tG1 = tb + 256 + lane_base,
                 tWT = tb + 320 + lane_base;
  const uint32_t mS = tb, mD1 = tb + 128, mG1 = tb + 256, mWT = tb + 320;  // MMA D addresses

  // Initial state -> TMEM (row t = key index t).
  {
    const float* src = init ? init + ((size_t)p * D + t) * D : nullptr;
#pragma unroll 1
    for (int cb = 0; cb < 4; ++cb) {
      float v[32];
#pragma unroll
      for (int k = 0; k < 32; ++k) v[k] = src ? src[cb * 32 + k] : 0.f;
      tc::tmem_st32(tS + cb * 32, v);
    }
    tc::tmem_st_wait();
  }

  uint32_t ph_tma = 0, ph_mma = 0;
  bool failed = false;
  const int nchunks = (S + C - 1) / C;
  constexpr uint32_t ID_G1 = tc::idesc_f16(128, 64, false, false);
  constexpr uint32_t ID_U = tc::idesc_f16(128, 128, false, true);
  constexpr uint32_t ID_WT = tc::idesc_f16(128, 64, true, false);
  constexpr uint32_t ID_1 = tc::idesc_f16(128, 128, false, true);
  constexpr uint32_t ID_2A = tc::idesc_f16(128, 128, true, true);

  auto wait_mma = [&]() -> bool {
    bool ok = tc::mbar_wait_bounded(bar_mma, ph_mma, kWaitLimit);
    ph_mma ^= 1;
    return __syncthreads_or(!ok) == 0;
  };

  for (int c = 0; c < nchunks; ++c) {
    // ---- 1. loads: q/k/v tiles by TMA, g/beta by threads -----------------
    if (t == 0) {
      tc::mbar_arrive_expect_tx(bar_tma, (kPrecise ? 12 : 6) * 64 * 64 * 2);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        tc::tma_load_3d(sm + OFF_QK + h * 16384, &tmq, bar_tma, h * 64, c * C, p);
        tc::tma_load_3d(sm + OFF_QK + h * 16384 + 8192, &tmk, bar_tma, h * 64, c * C, p);
        tc::tma_load_3d(sm + OFF_V + h * 8192, &tmv, bar_tma, h * 64, c * C, p);
        if constexpr (kPrecise) {
          tc::tma_load_3d(sm + OFF_VLO + h * 8192, &tmvlo, bar_tma, h * 64, c * C, p);
          // [Q_lo ; K_lo] in the AW region (idle until Q' at step 4), laid out as [Q ; K]
          tc::tma_load_3d(sm + OFF_AW + h * 16384, &tmqlo, bar_tma, h * 64, c * C, p);
          tc::tma_load_3d(sm + OFF_AW + h * 16384 + 8192, &tmklo, bar_tma, h * 64, c * C, p);
        }
      }
    }
    if (t < C) {
      const int tok = c * C + t;
      s_g[t] = tok < S ? g[(size_t)p * S + tok] : 0.f;
      s_beta[t] = tok < S ? beta[(size_t)p * S + tok] : 0.f;
    }
    __syncthreads();
    if (t == 0) {  // cumulative g in token order, as the reference
      float run = 0.f;
      for (int i = 0; i < C; ++i) {
        run = run + s_g[i];
        s_g[i] = run;
      }
    }
    __syncthreads();
    if (t < C) s_eg[t] = expf(s_g[t]);
    const float gL = s_g[C - 1];
    const float egL = expf(gL);

    // ---- 2. S16 <- S, S <- e^{gL} S (TMEM, row t) ------------------------
    tc::tc_fence_after();
#pragma unroll 1
    for (int cb = 0; cb < 4; ++cb) {
      float v[32];
      tc::tmem_ld32(tS + cb * 32, v);
      uint8_t* dst = sm + OFF_SB + (cb >> 1) * 16384;
#pragma unroll
      for (int q = 0; q < 4; ++q)
        *reinterpret_cast<uint4*>(dst + sw128(t, (cb & 1) * 4 + q)) = pack8(&v[8 * q]);
#pragma unroll
      for (int k = 0; k < 32; ++k) v[k] = mul_rn(v[k], egL);
      tc::tmem_st32(tS + cb * 32, v);
    }
    tc::tmem_st_wait();

    bool ok = tc::mbar_wait_bounded(bar_tma, ph_tma, kWaitLimit);
    ph_tma ^= 1;
    if (__syncthreads_or(!ok)) { failed = true; break; }
    if constexpr (kBf16In) {  // bf16 -> fp16 in place (exact for |x| in fp16 normal range)
      uint4* qkv = reinterpret_cast<uint4*>(sm + OFF_QK);
      for (int i = t; i < 48 * 1024 / 16; i += kThreads) {
        uint4 u = qkv[i];
        uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&w[k]);
          float2 f = __bfloat1622float2(b);
          w[k] = pack_h2(f.x, f.y);
        }
        qkv[i] = u;
      }
    }
    tc::fence_async_smem();
    tc::tc_fence_before();
    __syncthreads();

    // ---- 3. G1 = [Q;K] K^T ------------------------------------------------
    if (t == 0) {
      tc::tc_fence_after();
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const uint32_t koff = (ks >> 2) * 16384 + (ks & 3) * 32;
        tc::mma_f16(mG1, tc::sdesc(sbase + OFF_QK + koff, 16, 1024),
                    tc::sdesc(sbase + OFF_QK + 8192 + koff, 16, 1024), ID_G1, ks > 0);
      }
      if constexpr (kPrecise) {  // [Q;K]_hi K_lo^T + [Q;K]_lo K_hi^T
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint32_t koff = (ks >> 2) * 16384 + (ks & 3) * 32;
          tc::mma_f16(mG1, tc::sdesc(sbase + OFF_QK + koff, 16, 1024),
                      tc::sdesc(sbase + OFF_AW + 8192 + koff, 16, 1024), ID_G1, 1);
          tc::mma_f16(mG1, tc::sdesc(sbase + OFF_AW + koff, 16, 1024),
                      tc::sdesc(sbase + OFF_QK + 8192 + koff, 16, 1024), ID_G1, 1);
        }
      }
      tc::mma_commit(bar_mma);
    }
    if (!wait_mma()) { failed = true; break; }
    tc::tc_fence_after();
    {
      float a[64];
      tc::tmem_ld32(tG1, *reinterpret_cast<float(*)[32]>(&a[0]));
      tc::tmem_ld32(tG1 + 32, *reinterpret_cast<float(*)[32]>(&a[32]));
      if (t < C) {  // P row t
        const float gi = s_g[t];
        uint8_t* dst = sm + OFF_TB + 16384;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          float x[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const int j = q * 8 + k;
            x[k] = (j <= t) ? (a[j] * scale) * expf(gi - s_g[j]) : 0.f;
          }
          const uint4 xh = pack8(x);
          *reinterpret_cast<uint4*>(dst + sw128(t, q)) = xh;
          if constexpr (kPrecise) {  // P_lo
            float xr[8];
            unpack8(xh, xr);
#pragma unroll
            for (int k = 0; k < 8; ++k) xr[k] = x[k] - xr[k];
            *reinterpret_cast<uint4*>(sm + OFF_PLO + sw128(t, q)) = pack8(xr);
          }
        }
      } else {  // N row i
        const int i = t - C;
        const float gi = s_g[i], bi = s_beta[i];
#pragma unroll
        for (int j = 0; j < C; ++j)
          NM[i * LDN + j] = (j < i) ? -(bi * a[j]) * expf(gi - s_g[j]) : 0.f;
      }
    }
    __syncthreads();

    // ---- 4. T = (I - N)^-1, then T diag(beta), T diag(beta e^gc), Q' --------
    chunk::solve_unit_lower(NM, TM, YM, t, kThreads, [] { __syncthreads(); });
    {
      const int i = t >> 1, jh = (t & 1) * 32;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float x[8], y[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int j = jh + q * 8 + k;
          const float tv = (j <= i) ? TM[i * LDN + j] : 0.f;
          x[k] = tv * s_beta[j];
          y[k] = x[k] * s_eg[j];
        }
        const int ch = (jh >> 3) + q;
        const uint4 xh = pack8(x);
        *reinterpret_cast<uint4*>(sm + OFF_TB + sw128(i, ch)) = xh;
        *reinterpret_cast<uint4*>(sm + OFF_TBE + sw128(i, ch)) = pack8(y);
        if constexpr (kPrecise) {
          float xr[8];
          unpack8(xh, xr);
#pragma unroll
          for (int k = 0; k < 8; ++k) xr[k] = x[k] - xr[k];
          *reinterpret_cast<uint4*>(sm + OFF_TBL + sw128(i, ch)) = pack8(xr);
        }
      }
    }
    {
      const int row = t & 63, h = t >> 6;
      const float f = scale * s_eg[row];
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) {
        float x[8];
        unpack8(*reinterpret_cast<const uint4*>(sm + OFF_QK + h * 16384 + sw128(row, ch)), x);
#pragma unroll
        for (int k = 0; k < 8; ++k) x[k] *= f;
        *reinterpret_cast<uint4*>(sm + OFF_AW + h * 16384 + sw128(64 + row, ch)) = pack8(x);
      }
    }
    tc::fence_async_smem();
    tc::tc_fence_before();
    __syncthreads();

    // ---- 5. D1 = [T diag(beta); 0] V ; Wt = K^T (T diag(beta e^gc))^T -----------
    if constexpr (kPrecise) {
      // the low fp16 half of K into the N matrix's region, dead until the
      // next chunk's G1 epilogue; the state update (step 9) reads it
      if (t == 0) {
        tc::mbar_arrive_expect_tx(bar_tma, 2 * 64 * 64 * 2);
#pragma unroll
        for (int h = 0; h < 2; ++h) tc::tma_load_3d(sm + OFF_KLO + h * 8192, &tmklo, bar_tma, h * 64, c * C, p);
      }
    }
    if (t == 0) {
      tc::tc_fence_after();
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        tc::mma_f16(mD1, tc::sdesc(sbase + OFF_TB + ks * 32, 16, 1024),
                    tc::sdesc(sbase + OFF_V + ks * 2048, 8192, 1024), ID_U, ks > 0);
      if constexpr (kPrecise) {
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          tc::mma_f16(mD1, tc::sdesc(sbase + OFF_TB + ks * 32, 16, 1024),
                      tc::sdesc(sbase + OFF_VLO + ks * 2048, 8192, 1024), ID_U, 1);
          tc::mma_f16(mD1, tc::sdesc(sbase + OFF_TBL + ks * 32, 16, 1024),
                      tc::sdesc(sbase + OFF_V + ks * 2048, 8192, 1024), ID_U, 1);
        }
      }
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        tc::mma_f16(mWT, tc::sdesc(sbase + OFF_QK + 8192 + ks * 2048, 16384, 1024),
                    tc::sdesc(sbase + OFF_TBE + ks * 32, 16, 1024), ID_WT, ks > 0);
      tc::mma_commit(bar_mma);
    }
    if (!wait_mma()) { failed = true; break; }
    tc::tc_fence_after();

    // ---- 6. -W -> AW rows 0..63 (thread t holds column kd = t of W) -------
    {
      float w[64];
      tc::tmem_ld32(tWT, *reinterpret_cast<float(*)[32]>(&w[0]));
      tc::tmem_ld32(tWT + 32, *reinterpret_cast<float(*)[32]>(&w[32]));
      const int h = t >> 6, cc = t & 63, ch = cc >> 3, e = cc & 7;
      uint8_t* base = sm + OFF_AW + h * 16384 + e * 2;
#pragma unroll
      for (int i = 0; i < C; ++i)
        *reinterpret_cast<__half*>(base + sw128(i, ch)) = __float2half_rn(-w[i]);
    }
    tc::fence_async_smem();
    tc::tc_fence_before();
    __syncthreads();

    // ---- 7. D1 += [-W ; Q'] S16 -----------------------------------------------
    if (t == 0) {
      tc::tc_fence_after();
#pragma unroll
      for (int ks = 0; ks < 8; ++ks)
        tc::mma_f16(mD1, tc::sdesc(sbase + OFF_AW + (ks >> 2) * 16384 + (ks & 3) * 32, 16, 1024),
                    tc::sdesc(sbase + OFF_SB + ks * 2048, 16384, 1024), ID_1, 1);
      tc::mma_commit(bar_mma);
    }
    if (!wait_mma()) { failed = true; break; }
    tc::tc_fence_after();

    // ---- 8. v_new rows -> VN, VS (fp16, MN-major [token][v]) -------------------
    if (t < C) {
      const float fs = expf(gL - s_g[t]);
#pragma unroll 1
      for (int cb = 0; cb < 4; ++cb) {
        float v[32];
        tc::tmem_ld32(tD1 + cb * 32, v);
        const int h = cb >> 1;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int ch = (cb & 1) * 4 + q;
          const uint4 vh = pack8(&v[8 * q]);
          *reinterpret_cast<uint4*>(sm + OFF_VN + h * 8192 + sw128(t, ch)) = vh;
          if constexpr (kPrecise) {  // v_new low half into the second half of the dead AW region
            float vr[8];
            unpack8(vh, vr);
#pragma unroll
            for (int k = 0; k < 8; ++k) vr[k] = v[8 * q + k] - vr[k];
            *reinterpret_cast<uint4*>(sm + OFF_AW + 16384 + h * 8192 + sw128(t, ch)) = pack8(vr);
          }
          float y[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) y[k] = v[8 * q + k] * fs;
          const uint4 yh = pack8(y);
          *reinterpret_cast<uint4*>(sm + OFF_VS + h * 8192 + sw128(t, ch)) = yh;
          if constexpr (kPrecise) {  // low half into the dead AW region
            float yr[8];
            unpack8(yh, yr);
#pragma unroll
            for (int k = 0; k < 8; ++k) yr[k] = y[k] - yr[k];
            *reinterpret_cast<uint4*>(sm + OFF_AW + h * 8192 + sw128(t, ch)) = pack8(yr);
          }
        }
      }
    }
    tc::fence_async_smem();
    tc::tc_fence_before();
    __syncthreads();

    // ---- 9. S += K^T VS ; D1 += [0 ; P] VN ---------------------------------------
    if constexpr (kPrecise) {
      ok = tc::mbar_wait_bounded(bar_tma, ph_tma, kWaitLimit);
      ph_tma ^= 1;
      if (__syncthreads_or(!ok)) { failed = true; break; }
    }
    if (t == 0) {
      tc::tc_fence_after();
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        tc::mma_f16(mS, tc::sdesc(sbase + OFF_QK + 8192 + ks * 2048, 16384, 1024),
                    tc::sdesc(sbase + OFF_VS + ks * 2048, 8192, 1024), ID_2A, 1);
      if constexpr (kPrecise) {
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_f16(mS, tc::sdesc(sbase + OFF_QK + 8192 + ks * 2048, 16384, 1024),
                      tc::sdesc(sbase + OFF_AW + ks * 2048, 8192, 1024), ID_2A, 1);
        // K_lo^T VS_hi: fp16 K alone put ~2e-4 relative error into the state
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_f16(mS, tc::sdesc(sbase + OFF_KLO + ks * 2048, 8192, 1024),
                      tc::sdesc(sbase + OFF_VS + ks * 2048, 8192, 1024), ID_2A, 1);
      }
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        tc::mma_f16(mD1, tc::sdesc(sbase + OFF_TB + 8192 + ks * 32, 16, 1024),
                    tc::sdesc(sbase + OFF_VN + ks * 2048, 8192, 1024), ID_1, 1);
      if constexpr (kPrecise) {  // [0;P_hi] VN_lo + [0;P_lo] VN_hi
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          tc::mma_f16(mD1, tc::sdesc(sbase + OFF_TB + 8192 + ks * 32, 16, 1024),
                      tc::sdesc(sbase + OFF_AW + 16384 + ks * 2048, 8192, 1024), ID_1, 1);
          tc::mma_f16(mD1, tc::sdesc(sbase + OFF_TBL + 8192 + ks * 32, 16, 1024),
                      tc::sdesc(sbase + OFF_VN + ks * 2048, 8192, 1024), ID_1, 1);
        }
      }
      tc::mma_commit(bar_mma);
    }
    if (!wait_mma()) { failed = true; break; }
    tc::tc_fence_after();

    // ---- 10. output rows ------------------------------------------------------------
    if (t >= C) {
      const int tok = c * C + (t - C);
#pragma unroll 1
      for (int cb = 0; cb < 4; ++cb) {
        float v[32];
        tc::tmem_ld32(tD1 + cb * 32, v);
        if (tok < S) store_row32<kOut>(out, ((size_t)p * S + tok) * D + cb * 32, v);
      }
    }
    tc::tc_fence_before();
    __syncthreads();
  }

  if (!failed) {
    tc::tc_fence_after();
#pragma unroll 1
    for (int cb = 0; cb < 4; ++cb) {
      float v[32];
      tc::tmem_ld32(tS + cb * 32, v);
      float4* dst = reinterpret_cast<float4*>(final_state + ((size_t)p * D + t) * D + cb * 32);
#pragma unroll
      for (int q = 0; q < 8; ++q) dst[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    }
  } else if (t == 0) {
    atomicExch(err_flag, 1);
    // let outstanding async work land before TMEM is released (bounded)
    tc::mbar_wait_bounded(bar_mma, ph_mma, kWaitLimit);
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tb, 512);
}

// Converts q/k/v to fp16 (optionally L2-normalising q and k per row, eps 1e-6
// inside the sqrt as deltanet_chunk.cpp:27-39) for the tensor-core kernel.
// One warp per 128-wide row.
template <typename Tin>
__global__ void chunk_stage_fp16_kernel(const Tin* __restrict__ x, __half* __restrict__ y,
                                        __half* __restrict__ y_lo, int64_t rows, int l2) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float v[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) v[k] = load_as_f32(x, row * D + lane * 4 + k);
  if (l2) {
    float ss = v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = 1.0f / sqrtf(ss + 1e-6f);
#pragma unroll
    for (int k = 0; k < 4; ++k) v[k] *= inv;
  }
  uint2 o;
  o.x = pack_h2(v[0], v[1]);
  o.y = pack_h2(v[2], v[3]);
  *reinterpret_cast<uint2*>(y + row * D + lane * 4) = o;
  if (y_lo) {  // residual x - fp16(x), itself rounded to fp16
    const __half2* hh = reinterpret_cast<const __half2*>(&o);
    const float2 a = __half22float2(hh[0]), b = __half22float2(hh[1]);
    uint2 r;
    r.x = pack_h2(v[0] - a.x, v[1] - a.y);
    r.y = pack_h2(v[2] - b.x, v[3] - b.y);
    *reinterpret_cast<uint2*>(y_lo + row * D + lane * 4) = r;
  }
}

// Truncating, flush-to-zero fp32 -> fp16 of deltanet_chunk_last_to_fp16.comp:37-66.
__device__ __forceinline__ uint16_t f2h_trunc_ftz(float f) {
  const uint32_t bits = __float_as_uint(f);
  const uint32_t sign = (bits >> 31) & 1u, ex = (bits >> 23) & 0xffu, man = bits & 0x7fffffu;
  const uint16_t hs = (uint16_t)(sign << 15);
  if (ex == 0u) return hs;
  if (ex == 0xffu) return (uint16_t)(hs | 0x7c00u | (man ? 0x200u : 0u));
  const int ne = (int)ex - 127 + 15;
  if (ne <= 0) return hs;
  if (ne >= 31) return (uint16_t)(hs | 0x7c00u);
  return (uint16_t)(hs | ((uint32_t)ne << 10) | (man >> 13));
}

__global__ void last_to_fp16_kernel(const float* __restrict__ core, uint16_t* __restrict__ out,
                                    int64_t batch, int64_t H, int64_t S, int64_t V) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= batch * H * V) return;
  const int64_t bh = idx / V, vd = idx % V;
  out[idx] = f2h_trunc_ftz(core[(bh * S + (S - 1)) * V + vd]);
}

// ---- host side ---------------------------------------------------------------

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 3-D view [pairs][seq][128] of a 16-bit tensor, 64x64 boxes, 128B swizzle.
// Rows past seq_len read as zeros (the reference's zero padding).
Status make_map(CUtensorMap* m, const void* base, int64_t pairs, int64_t S) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return Status::err(SPOCK_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)S, (cuuint64_t)pairs};
  cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)S * D * 2};
  cuuint32_t box[3] = {64, 64, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box,
                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return Status::err(SPOCK_ERR_CUDA, "cuTensorMapEncodeTiled failed (code " + std::to_string((int)r) + ")");
  return Status::ok();
}

}  // namespace
template <bool kBf16, int kOut>
Status launch_chunk_pipeline(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                             const float* g, const float* beta, const float* init, void* out,
                             float* final_state, int64_t pairs, int S, int* err, cudaStream_t st);
namespace {

// fp16/bf16 inputs run the pipelined kernel (chunk_pipeline.cu); fp32 inputs
// run the serial kernel above in its precise (hi/lo) form.
template <bool kBf16In, int kOut, bool kPrecise>
Status launch_kernel(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                     const CUtensorMap& mvlo, const CUtensorMap& mklo, const CUtensorMap& mqlo,
                     const float* g, const float* beta,
                     const float* init, void* out, float* final_state, int64_t pairs, int S, int* err,
                     cudaStream_t st) {
  if constexpr (!kPrecise)
    return launch_chunk_pipeline<kBf16In, kOut>(mq, mk, mv, g, beta, init, out, final_state, pairs, S, err, st);
  auto kern = chunk_rule_kernel<kBf16In, kOut, kPrecise>;
  const int smem = kPrecise ? SMEM_BYTES_PRECISE : SMEM_BYTES;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return cuda_status(e, "chunk_rule_kernel smem attribute");
  kern<<<(unsigned)pairs, kThreads, smem, st>>>(mq, mk, mv, mvlo, mklo, mqlo, g, beta, init, out, final_state, S,
                                                err);
  SPOCK_LAUNCH_CHECK("chunk_rule_kernel");
  return Status::ok();
}

}  // namespace

Status launch_chunk_prefill(ChunkScratch& scratch, const spock_chunk_desc& d, const void* q,
                            const void* k, const void* v, const float* g, const float* beta,
                            const float* init, void* out, float* final_state, int* err_flag,
                            cudaStream_t stream) {
  if (d.key_dim != D || d.value_dim != D || d.chunk_size != C)
    return Status::err(SPOCK_ERR_UNSUPPORTED,
                       "chunk prefill: CUDA path implements key_dim=value_dim=128, chunk_size=64");
  const int64_t pairs = d.batch * d.num_heads;
  if (pairs > 0x7fffffff || d.seq_len > 0x7fffffff)
    return Status::err(SPOCK_ERR_INVALID, "chunk prefill: batch*num_heads and seq_len must fit in int32");
  for (const void* ptr : {q, k, v})
    if ((uintptr_t)ptr & 15) return Status::err(SPOCK_ERR_INVALID, "chunk prefill: q/k/v must be 16-byte aligned");
  if (((uintptr_t)final_state & 15) || ((uintptr_t)out & 15) || ((uintptr_t)init & 15))
    return Status::err(SPOCK_ERR_INVALID, "chunk prefill: outputs and init_state must be 16-byte aligned");

  const int S = (int)d.seq_len;
  const void *q16 = q, *k16 = k, *v16 = v;
  bool bf16 = d.dtype_in == SPOCK_BF16;
  const bool precise = d.dtype_in == SPOCK_F32;
  const void *vlo16 = nullptr, *klo16 = nullptr, *qlo16 = nullptr;
  if (d.dtype_in == SPOCK_F32 || d.use_qk_l2norm) {
    // Stage fp16 copies (the optional L2 norm, and for fp32 inputs the low
    // fp16 half of v) in the context's scratch.
    const size_t n = (size_t)pairs * S * D;
    cudaError_t e = scratch.reserve((precise ? 6 : 3) * n * sizeof(__half));
    if (e != cudaSuccess) return Status::err(SPOCK_ERR_ALLOC, "chunk prefill: scratch allocation failed");
    __half* base = static_cast<__half*>(scratch.buf);
    const int64_t rows = (int64_t)pairs * S;
    const unsigned blocks = (unsigned)((rows + 7) / 8);
    const void* src[3] = {q, k, v};
    for (int i = 0; i < 3; ++i) {
      const int l2 = (i < 2) && d.use_qk_l2norm;
      __half* dst = base + i * n;
      __half* lo = !precise ? nullptr : base + (i == 2 ? 3 : i == 1 ? 4 : 5) * n;
      if (d.dtype_in == SPOCK_F32)
        chunk_stage_fp16_kernel<float><<<blocks, 256, 0, stream>>>((const float*)src[i], dst, lo, rows, l2);
      else if (d.dtype_in == SPOCK_F16)
        chunk_stage_fp16_kernel<__half><<<blocks, 256, 0, stream>>>((const __half*)src[i], dst, lo, rows, l2);
      else
        chunk_stage_fp16_kernel<__nv_bfloat16><<<blocks, 256, 0, stream>>>((const __nv_bfloat16*)src[i], dst, lo, rows, l2);
      SPOCK_LAUNCH_CHECK("chunk_stage_fp16_kernel");
    }
    q16 = base;
    k16 = base + n;
    v16 = base + 2 * n;
    if (precise) {
      vlo16 = base + 3 * n;
      klo16 = base + 4 * n;
      qlo16 = base + 5 * n;
    }
    bf16 = false;
  }
  CUtensorMap mq, mk, mv, mvlo, mklo, mqlo;
  Status s = make_map(&mq, q16, pairs, S);
  if (s.code) return s;
  s = make_map(&mk, k16, pairs, S);
  if (s.code) return s;
  s = make_map(&mv, v16, pairs, S);
  if (s.code) return s;
  s = make_map(&mvlo, precise ? vlo16 : v16, pairs, S);
  if (s.code) return s;
  s = make_map(&mklo, precise ? klo16 : k16, pairs, S);
  if (s.code) return s;
  s = make_map(&mqlo, precise ? qlo16 : q16, pairs, S);
  if (s.code) return s;
#define SPOCK_CHUNK_CASE(BF, OUT, PR)                                                          \
  if (bf16 == BF && d.dtype_out == OUT && precise == PR)                                       \
    return launch_kernel<BF, OUT, PR>(mq, mk, mv, mvlo, mklo, mqlo, g, beta, init, out, final_state, pairs, \
                                      S, err_flag, stream);
  SPOCK_CHUNK_CASE(false, SPOCK_F32, false)
  SPOCK_CHUNK_CASE(false, SPOCK_F16, false)
  SPOCK_CHUNK_CASE(false, SPOCK_BF16, false)
  SPOCK_CHUNK_CASE(true, SPOCK_F32, false)
  SPOCK_CHUNK_CASE(true, SPOCK_F16, false)
  SPOCK_CHUNK_CASE(true, SPOCK_BF16, false)
  SPOCK_CHUNK_CASE(false, SPOCK_F32, true)
  SPOCK_CHUNK_CASE(false, SPOCK_F16, true)
  SPOCK_CHUNK_CASE(false, SPOCK_BF16, true)
#undef SPOCK_CHUNK_CASE
  return Status::err(SPOCK_ERR_INVALID, "chunk prefill: unknown dtype");
}

Status launch_last_to_fp16(int64_t batch, int64_t H, int64_t S, int64_t V, const float* core,
                           void* out, cudaStream_t stream) {
  const int64_t n = batch * H * V;
  last_to_fp16_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(core, (uint16_t*)out, batch, H, S, V);
  SPOCK_LAUNCH_CHECK("last_to_fp16_kernel");
  return Status::ok();
}

}  // namespace spock

// ---------------------------------------------------------------------------
// Allocation-free variant of spock_chunk_prefill.
//
// Some callers cannot allocate device memory at call time: code that runs
// under an allocator it does not own (a host framework's caching allocator or
// a memory pool with a hard budget), code that must not synchronise the
// device (cudaMalloc/cudaFree can), and plugins that receive only the
// caller's buffers and no context. spock_chunk_prefill grows a per-context
// scratch buffer with cudaMalloc when it has to stage fp16 copies of the
// inputs (fp32 inputs, or use_qk_l2norm=1); this variant stages them in a
// fixed array compiled into the library instead and calls no allocator.
// ---------------------------------------------------------------------------
namespace spock {
void record_global_error(const std::string& msg);

namespace {
// Staged tensors hold at most this many elements each (batch*num_heads*
// seq_len*128), i.e. batch*num_heads*seq_len <= 16384 token-heads.
constexpr size_t kNoAllocMaxElems = size_t(1) << 21;
constexpr size_t kNoAllocHeader = 256;  // error word of the bounded waits
constexpr size_t kNoAllocBytes = kNoAllocHeader + 6 * kNoAllocMaxElems * sizeof(__half);  // 24 MiB + 256 B

// Every GPU that loads this library holds this array until the process exits.
// It is shared by all calls on a device and keeps the last call's contents.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_addr[kMaxDevices] = {};

// Device address of g_noalloc_scratch for the current device. In host code the
// symbol's name is only a host-side stand-in, so the address must come from
// cudaGetSymbolAddress, once per device, with that device current.
Status noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "spock_chunk_prefill_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices)
    return Status::err(SPOCK_ERR_UNSUPPORTED, "spock_chunk_prefill_noalloc: device ordinal >= 64");
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_status(e, "spock_chunk_prefill_noalloc: cudaGetSymbolAddress");
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return Status::ok();
}

Status chunk_prefill_noalloc(const spock_chunk_desc& d, const void* q, const void* k, const void* v,
                             const float* g, const float* beta, const float* init, void* out,
                             float* final_state, cudaStream_t stream) {
  if (d.key_dim != D || d.value_dim != D || d.chunk_size != C)
    return Status::err(SPOCK_ERR_UNSUPPORTED,
                       "chunk prefill: CUDA path implements key_dim=value_dim=128, chunk_size=64");
  const int64_t pairs = d.batch * d.num_heads;
  if (pairs > 0x7fffffff || d.seq_len > 0x7fffffff)
    return Status::err(SPOCK_ERR_INVALID, "chunk prefill: batch*num_heads and seq_len must fit in int32");
  for (const void* ptr : {q, k, v})
    if ((uintptr_t)ptr & 15) return Status::err(SPOCK_ERR_INVALID, "chunk prefill: q/k/v must be 16-byte aligned");
  if (((uintptr_t)final_state & 15) || ((uintptr_t)out & 15) || ((uintptr_t)init & 15))
    return Status::err(SPOCK_ERR_INVALID, "chunk prefill: outputs and init_state must be 16-byte aligned");
  const int S = (int)d.seq_len;
  const bool stage = d.dtype_in == SPOCK_F32 || d.use_qk_l2norm;
  const size_t n = (size_t)pairs * S * D;
  if (stage && n > kNoAllocMaxElems)
    return Status::err(SPOCK_ERR_INVALID,
                       "spock_chunk_prefill_noalloc: batch*num_heads*seq_len = " + std::to_string(pairs * (int64_t)S) +
                           " exceeds the fixed scratch of this entry point (max 16384 token-heads when the "
                           "inputs are fp32 or use_qk_l2norm=1); use spock_chunk_prefill");
  void* base_v = nullptr;
  Status s = noalloc_scratch(&base_v);
  if (s.code) return s;
  unsigned char* base = static_cast<unsigned char*>(base_v);
  // The kernels only ever set this word (a bounded wait that gave up). It is
  // not cleared here: spock_noalloc_sync reads it and clears it after reading,
  // so a timeout stays visible until the caller has looked. The staged
  // tensors are fully rewritten by every call.
  int* err_flag = reinterpret_cast<int*>(base);

  const void *q16 = q, *k16 = k, *v16 = v, *vlo16 = nullptr, *klo16 = nullptr, *qlo16 = nullptr;
  bool bf16 = d.dtype_in == SPOCK_BF16;
  const bool precise = d.dtype_in == SPOCK_F32;
  if (stage) {
    __half* st = reinterpret_cast<__half*>(base + kNoAllocHeader);
    const int64_t rows = (int64_t)pairs * S;
    const unsigned blocks = (unsigned)((rows + 7) / 8);
    const void* src[3] = {q, k, v};
    for (int i = 0; i < 3; ++i) {
      const int l2 = (i < 2) && d.use_qk_l2norm;
      __half* dst = st + i * n;
      __half* lo = !precise ? nullptr : st + (i == 2 ? 3 : i == 1 ? 4 : 5) * n;
      if (d.dtype_in == SPOCK_F32)
        chunk_stage_fp16_kernel<float><<<blocks, 256, 0, stream>>>((const float*)src[i], dst, lo, rows, l2);
      else if (d.dtype_in == SPOCK_F16)
        chunk_stage_fp16_kernel<__half><<<blocks, 256, 0, stream>>>((const __half*)src[i], dst, lo, rows, l2);
      else
        chunk_stage_fp16_kernel<__nv_bfloat16><<<blocks, 256, 0, stream>>>((const __nv_bfloat16*)src[i], dst, lo, rows, l2);
      SPOCK_LAUNCH_CHECK("chunk_stage_fp16_kernel");
    }
    q16 = st;
    k16 = st + n;
    v16 = st + 2 * n;
    if (precise) {
      vlo16 = st + 3 * n;
      klo16 = st + 4 * n;
      qlo16 = st + 5 * n;
    }
    bf16 = false;
  }
  CUtensorMap mq, mk, mv, mvlo, mklo, mqlo;
  if ((s = make_map(&mq, q16, pairs, S)).code) return s;
  if ((s = make_map(&mk, k16, pairs, S)).code) return s;
  if ((s = make_map(&mv, v16, pairs, S)).code) return s;
  if ((s = make_map(&mvlo, precise ? vlo16 : v16, pairs, S)).code) return s;
  if ((s = make_map(&mklo, precise ? klo16 : k16, pairs, S)).code) return s;
  if ((s = make_map(&mqlo, precise ? qlo16 : q16, pairs, S)).code) return s;
#define SPOCK_NOALLOC_CASE(BF, OUT, PR)                                                            \
  if (bf16 == BF && d.dtype_out == OUT && precise == PR)                                           \
    return launch_kernel<BF, OUT, PR>(mq, mk, mv, mvlo, mklo, mqlo, g, beta, init, out, final_state, pairs, S, \
                                      err_flag, stream);
  SPOCK_NOALLOC_CASE(false, SPOCK_F32, false)
  SPOCK_NOALLOC_CASE(false, SPOCK_F16, false)
  SPOCK_NOALLOC_CASE(false, SPOCK_BF16, false)
  SPOCK_NOALLOC_CASE(true, SPOCK_F32, false)
  SPOCK_NOALLOC_CASE(true, SPOCK_F16, false)
  SPOCK_NOALLOC_CASE(true, SPOCK_BF16, false)
  SPOCK_NOALLOC_CASE(false, SPOCK_F32, true)
  SPOCK_NOALLOC_CASE(false, SPOCK_F16, true)
  SPOCK_NOALLOC_CASE(false, SPOCK_BF16, true)
#undef SPOCK_NOALLOC_CASE
  return Status::err(SPOCK_ERR_INVALID, "chunk prefill: unknown dtype");
}
}  // namespace

// Device address of the fixed array's error word on the current device (the
// word the allocation-free entry point's kernels set when a bounded wait
// gives up). Used by spock_noalloc_sync and the context-free self-test.
Status noalloc_err_word(int** out) {
  void* base = nullptr;
  Status s = noalloc_scratch(&base);
  if (s.code) return s;
  *out = static_cast<int*>(base);
  return Status::ok();
}

Status noalloc_sync(cudaStream_t stream) {
  cudaError_t e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return cuda_status(e, "spock_noalloc_sync: cudaStreamSynchronize");
  int* word = nullptr;
  Status s = noalloc_err_word(&word);
  if (s.code) return s;
  int flag = 0;
  e = cudaMemcpy(&flag, word, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_status(e, "spock_noalloc_sync: reading the error word");
  if (!flag) return Status::ok();
  e = cudaMemset(word, 0, sizeof(int));  // cleared only now that it has been read
  if (e != cudaSuccess) return cuda_status(e, "spock_noalloc_sync: clearing the error word");
  return Status::err(SPOCK_ERR_TIMEOUT, "spock_noalloc_sync: a kernel's bounded wait gave up (code " +
                                            std::to_string(flag) + ")");
}
}  // namespace spock

extern "C" __attribute__((visibility("default"))) int spock_noalloc_sync(void* stream) {
  spock::Status s = spock::noalloc_sync((cudaStream_t)stream);
  if (s.code) spock::record_global_error(s.msg);
  return s.code;
}

extern "C" __attribute__((visibility("default"))) int spock_chunk_prefill_noalloc(
    const spock_chunk_desc* d, const void* q, const void* k, const void* v, const float* g,
    const float* beta, const float* init_state, void* core_out, float* final_state, void* stream) {
  if (!d) {
    spock::record_global_error("spock_chunk_prefill_noalloc: desc is NULL");
    return SPOCK_ERR_INVALID;
  }
  if (d->batch <= 0 || d->num_heads <= 0 || d->seq_len <= 0 || d->key_dim <= 0 ||
      d->value_dim <= 0 || d->chunk_size <= 0) {
    spock::record_global_error("DeltaNet chunk config fields must be non-zero");
    return SPOCK_ERR_INVALID;
  }
  if (!q || !k || !v || !g || !beta || !core_out || !final_state) {
    spock::record_global_error("spock_chunk_prefill_noalloc: NULL tensor pointer");
    return SPOCK_ERR_INVALID;
  }
  if (d->dtype_in < SPOCK_F32 || d->dtype_in > SPOCK_BF16 || d->dtype_out < SPOCK_F32 ||
      d->dtype_out > SPOCK_BF16) {
    spock::record_global_error("spock_chunk_prefill_noalloc: unknown dtype");
    return SPOCK_ERR_INVALID;
  }
  spock::Status s = spock::chunk_prefill_noalloc(*d, q, k, v, g, beta, init_state, core_out,
                                                 final_state, (cudaStream_t)stream);
  if (s.code) spock::record_global_error(s.msg);
  return s.code;
}
