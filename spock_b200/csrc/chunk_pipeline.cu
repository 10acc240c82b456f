// Warp-specialised, pipelined chunked gated delta rule for sm_100a.
//
// Same mathematics and operand formulation as chunk_rule_kernel (see the
// header of chunk_prefill.cu), reorganised so the tensor cores, TMA and CUDA
// cores overlap. The per-chunk work splits into a state-INDEPENDENT part
// (cumulative g, G1 = [Q;K]K^T, P, N, T = (I-N)^-1, W, Q') and a state-
// DEPENDENT recurrence (S16, U + MMA1, v_new, state update + output). Chunk
// n+1's independent part runs on the PREP warpgroup while chunk n's recurrence
// runs on the REC warpgroup:
//
//   warps 0-7   PREP : g scan, G1 epilogue (P, N), fp32 solve,
//                      T diag(beta e^g) -> MMA, -W and Q' and T diag(beta) -> smem
//   warps 8-11  REC  : bf16->fp16 of V, S -> S16 (+ decay of S in TMEM), v_new
//                      epilogue, output epilogue and stores, initial / final state
//   warp 12     TMA  : q/k tiles (2-stage ring) and v (1 stage)
//   warp 13     MMA  : one thread issues every tcgen05.mma in dependency order
//
// CTAs are persistent (grid <= #SMs) and walk a stream of (pair, chunk) items:
// pair p = blockIdx.x + i*gridDim.x, all of its chunks in order, so the prep
// of a pair's first chunk overlaps the previous pair's last recurrence.
//
// Hand-offs are mbarriers (async proxy + cross-role) and named barriers
// (inside a warpgroup). Every wait is bounded; a timeout sets a shared abort
// flag and *err_flag, every role leaves its loop, TMEM is released.
#include <cuda.h>

#include "chunk_common.cuh"
#include "common.cuh"
#include "tc.cuh"

namespace spock {
namespace pipe {
namespace {

using chunk::C;
using chunk::D;
using chunk::pack8;
using chunk::pack_h2;
using chunk::store_row32;
using chunk::sw128;
using chunk::unpack8;

constexpr int kPrepThreads = 256;  // warps 0-7
constexpr int kRecBase = 256;      // warps 8-11
constexpr int kTmaWarp = 12, kMmaWarp = 13;
constexpr int kThreads = 448;
constexpr uint32_t kWaitLimit = 1u << 25;  // >= ~4 s of polling with back-off

// Shared memory (offsets from a 1024-aligned base).
constexpr int OFF_QK = 0;                    // 2 stages x 32K: per column half [Q 8K | K 8K]
constexpr int OFF_AW = 64 * 1024;            // [-W ; Q'] K-major 128x128 (2 halves x 16K)
constexpr int OFF_TB = 96 * 1024;            // [T diag(beta) 8K | zero 8K | P 8K]
constexpr int OFF_TBE = 120 * 1024;          // T diag(beta e^gc), K-major 64x64
constexpr int OFF_V = 128 * 1024;            // V, 2 halves x 8K
constexpr int OFF_SB = 144 * 1024;           // S16 MN-major [kd][v]; later VN | VS
constexpr int OFF_VN = OFF_SB;
constexpr int OFF_VS = OFF_SB + 16 * 1024;
constexpr int OFF_NM = 176 * 1024;
constexpr int OFF_TM = OFF_NM + C * chunk::LDT * 4;  // N and T: 64 x LDT fp32
constexpr int OFF_YM = OFF_TM + C * chunk::LDT * 4;  // solve scratch: 32 x kLDY fp32
constexpr int OFF_SMALL = OFF_YM + 32 * chunk::kLDY * 4;
constexpr int SMALL_BYTES = 4096;
constexpr int SMEM_BYTES = OFF_SMALL + SMALL_BYTES + 1024;
static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");

enum Bar {
  QK_FULL0, QK_FULL1, QK_EMPTY0, QK_EMPTY1, V_FULL, V_EMPTY, PREP_A, G1_DONE0, G1_DONE1, TBE_READY, WT_DONE,
  PREP_DONE, S16_READY, M1_DONE, VN_READY, M2_DONE, V_CONV, AW_READY, GC_READY0, GC_READY1, D1_FREE, DRAIN,
  NUM_BARS
};

struct Small {
  float gc[2][C];    // cumulative g per stage
  float beta[2][C];
  float eg[2][C];    // exp(gc)
  float gl[2][C];    // gc * log2(e)
  float graw[2][C];  // g, beta of an item, prefetched by cp.async one item ahead
  float braw[2][C];
  uint64_t bar[NUM_BARS];
  uint32_t tmem_base;
  int abort;
};
static_assert(sizeof(Small) <= SMALL_BYTES, "small region");

constexpr float kLog2e = 1.4426950408889634f;
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Barrier over one warpgroup (named barrier `id`, 128 threads) that also ORs a
// predicate, so every thread of the group takes the same branch afterwards.
__device__ __forceinline__ bool group_any(int id, int nthreads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 q, %1, 0;\n"
      " bar.red.or.pred p, %2, %3, q;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void group_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// 4-byte asynchronous global->shared copy; src_bytes 0 writes a zero.
__device__ __forceinline__ void cp_async4(void* dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(tc::smem_u32(dst)), "l"(src),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Bounded wait that also gives up early once another role has aborted.
// mbarrier.try_wait suspends the thread in hardware until the phase completes
// or a short time limit passes, so the loop neither spins hot nor oversleeps.
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, volatile int* abort) {
  if (*abort) return false;
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    if (tc::mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 255u && *abort) return false;
  }
  return false;
}

// Optional per-phase cycle accounting (compile with -DSPOCK_PHASE_PROF; never
// in the shipped library): one row of 32 counters per CTA and role. With
// -DSPOCK_TRACE_ONLY only the per-item event timestamps of CTA 0 are kept
// (one clock read per event), which perturbs the timing far less.
#if defined(SPOCK_TRACE_ONLY) && !defined(SPOCK_PHASE_PROF)
__device__ long long g_trace[64 * 32];
#define TRACE(ev, n)                                                                 \
  do {                                                                               \
    if (blockIdx.x == 0 && (n) < 64) g_trace[(n) * 32 + (ev)] = clock64();           \
  } while (0)
#define PROF_DECL
#define PROF_MARK(role, k) \
  do {                     \
  } while (0)
#define PROF_FLUSH(role) \
  do {                   \
  } while (0)
#elif defined(SPOCK_PHASE_PROF)
__device__ unsigned long long g_phase_prof[148 * 4 * 32];
#define PROF_DECL                       \
  long long _pt = clock64();            \
  unsigned long long _acc[32] = {};
#define PROF_MARK(role, k)                                  \
  do {                                                      \
    long long _now = clock64();                             \
    _acc[k] += (unsigned long long)(_now - _pt);            \
    _pt = _now;                                             \
  } while (0)
#define PROF_FLUSH(role)                                                        \
  do {                                                                          \
    if ((threadIdx.x & 127) == 0 && blockIdx.x < 148)                           \
      for (int _k = 0; _k < 32; ++_k) g_phase_prof[(blockIdx.x * 4 + (role)) * 32 + _k] += _acc[_k]; \
  } while (0)
__device__ long long g_trace[64 * 32];
#define TRACE(ev, n)                                                                 \
  do {                                                                               \
    if (blockIdx.x == 0 && (n) < 64) g_trace[(n) * 32 + (ev)] = clock64();           \
  } while (0)
#else
#define TRACE(ev, n) \
  do {               \
  } while (0)
#define PROF_DECL
#define PROF_MARK(role, k) \
  do {                     \
  } while (0)
#define PROF_FLUSH(role) \
  do {                   \
  } while (0)
#endif

struct Items {
  int nch, pairs, S;
  __device__ int count() const {
    const int my_pairs = pairs > (int)blockIdx.x ? (pairs - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    return my_pairs * nch;
  }
  __device__ int pair(int n) const { return (int)blockIdx.x + (n / nch) * (int)gridDim.x; }
  __device__ int chunk(int n) const { return n % nch; }
};

// ---- TMA producer (one thread) -------------------------------------------------
__device__ void tma_role(uint8_t* sm, Small* sh, const CUtensorMap* mq, const CUtensorMap* mk,
                         const CUtensorMap* mv, Items it, int* err) {
  volatile int* abort = &sh->abort;
  const int N = it.count();
  // Greedy: the q/k ring and the single V buffer are refilled independently,
  // each in item order, as soon as their consumers release them.
  int nq = 0, nv = 0;
  uint32_t idle = 0;
  while (nq < N || nv < N) {
    bool progressed = false;
    if (nq < N && tc::mbar_test_wait(&sh->bar[QK_EMPTY0 + (nq & 1)], ((nq >> 1) & 1) ^ 1)) {
      const int s = nq & 1, p = it.pair(nq), c = it.chunk(nq);
      tc::mbar_arrive_expect_tx(&sh->bar[QK_FULL0 + s], 4 * 64 * 64 * 2);
      for (int h = 0; h < 2; ++h) {
        uint8_t* base = sm + OFF_QK + s * 32768 + h * 16384;
        tc::tma_load_3d(base, mq, &sh->bar[QK_FULL0 + s], h * 64, c * C, p);
        tc::tma_load_3d(base + 8192, mk, &sh->bar[QK_FULL0 + s], h * 64, c * C, p);
      }
      TRACE(0, nq);
      ++nq;
      progressed = true;
    }
    if (nv < N && tc::mbar_test_wait(&sh->bar[V_EMPTY], (nv & 1) ^ 1)) {
      tc::mbar_arrive_expect_tx(&sh->bar[V_FULL], 2 * 64 * 64 * 2);
      for (int h = 0; h < 2; ++h)
        tc::tma_load_3d(sm + OFF_V + h * 8192, mv, &sh->bar[V_FULL], h * 64, it.chunk(nv) * C, it.pair(nv));
      TRACE(1, nv);
      ++nv;
      progressed = true;
    }
    if (progressed) {
      idle = 0;
    } else {
      if (++idle > kWaitLimit || *abort) goto fail;
    }
  }
  return;
fail:
  sh->abort = 1;
  atomicExch(err, 2);
}

// ---- MMA issuer (one thread) -----------------------------------------------------
template <bool kBf16>
__device__ void mma_role(uint8_t* sm, Small* sh, uint32_t tb, Items it, int* err) {
  volatile int* abort = &sh->abort;
  const uint32_t sbase = tc::smem_u32(sm);
  // TMEM: S [0,128), D1 [128,256), G1 x2 [256,384), W^T [384,448)
  const uint32_t mS = tb, mD1 = tb + 128, mG1 = tb + 256, mWT = tb + 384;
  // G1 reads the raw input tiles (bf16 or fp16); every other product is fp16
  constexpr uint32_t ID_G1 = tc::idesc_f16(128, 64, false, false) | (kBf16 ? (1u << 7) | (1u << 10) : 0u);
  constexpr uint32_t ID_U = tc::idesc_f16(128, 128, false, true);
  constexpr uint32_t ID_WT = tc::idesc_f16(128, 64, true, false);
  constexpr uint32_t ID_2A = tc::idesc_f16(128, 128, true, true);
  const int N = it.count();

  {
    // Greedy issue: each of the four MMA queues stays in item order, and
    // whichever queue's next group is ready goes first, so the prep of item
    // n+1 (G1, W^T) is not held behind the recurrence of item n.
    int g1 = 0, wt = 0, uu = 0, um = 0, m2 = 0, pa = 0;
    uint32_t idle = 0;
#ifdef SPOCK_PHASE_PROF
    long long iters = 0;
#endif
    while (m2 < N) {
#ifdef SPOCK_PHASE_PROF
      ++iters;
#endif
      bool progressed = false;
      if (m2 < um && tc::mbar_test_wait(&sh->bar[VN_READY], m2 & 1)) {
        // state update + output of item m2: S += K^T VS ; D1 += [0 ; P] VN
        tc::tc_fence_after();
        const uint32_t k = sbase + OFF_QK + (m2 & 1) * 32768 + 8192;
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_f16(mS, tc::sdesc(k + ks * 2048, 16384, 1024), tc::sdesc(sbase + OFF_VS + ks * 2048, 8192, 1024),
                      ID_2A, 1);
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_f16(mD1, tc::sdesc(sbase + OFF_TB + 8192 + ks * 32, 16, 1024),
                      tc::sdesc(sbase + OFF_VN + ks * 2048, 8192, 1024), ID_U, 1);
        tc::mma_commit(&sh->bar[M2_DONE]);
        tc::mma_commit(&sh->bar[QK_EMPTY0 + (m2 & 1)]);
        TRACE(5, m2);
#ifdef SPOCK_PHASE_PROF
        if (blockIdx.x == 0 && m2 < 64) g_trace[m2 * 32 + 26] = iters;
#endif
        ++m2;
        progressed = true;
      }
      // U of item uu as soon as D1 is free (the REC group has stored the
      // previous item's output rows) and PREP has published T diag(beta) and V:
      // it then runs while the REC group builds -W and Q'
      if (uu < N && uu == um && uu == m2 && tc::mbar_test_wait(&sh->bar[PREP_DONE], uu & 1) &&
          tc::mbar_test_wait(&sh->bar[D1_FREE], uu & 1)) {
        tc::tc_fence_after();
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_f16(mD1, tc::sdesc(sbase + OFF_TB + ks * 32, 16, 1024),
                      tc::sdesc(sbase + OFF_V + ks * 2048, 8192, 1024), ID_U, ks > 0);
        ++uu;
        progressed = true;
      }
      if (um < wt && um < uu && tc::mbar_test_wait(&sh->bar[S16_READY], um & 1) &&
          tc::mbar_test_wait(&sh->bar[AW_READY], um & 1)) {
        // MMA1 of item um: D1 (= [T diag(beta); 0] V) += [-W ; Q'] S16
        tc::tc_fence_after();
        for (int ks = 0; ks < 8; ++ks)
          tc::mma_f16(mD1, tc::sdesc(sbase + OFF_AW + (ks >> 2) * 16384 + (ks & 3) * 32, 16, 1024),
                      tc::sdesc(sbase + OFF_SB + ks * 2048, 16384, 1024), ID_U, 1);
        tc::mma_commit(&sh->bar[M1_DONE]);
        tc::mma_commit(&sh->bar[V_EMPTY]);
        TRACE(4, um);
        ++um;
        progressed = true;
      }
      // W^T of item wt overwrites W^T of item wt-1 in TMEM: the REC warps
      // must have read that one first (they did once MMA1 of wt-1 is issued,
      // which waits for their AW_READY).
      if (wt < g1 && wt <= um && tc::mbar_test_wait(&sh->bar[TBE_READY], wt & 1)) {
        tc::tc_fence_after();
        const uint32_t k = sbase + OFF_QK + (wt & 1) * 32768 + 8192;
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_f16(mWT, tc::sdesc(k + ks * 2048, 16384, 1024), tc::sdesc(sbase + OFF_TBE + ks * 32, 16, 1024),
                      ID_WT, ks > 0);
        tc::mma_commit(&sh->bar[WT_DONE]);
        TRACE(3, wt);
        ++wt;
        progressed = true;
      }
      // prep has started item pa-1 (so it is done reading G1 of item pa-2)
      if (pa < N && tc::mbar_test_wait(&sh->bar[PREP_A], pa & 1)) {
        ++pa;
        progressed = true;
      }
      // G1 straight from the landed q/k tile, into the TMEM buffer of g1 & 1
      if (g1 < N && (g1 < 2 || pa >= g1 - 1) && tc::mbar_test_wait(&sh->bar[QK_FULL0 + (g1 & 1)], (g1 >> 1) & 1)) {
        tc::tc_fence_after();
        const uint32_t qk = sbase + OFF_QK + (g1 & 1) * 32768;
        for (int ks = 0; ks < 8; ++ks) {
          const uint32_t koff = (ks >> 2) * 16384 + (ks & 3) * 32;
          tc::mma_f16(mG1 + (g1 & 1) * 64, tc::sdesc(qk + koff, 16, 1024), tc::sdesc(qk + 8192 + koff, 16, 1024),
                      ID_G1, ks > 0);
        }
        tc::mma_commit(&sh->bar[G1_DONE0 + (g1 & 1)]);
        TRACE(2, g1);
        ++g1;
        progressed = true;
      }
      if (progressed) {
        idle = 0;
      } else {
        if (++idle > kWaitLimit || *abort) goto fail;
      }
    }
  }
  return;
fail:
  sh->abort = 1;
  atomicExch(err, 2);
  // let MMAs already issued finish before TMEM is released (bounded)
  tc::mma_commit(&sh->bar[DRAIN]);
  for (uint32_t i = 0; i < kWaitLimit && !tc::mbar_test_wait(&sh->bar[DRAIN], 0); ++i) {
  }
}

__device__ __forceinline__ void bf16_to_f16_inplace(uint4* p, int n16, int t, int nt) {
  for (int i = t; i < n16; i += nt) {
    uint4 u = p[i];
    uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float2 f = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&w[k]));
      w[k] = pack_h2(f.x, f.y);
    }
    p[i] = u;
  }
}

constexpr int BAR_PREP = 1, BAR_REC = 2;  // named barriers of the two warpgroups

// ---- PREP (warps 0-7, 256 threads; TMEM lane l = t & 127, column half hf = t >> 7) ----
template <bool kBf16>
__device__ void prep_role(uint8_t* sm, Small* sh, uint32_t tb, Items it, const float* __restrict__ g,
                          const float* __restrict__ beta, int* err) {
  volatile int* abort = &sh->abort;
  const int t = threadIdx.x, l = t & 127, hf = t >> 7;
  const uint32_t lane_base = (uint32_t)((l >> 5) * 32) << 16;
  const uint32_t tG1 = tb + 256 + lane_base + hf * 32;  // + (n & 1) * 64: double buffer
  float* NM = reinterpret_cast<float*>(sm + OFF_NM);
  float* TM = reinterpret_cast<float*>(sm + OFF_TM);
  float* YM = reinterpret_cast<float*>(sm + OFF_YM);
  const float scale = 0.08838834764831845f;
  const int N = it.count();
  auto sync = [] { group_sync(BAR_PREP, kPrepThreads); };
  // Waits are per thread (no barrier): a thread whose wait gives up sets the
  // shared abort flag, later waits return at once, and every thread still
  // runs the item to its end, where one group-wide OR decides to leave.
  bool bad = false;
  auto wait_all = [&](int b, uint32_t parity) { bad |= !wait_bar(&sh->bar[b], parity, abort); };
  auto prefetch_gb = [&](int n) {  // cp.async by the thread of each token; waited for at item n
    if (n < N && t < C) {
      const int tok = it.chunk(n) * C + t;
      const bool in = tok < it.S;
      const size_t idx = in ? (size_t)it.pair(n) * it.S + tok : 0;
      cp_async4(&sh->graw[n & 1][t], g + idx, in ? 4u : 0u);
      cp_async4(&sh->braw[n & 1][t], beta + idx, in ? 4u : 0u);
    }
    cp_async_commit();
  };
  prefetch_gb(0);
  // the solve reads the strictly upper blocks T[0:16,16:32] and T[32:48,48:64]
  // as zeros and never writes them
  for (int i = t; i < C * chunk::LDT; i += kPrepThreads) TM[i] = 0.f;
  sync();

  PROF_DECL
  for (int n = 0; n < N; ++n) {
    const int s = n & 1;
    uint8_t* qk = sm + OFF_QK + s * 32768;
    if (t == 0) TRACE(6, n);
    // 1. cumulative g (shuffle scan over two warps); g/beta of n+1 prefetched
    {
      __shared__ float s_warp_total;
      float gv = 0.f, bv = 0.f;
      cp_async_wait_all();
      if (t < C) {
        gv = sh->graw[s][t];
        bv = sh->braw[s][t];
      }
      prefetch_gb(n + 1);
      if (t < C) {
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float y = __shfl_up_sync(0xffffffffu, gv, o);
          if ((t & 31) >= o) gv += y;
        }
        if (t == 31) s_warp_total = gv;
      }
      sync();
      if (t < C) {
        if (t >= 32) gv += s_warp_total;
        sh->gc[s][t] = gv;
        sh->gl[s][t] = gv * kLog2e;
        sh->beta[s][t] = bv;
        sh->eg[s][t] = ex2(gv * kLog2e);
      }
    }
    PROF_MARK(0, 0);
    // 2. q/k tile landed: convert, publish for G1
    wait_all(QK_FULL0 + s, (n >> 1) & 1);
    if (t == 0) TRACE(7, n);
    PROF_MARK(0, 1);
    sync();
    if (t == 0) {
      tc::mbar_arrive_expect_tx(&sh->bar[PREP_A], 0);
      // per-stage copy for the REC warps: they may lag this prep by more than
      // one item, which a single barrier's parity could not tell apart
      tc::mbar_arrive_expect_tx(&sh->bar[GC_READY0 + s], 0);
    }
    PROF_MARK(0, 2);
    // 3. G1 epilogue on 32 columns: P row (kept in registers) or N row. The
    //    decay factors (and scale / -beta) are formed while G1 is in flight.
    uint4 preg[4];
    {
      const float* gl = sh->gl[s];
      const int j0 = hf * 32, row = l & 63;
      const float gi = gl[row];
      const float f = (l < C) ? scale : -sh->beta[s][row];
      float dec[32];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 v4 = *reinterpret_cast<const float4*>(gl + j0 + 4 * q);
        const float gj[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int j = j0 + 4 * q + k;
          const bool keep = (l < C) ? (j <= row) : (j < row);
          dec[4 * q + k] = keep ? f * ex2(gi - gj[k]) : 0.f;
        }
      }
      wait_all(G1_DONE0 + (n & 1), (n >> 1) & 1);
      if (t == 0) TRACE(8, n);
      PROF_MARK(0, 3);
      tc::tc_fence_after();
      float a[32];
      tc::tmem_ld32(tG1 + (n & 1) * 64, a);
      if (l < C) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float x[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) x[k] = a[q * 8 + k] * dec[q * 8 + k];
          preg[q] = pack8(x);
        }
      } else {
        const int i = l - C;
#pragma unroll
        for (int k = 0; k < 32; k += 4)
          *reinterpret_cast<float4*>(NM + i * chunk::LDT + j0 + k) =
              make_float4(a[k] * dec[k], a[k + 1] * dec[k + 1], a[k + 2] * dec[k + 2], a[k + 3] * dec[k + 3]);
      }
    }
    if constexpr (kBf16) {  // K -> fp16 in place (G1, the only bf16 reader, is done)
      bf16_to_f16_inplace(reinterpret_cast<uint4*>(qk + 8192), 8192 / 16, t, kPrepThreads);
      bf16_to_f16_inplace(reinterpret_cast<uint4*>(qk + 16384 + 8192), 8192 / 16, t, kPrepThreads);
      tc::fence_async_smem();
    }
    tc::tc_fence_before();
    sync();
    PROF_MARK(0, 4);
    if (t == 0) TRACE(9, n);
    // 4. T = (I - N)^-1
#ifdef SPOCK_PHASE_PROF
    {
      int kk = 16;
      auto sync_prof = [&] {
        PROF_MARK(0, kk);
        ++kk;
        sync();
        PROF_MARK(0, kk);
        ++kk;
      };
      chunk::solve_unit_lower_blk(NM, TM, YM, t, sync_prof);
    }
#else
    chunk::solve_unit_lower_blk(NM, TM, YM, t, sync);
#endif
    PROF_MARK(0, 5);
    if (t == 0) TRACE(10, n);
    // 5. T diag(beta e^gc) -> TBE (for W^T) once W^T of the previous item has
    //    read it; T diag(beta) kept in registers
    if (n > 0) wait_all(WT_DONE, (n - 1) & 1);
    uint4 tbreg[2];
    {
      const int i = t >> 2;
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int ch = (t & 3) * 2 + q, j0 = ch * 8;
        float x[8], y[8];
        const float4 t0 = *reinterpret_cast<const float4*>(TM + i * chunk::LDT + j0);
        const float4 t1 = *reinterpret_cast<const float4*>(TM + i * chunk::LDT + j0 + 4);
        const float tr[8] = {t0.x, t0.y, t0.z, t0.w, t1.x, t1.y, t1.z, t1.w};
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int j = j0 + k;
          const float tv = (j <= i) ? tr[k] : 0.f;
          x[k] = tv * sh->beta[s][j];
          y[k] = x[k] * sh->eg[s][j];
        }
        tbreg[q] = pack8(x);
        *reinterpret_cast<uint4*>(sm + OFF_TBE + sw128(i, ch)) = pack8(y);
      }
    }
    tc::fence_async_smem();
    sync();
    if (t == 0) tc::mbar_arrive_expect_tx(&sh->bar[TBE_READY], 0);
    if (t == 0) TRACE(11, n);
    PROF_MARK(0, 6);
    // 6. once MMA1 of the previous item has read them: T diag(beta) and Q'
    if (n > 0) wait_all(M1_DONE, (n - 1) & 1);
    PROF_MARK(0, 7);
    if (t == 0) TRACE(12, n);
    {
      const int i = t >> 2;
#pragma unroll
      for (int q = 0; q < 2; ++q) *reinterpret_cast<uint4*>(sm + OFF_TB + sw128(i, (t & 3) * 2 + q)) = tbreg[q];
    }
    PROF_MARK(0, 8);
    // 8. once the previous item's output MMA has read it: P
    if (n > 0) wait_all(M2_DONE, (n - 1) & 1);
    PROF_MARK(0, 11);
    if (t == 0) TRACE(13, n);
    if (l < C) {
#pragma unroll
      for (int q = 0; q < 4; ++q)
        *reinterpret_cast<uint4*>(sm + OFF_TB + 16384 + sw128(l, hf * 4 + q)) = preg[q];
    }
    PROF_MARK(0, 12);
    // 9. V of this item (converted to fp16 by the REC warpgroup)
    wait_all(V_CONV, n & 1);
    PROF_MARK(0, 13);
    if (t == 0) TRACE(14, n);
    tc::fence_async_smem();
    if (group_any(BAR_PREP, kPrepThreads, bad)) break;
    if (t == 0) tc::mbar_arrive_expect_tx(&sh->bar[PREP_DONE], 0);
    if (t == 0) TRACE(15, n);
    PROF_MARK(0, 14);
  }
  cp_async_wait_all();
  PROF_FLUSH(0);
  if (*abort && t == 0) atomicExch(err, 2);
}

// ---- REC warpgroup (warps 4-7; rt <-> TMEM lane rt) --------------------------------------
template <bool kBf16, int kOut>
__device__ void rec_role(uint8_t* sm, Small* sh, uint32_t tb, Items it, const float* __restrict__ init,
                         void* __restrict__ out, float* __restrict__ final_state, int* err) {
  volatile int* abort = &sh->abort;
  const int rt = threadIdx.x - kRecBase;
  const uint32_t lane_base = (uint32_t)((rt >> 5) * 32) << 16;
  const uint32_t tS = tb + lane_base, tD1 = tb + 128 + lane_base, tWT = tb + 384 + lane_base;
  int N = it.count();
  auto sync = [] { group_sync(BAR_REC, 128); };
  // per-thread waits; one group-wide OR per item decides to leave (as in PREP)
  bool bad = false;
  auto wait_all = [&](int b, uint32_t parity) { bad |= !wait_bar(&sh->bar[b], parity, abort); };

  // V of item m -> fp16 in place, then published to PREP as V_CONV
  auto convert_v = [&](int m) {
    wait_all(V_FULL, m & 1);
    if constexpr (kBf16) {
      bf16_to_f16_inplace(reinterpret_cast<uint4*>(sm + OFF_V), 16384 / 16, rt, 128);
      tc::fence_async_smem();
    }
    sync();
    if (rt == 0) tc::mbar_arrive_expect_tx(&sh->bar[V_CONV], 0);
  };
  if (N > 0) convert_v(0);
  // output rows of item m (TMEM lanes 64..127 of D1)
  auto store_out = [&](int m) {
    if (rt >= C) {
      const int tok = it.chunk(m) * C + (rt - C);
      const size_t row = (size_t)it.pair(m) * it.S + tok;
#pragma unroll 1
      for (int cb = 0; cb < 4; ++cb) {
        float v[32];
        tc::tmem_ld32(tD1 + cb * 32, v);
        if (tok < it.S) store_row32<kOut>(out, row * D + cb * 32, v);
      }
    }
  };

  PROF_DECL
  for (int n = 0; n < N; ++n) {
    const int s = n & 1, p = it.pair(n), c = it.chunk(n);
    // 1. first chunk of a pair: initial state -> TMEM (row rt = key index)
    if (c == 0) {
      const float* src = init ? init + ((size_t)p * D + rt) * D : nullptr;
#pragma unroll 1
      for (int cb = 0; cb < 4; ++cb) {
        float v[32];
        if (src) {
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 x = reinterpret_cast<const float4*>(src + cb * 32)[q];
            v[4 * q] = x.x; v[4 * q + 1] = x.y; v[4 * q + 2] = x.z; v[4 * q + 3] = x.w;
          }
        } else {
#pragma unroll
          for (int k = 0; k < 32; ++k) v[k] = 0.f;
        }
        tc::tmem_st32(tS + cb * 32, v);
      }
      tc::tmem_st_wait();
    }
    PROF_MARK(1, 0);
    if (rt == 0) TRACE(16, n);
    // 2. S16 <- S ; S <- e^{gL} S
    wait_all(GC_READY0 + s, (n >> 1) & 1);
    PROF_MARK(1, 1);
    if (rt == 0) TRACE(17, n);
    const float egL = sh->eg[s][C - 1];
    tc::tc_fence_after();
#pragma unroll 1
    for (int cb = 0; cb < 4; ++cb) {
      float v[32];
      tc::tmem_ld32(tS + cb * 32, v);
      uint8_t* dst = sm + OFF_SB + (cb >> 1) * 16384;
#pragma unroll
      for (int q = 0; q < 4; ++q) *reinterpret_cast<uint4*>(dst + sw128(rt, (cb & 1) * 4 + q)) = pack8(&v[8 * q]);
#pragma unroll
      for (int k = 0; k < 32; ++k) v[k] = mul_rn(v[k], egL);
      tc::tmem_st32(tS + cb * 32, v);
    }
    tc::tmem_st_wait();
    tc::fence_async_smem();
    tc::tc_fence_before();
    sync();
    if (rt == 0) tc::mbar_arrive_expect_tx(&sh->bar[S16_READY], 0);
    if (rt == 0) TRACE(18, n);
    // output of the previous item, off the S16 path; D1 is next written by
    // MMA1 of this item, which waits for AW_READY below
    if (n > 0) {
      wait_all(M2_DONE, (n - 1) & 1);  // the previous item's output MMAs
      tc::tc_fence_after();
      store_out(n - 1);
    }
    // D1 is free for this item's U (its previous rows have all been read)
    tc::tc_fence_before();
    sync();
    if (rt == 0) tc::mbar_arrive_expect_tx(&sh->bar[D1_FREE], 0);
    // 2b. A operand of MMA1: -W (from W^T in TMEM) and Q' = diag(s e^gc) Q.
    //     MMA1 of the previous item, the last reader of AW, has completed.
    wait_all(WT_DONE, n & 1);
    if (rt == 0) TRACE(19, n);
    tc::tc_fence_after();
    {
      float w[64];
      tc::tmem_ld32(tWT, *reinterpret_cast<float(*)[32]>(&w[0]));
      tc::tmem_ld32(tWT + 32, *reinterpret_cast<float(*)[32]>(&w[32]));
      // lanes kd, kd^1 hold adjacent columns: exchange so that each stores one
      // 32-bit pair (even lane: even rows, odd lane: odd rows)
      const int h = rt >> 6, cc = rt & 63, ch = cc >> 3, e = cc & 6, odd = rt & 1;
      uint8_t* base = sm + OFF_AW + h * 16384 + e * 2;
#pragma unroll
      for (int k = 0; k < 64; k += 2) {
        const float mine = odd ? w[k] : w[k + 1];
        const float other = __shfl_xor_sync(0xffffffffu, mine, 1);
        const float lo = odd ? other : w[k], hi = odd ? w[k + 1] : other;
        *reinterpret_cast<uint32_t*>(base + sw128(k + odd, ch)) = pack_h2(-lo, -hi);
      }
      const uint8_t* qk = sm + OFF_QK + s * 32768;
      const int row = rt & 63, hq = rt >> 6;
      const float f = 0.08838834764831845f * sh->eg[s][row];
#pragma unroll
      for (int ch2 = 0; ch2 < 8; ++ch2) {
        float x[8];
        const uint4 raw = *reinterpret_cast<const uint4*>(qk + hq * 16384 + sw128(row, ch2));
        if constexpr (kBf16) {
          const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float2 f2 = __bfloat1622float2(b2[k]);
            x[2 * k] = f2.x;
            x[2 * k + 1] = f2.y;
          }
        } else {
          unpack8(raw, x);
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) x[k] *= f;
        *reinterpret_cast<uint4*>(sm + OFF_AW + hq * 16384 + sw128(64 + row, ch2)) = pack8(x);
      }
    }
    tc::fence_async_smem();
    tc::tc_fence_before();
    sync();
    if (rt == 0) tc::mbar_arrive_expect_tx(&sh->bar[AW_READY], 0);
    if (rt == 0) TRACE(20, n);
    PROF_MARK(1, 2);
    // 3. v_new rows (lanes 0..63) -> VN, VS
    wait_all(M1_DONE, n & 1);
    PROF_MARK(1, 3);
    if (rt == 0) TRACE(21, n);
    tc::tc_fence_after();
    if (rt < C) {
      const float fs = ex2((sh->gc[s][C - 1] - sh->gc[s][rt]) * kLog2e);
#pragma unroll 1
      for (int cb = 0; cb < 4; ++cb) {
        float v[32];
        tc::tmem_ld32(tD1 + cb * 32, v);
        const int h = cb >> 1;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int ch = (cb & 1) * 4 + q;
          *reinterpret_cast<uint4*>(sm + OFF_VN + h * 8192 + sw128(rt, ch)) = pack8(&v[8 * q]);
          float y[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) y[k] = v[8 * q + k] * fs;
          *reinterpret_cast<uint4*>(sm + OFF_VS + h * 8192 + sw128(rt, ch)) = pack8(y);
        }
      }
    }
    tc::fence_async_smem();
    tc::tc_fence_before();
    sync();
    if (rt == 0) tc::mbar_arrive_expect_tx(&sh->bar[VN_READY], 0);
    if (rt == 0) TRACE(22, n);
    if (n + 1 < N) convert_v(n + 1);
    PROF_MARK(1, 4);
    if (rt == 0) TRACE(23, n);
    // 4. final state after a pair's last chunk (the output rows are stored
    //    at the next item, or after the loop). All of M2 must be complete, not
    //    just the state update: the next item's S16 overwrites VN/VS, which
    //    the output MMA reads.
    wait_all(M2_DONE, n & 1);
    PROF_MARK(1, 5);
    if (rt == 0) TRACE(24, n);
    tc::tc_fence_after();
    if (c == it.nch - 1) {
#pragma unroll 1
      for (int cb = 0; cb < 4; ++cb) {
        float v[32];
        tc::tmem_ld32(tS + cb * 32, v);
        float4* dst = reinterpret_cast<float4*>(final_state + ((size_t)p * D + rt) * D + cb * 32);
#pragma unroll
        for (int q = 0; q < 8; ++q) dst[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
      }
    }
    tc::tc_fence_before();
    PROF_MARK(1, 6);
    if (rt == 0) TRACE(25, n);
    if (group_any(BAR_REC, 128, bad)) break;
  }
  if (N > 0 && !*abort) {
    wait_all(M2_DONE, (N - 1) & 1);
    tc::tc_fence_after();
    store_out(N - 1);
  }
  PROF_FLUSH(1);
  if (*abort && rt == 0) atomicExch(err, 2);
}

template <bool kBf16, int kOut>
__global__ void __launch_bounds__(kThreads, 1)
    chunk_pipe_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                      const __grid_constant__ CUtensorMap tmv, const float* __restrict__ g,
                      const float* __restrict__ beta, const float* __restrict__ init, void* __restrict__ out,
                      float* __restrict__ final_state, int S, int pairs, int* __restrict__ err_flag) {
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment by pointer arithmetic on the __shared__ array keeps the
  // shared address space visible to the compiler (LDS/STS, not generic loads).
  uint8_t* sm = smem_raw + ((1024u - (tc::smem_u32(smem_raw) & 1023u)) & 1023u);
  Small* sh = reinterpret_cast<Small*>(sm + OFF_SMALL);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int b = 0; b < NUM_BARS; ++b) tc::mbar_init(&sh->bar[b], 1);
    sh->abort = 0;
    tc::fence_mbar_init();
    tc::prefetch_tmap(&tmq);
    tc::prefetch_tmap(&tmk);
    tc::prefetch_tmap(&tmv);
  }
  if (warp == kMmaWarp) {
    tc::tmem_alloc(&sh->tmem_base, 512);
    tc::tmem_relinquish();
  }
  for (int i = threadIdx.x; i < 8192 / 16; i += kThreads)  // zero block of [T diag(beta) | 0 | P]
    reinterpret_cast<uint4*>(sm + OFF_TB + 8192)[i] = make_uint4(0, 0, 0, 0);
  tc::fence_async_smem();
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tb = sh->tmem_base;
  const Items it{(S + C - 1) / C, pairs, S};
  if (warp < kRecBase / 32) {
    prep_role<kBf16>(sm, sh, tb, it, g, beta, err_flag);
  } else if (warp < kTmaWarp) {
    rec_role<kBf16, kOut>(sm, sh, tb, it, init, out, final_state, err_flag);
  } else if (warp == kTmaWarp) {
    if (lane == 0) tma_role(sm, sh, &tmq, &tmk, &tmv, it, err_flag);
  } else if (lane == 0) {
    mma_role<kBf16>(sm, sh, tb, it, err_flag);
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) tc::tmem_dealloc(tb, 512);
}

}  // namespace
}  // namespace pipe

// Launches the pipelined kernel: persistent, grid = min(pairs, #SMs).
template <bool kBf16, int kOut>
Status launch_chunk_pipeline(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                             const float* g, const float* beta, const float* init, void* out,
                             float* final_state, int64_t pairs, int S, int* err, cudaStream_t st) {
  auto kern = pipe::chunk_pipe_kernel<kBf16, kOut>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, pipe::SMEM_BYTES);
  if (e != cudaSuccess) return cuda_status(e, "chunk_pipe_kernel smem attribute");
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const unsigned grid = (unsigned)(pairs < sms ? pairs : sms);
  kern<<<grid, pipe::kThreads, pipe::SMEM_BYTES, st>>>(mq, mk, mv, g, beta, init, out, final_state, S,
                                                       (int)pairs, err);
  SPOCK_LAUNCH_CHECK("chunk_pipe_kernel");
  return Status::ok();
}

#define SPOCK_PIPE_INST(BF, OUT)                                                                   \
  template Status launch_chunk_pipeline<BF, OUT>(const CUtensorMap&, const CUtensorMap&,          \
                                                 const CUtensorMap&, const float*, const float*,  \
                                                 const float*, void*, float*, int64_t, int, int*, \
                                                 cudaStream_t);
SPOCK_PIPE_INST(false, SPOCK_F32)
SPOCK_PIPE_INST(false, SPOCK_F16)
SPOCK_PIPE_INST(false, SPOCK_BF16)
SPOCK_PIPE_INST(true, SPOCK_F32)
SPOCK_PIPE_INST(true, SPOCK_F16)
SPOCK_PIPE_INST(true, SPOCK_BF16)
#undef SPOCK_PIPE_INST

}  // namespace spock

#ifdef SPOCK_PHASE_PROF
extern "C" __attribute__((visibility("default"))) int spock_debug_phase_profile(unsigned long long* out, int n) {
  if (n > 148 * 4 * 32) n = 148 * 4 * 32;
  return (int)cudaMemcpyFromSymbol(out, spock::pipe::g_phase_prof, n * sizeof(unsigned long long));
}
#endif
#if defined(SPOCK_PHASE_PROF) || defined(SPOCK_TRACE_ONLY)
extern "C" __attribute__((visibility("default"))) int spock_debug_trace(long long* out) {
  return (int)cudaMemcpyFromSymbol(out, spock::pipe::g_trace, 64 * 32 * sizeof(long long));
}
#endif
