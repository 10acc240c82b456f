// Weight-streaming projection for the decode glue: y[b][n] = sum_k x[b][k] W[n][k]
// (fp16 in, fp32 accumulate), the batched form of spock's matvec / matvec_tiled /
// lm_head_tiled shaders (shaders/matvec.comp:28-41, matvec_tiled.comp:41-83,
// lm_head_tiled.comp:40-86). Their outputs are fp16-rounded; so are these.
//
// More than 8 activation rows: a persistent tcgen05 GEMM (gemm_tc_kernel).
// A 128-row slab of W is the M=128 operand (K-major, TMA, 128B swizzle) and
// a block of up to 256 activation rows is the N operand, so one pass over the
// weights serves a whole block; decode is HBM-bound on W. Accumulators live
// in TMEM (lane = weight row, column = activation row), double-buffered so a
// unit's epilogue overlaps the next unit's MMAs. Short grids split K over a
// thread-block cluster whose ranks exchange fp32 partials through an
// L2-resident workspace and reduce them in rank order (deterministic).
// Up to 8 rows run on CUDA cores (gemv_kernel), streaming the weights once.
//
// Epilogues (fused):
//   F16      y = fp16(acc)
//   RESIDUAL y = fp16(fp32(fp16(acc)) + res)          (matvec + residual_add.comp)
//   SWIGLU   W rows interleaved in 16-row groups [gate g..g+15 | up g..g+15]:
//            m = fp16(silu(fp16(gate)) * fp16(up))     (2 matvecs + silu_gate.comp)
//   ARGMAX   logits = fp16(acc); per batch row the tile's (max, lowest index)
//            goes to a partials array, reduced by argmax_finish (argmax.comp)
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "gemm.h"
#include "tc.cuh"

namespace spock {

namespace {

constexpr uint32_t kWaitLimit = 1u << 25;

__device__ __forceinline__ bool wait_spin(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    if (tc::mbar_try_wait(bar, parity)) return true;
    if (i >= 8) __nanosleep(64);
  }
  return false;
}

// Barrier across the CTAs of a thread-block cluster (release / acquire).
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// ---- batched rows (> kGemvMaxB): persistent tcgen05 GEMM --------------------
// A unit is one 128-row weight tile x one block of bn activation rows (the MMA
// N), optionally one of `split` K ranges. Roles per CTA (384 threads):
//   warp 0      TMA producer: weight tile [128][64] and activation block
//               [bn][64] per ring stage (128B swizzle, no multicast)
//   warp 1      MMA issuer: 4 x K16 tcgen05.mma per stage into a TMEM
//               accumulator; two accumulators alternate between units, so
//               one unit's epilogue runs under the next unit's MMAs
//   warp 2      TMEM allocation
//   warps 4-11  epilogue: two warpgroups (columns interleaved in 32-wide
//               chunks), each warp reading its 32 TMEM lanes (weight rows)
// Without a K split the grid is min(units, SMs) and each CTA walks units
// blockIdx.x, blockIdx.x + gridDim.x, ... With a split each CTA owns exactly
// one (unit, K range); the ranks of a unit form one thread-block cluster
// (co-scheduled, so they can wait on each other), park their fp32 partial
// chunks in an L2-resident workspace, and after a cluster barrier each
// chunk's owner adds the ranks' partials in rank order (deterministic) and
// runs the epilogue for it.
constexpr int kTcEpiWarps = 8;
constexpr int kTcThreads = 128 + 32 * kTcEpiWarps;
constexpr int kTcMaxStages = 8;
constexpr int kTcKB = 2;             // 64-wide k blocks per ring stage
constexpr int kTcRing = 196608;      // 2 stages at bn = 256, more at narrower bn
constexpr int kStgHalves = 32 * 34;  // per-warp 32 x 32 transpose tile (ARGMAX rows padded to 34)
constexpr int kTcSmem = 1024 + kTcRing + kTcEpiWarps * kStgHalves * 2 + 2 * 4 * 32 * 8 + (2 * kTcMaxStages + 8) * 8;

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc::smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void named_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// One 32 x 32 chunk of a unit's accumulator: v[k] = acc[weight row
// tile*128 + wq*32 + lane][activation row col0 + k]. Transposed through the
// warp's staging tile so global stores are 16-byte row segments.
template <int kEpi>
__device__ __forceinline__ void tc_store_chunk(const GemmArgs& a, const float (&v)[32], __half* stg, int tile,
                                               int col0, int ncol, int wq, int lane, int half, bool ok,
                                               float* amx_v, int* amx_i) {
  if constexpr (kEpi == EPI_ARGMAX) {
    const int row = tile * 128 + wq * 32 + lane;
#pragma unroll
    for (int k = 0; k < 32; ++k)
      stg[k * 34 + lane] = row < a.n_out ? __float2half_rn(v[k]) : __ushort_as_half(0xfc00);
    __syncwarp();
    // lane = activation row: the warp's 32 weight rows in order ('>' keeps the lowest index)
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll 8
    for (int j = 0; j < 32; ++j) {
      const float f = __half2float(stg[lane * 34 + j]);
      if (f > bv) {
        bv = f;
        bi = tile * 128 + wq * 32 + j;
      }
    }
    amx_v[(half * 4 + wq) * 32 + lane] = bv;
    amx_i[(half * 4 + wq) * 32 + lane] = bi;
    named_sync(1 + half, 128);
    if (wq == 0) {  // the tile's four 32-row parts in row order
      for (int q = 1; q < 4; ++q) {
        const float ov = amx_v[(half * 4 + q) * 32 + lane];
        if (ov > bv) {
          bv = ov;
          bi = amx_i[(half * 4 + q) * 32 + lane];
        }
      }
      const int b = col0 + lane;
      if (ok && lane < ncol && b < a.batch) {
        a.amax_val[(size_t)tile * a.batch + b] = bv;
        a.amax_idx[(size_t)tile * a.batch + b] = bi;
      }
    }
    named_sync(1 + half, 128);
  } else {
#pragma unroll
    for (int k = 0; k < 32; ++k) stg[k * 32 + lane] = __float2half_rn(v[k]);
    __syncwarp();
    if constexpr (kEpi == EPI_SWIGLU) {
      // weight rows 32wq..32wq+31 of the tile are [gate 16 | up 16]: outputs
      // tile*64 + 16wq + 0..15; two 8-output segments per activation row
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int item = lane + 32 * j, k = item >> 1, s = item & 1, b = col0 + k;
        const int out = tile * 64 + wq * 16 + 8 * s;
        if (!(ok && k < ncol && b < a.batch && out < a.n_out / 2)) continue;
        const uint4 gq = *reinterpret_cast<const uint4*>(stg + k * 32 + 8 * s);
        const uint4 uq = *reinterpret_cast<const uint4*>(stg + k * 32 + 16 + 8 * s);
        const __half* gh = reinterpret_cast<const __half*>(&gq);
        const __half* uh = reinterpret_cast<const __half*>(&uq);
        uint4 val;
        __half* o = reinterpret_cast<__half*>(&val);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float g = __half2float(gh[e]), u = __half2float(uh[e]);
          o[e] = __float2half_rn(__fdividef(g, 1.0f + __expf(-g)) * u);
        }
        *reinterpret_cast<uint4*>(a.y + (size_t)b * a.ldy + out) = val;
      }
    } else {
      // four 8-output segments per activation row: 128 segments, 4 per lane
      uint4 rv[4];
      if constexpr (kEpi == EPI_RESIDUAL) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int item = lane + 32 * j, k = item >> 2, s = item & 3, b = col0 + k;
          const int out = tile * 128 + wq * 32 + 8 * s;
          if (ok && k < ncol && b < a.batch && out < a.n_out)
            rv[j] = *reinterpret_cast<const uint4*>(a.res + (size_t)b * a.ldy + out);
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int item = lane + 32 * j, k = item >> 2, s = item & 3, b = col0 + k;
        const int out = tile * 128 + wq * 32 + 8 * s;
        if (!(ok && k < ncol && b < a.batch && out < a.n_out)) continue;
        uint4 val = *reinterpret_cast<const uint4*>(stg + k * 32 + 8 * s);
        if constexpr (kEpi == EPI_RESIDUAL) {
          __half2* pv = reinterpret_cast<__half2*>(&val);
          const __half2* pr = reinterpret_cast<const __half2*>(&rv[j]);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 x = __half22float2(pv[e]), y = __half22float2(pr[e]);
            pv[e] = __floats2half2_rn(x.x + y.x, x.y + y.y);
          }
        }
        *reinterpret_cast<uint4*>(a.y + (size_t)b * a.ldy + out) = val;
      }
    }
    __syncwarp();  // the staging tile is rewritten by the next chunk
  }
}

template <int kEpi>
__global__ void __launch_bounds__(kTcThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmw, const __grid_constant__ CUtensorMap tmx, GemmArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024u - (tc::smem_u32(smem_raw) & 1023u)) & 1023u);
  const int bn = a.bn, S = a.nsplit, nst = a.stages;
  // A ring stage holds kTcKB k blocks: [W 128 x 64] x kTcKB then
  // [x bn x 64] x kTcKB, one TMA box each. One barrier wait and one commit
  // per stage (each costs the issuing thread about as much as a k block's
  // MMAs at N <= 128, and each TMA issue about 200 cycles).
  const int xoff = kTcKB * 16384, stage_bytes = kTcKB * (16384 + bn * 128);
  __half* stg_all = reinterpret_cast<__half*>(sm + kTcRing);
  float* amx_v = reinterpret_cast<float*>(sm + kTcRing + kTcEpiWarps * kStgHalves * 2);
  int* amx_i = reinterpret_cast<int*>(amx_v + 2 * 4 * 32);
  uint64_t* full = reinterpret_cast<uint64_t*>(amx_i + 2 * 4 * 32);
  uint64_t* empty = full + kTcMaxStages;
  uint64_t* accf = empty + kTcMaxStages;  // [2] MMA -> epilogue
  uint64_t* acce = accf + 2;              // [2] epilogue -> MMA
  uint64_t* drain = acce + 2;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(drain + 1);

  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int nb = (a.bpad + bn - 1) / bn;
  const int units = ((a.n_out + 127) / 128) * nb;
  const int rank = S > 1 ? (int)(blockIdx.x % S) : 0;
  const int u0 = S > 1 ? (int)(blockIdx.x / S) : (int)blockIdx.x;
  const int ustep = S > 1 ? units : (int)gridDim.x;  // split: one unit per CTA
  const int kb0 = rank * a.kb_per_split;
  const int nkb = min(a.kb_per_split, a.k / 64 - kb0);
  const int nsg = (nkb + kTcKB - 1) / kTcKB;  // ring stages per unit
  auto subs = [&](int js) { return min(kTcKB, nkb - js * kTcKB); };
  uint32_t bnp = 32;
  while ((int)bnp < bn) bnp <<= 1;
  const int nch = (bn + 31) / 32;
  int pre = 0;

  if (warp == 0) {  // one barrier per lane
    if (lane < nst) {
      tc::mbar_init(&full[lane], 1);
      tc::mbar_init(&empty[lane], 1);
    } else if (lane >= 16 && lane < 18) {
      tc::mbar_init(&accf[lane - 16], 1);
      tc::mbar_init(&acce[lane - 16], kTcEpiWarps);
    } else if (lane == 18) {
      tc::mbar_init(drain, 1);
    }
    __syncwarp();
  }
  if (t == 0) {
    tc::fence_mbar_init();
    tc::prefetch_tmap(&tmw);
    tc::prefetch_tmap(&tmx);
    // The weights do not depend on the previous kernel: the first stages'
    // weight tiles stream while the TMEM allocation and that kernel drain.
    if (u0 < units) {
      pre = nsg < nst ? nsg : nst;
      for (int i = 0; i < pre; ++i) {  // boxes past K (or past a split's range) fill and count in full
        tc::mbar_arrive_expect_tx(&full[i], stage_bytes);
        tc::tma_load_3d(sm + i * stage_bytes, &tmw, &full[i], 0, (u0 / nb) * 128, kb0 + i * kTcKB);
      }
    }
  }
  __syncwarp();
  if (warp == 2) {
    tc::tmem_alloc(s_tmem, 2 * bnp);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tb = *s_tmem;
  bool ok = true;
  int issued = 0;

  if (warp == 0) {
    if (lane == 0) {  // TMA producer
      pdl_wait();
      pdl_launch();
      for (int u = u0; u < units && ok; u += ustep) {
        const int tile = u / nb, rb = u % nb;
        for (int js = 0; js < nsg; ++js, ++issued) {
          const int s = issued % nst, kb = kb0 + js * kTcKB;
          uint8_t* st = sm + s * stage_bytes;
          if (issued < pre) {  // weight tiles already in flight
            tc::tma_load_3d(st + xoff, &tmx, &full[s], 0, rb * bn, kb);
            continue;
          }
          if (issued >= nst && !(ok = wait_spin(&empty[s], ((issued / nst) - 1) & 1))) break;
          tc::mbar_arrive_expect_tx(&full[s], stage_bytes);
          tc::tma_load_3d(st, &tmw, &full[s], 0, tile * 128, kb);
          tc::tma_load_3d(st + xoff, &tmx, &full[s], 0, rb * bn, kb);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      const uint32_t idesc = tc::idesc_f16(128, bn, false, false);
      const uint32_t sbase = tc::smem_u32(sm);
      int it = 0, i = 0;
      for (int u = u0; u < units && ok; u += ustep, ++i) {
        const int b = i & 1;
        if (i >= 2 && !(ok = wait_spin(&acce[b], ((i >> 1) - 1) & 1))) break;
        tc::tc_fence_after();
        const uint32_t d = tb + b * bnp;
        for (int js = 0; js < nsg; ++js, ++it) {
          const int s = it % nst, n = subs(js);
          if (!(ok = wait_spin(&full[s], (it / nst) & 1))) break;
          tc::tc_fence_after();
          for (int q = 0; q < n; ++q) {
            const uint32_t wa = sbase + s * stage_bytes + q * 16384, xa = sbase + s * stage_bytes + xoff + q * bn * 128;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              tc::mma_f16(d, tc::sdesc(wa + kk * 32, 16, 1024), tc::sdesc(xa + kk * 32, 16, 1024), idesc,
                          (js | q | kk) ? 1u : 0u);
          }
          tc::mma_commit(&empty[s]);
        }
        if (ok) tc::mma_commit(&accf[b]);
      }
      tc::mma_commit(drain);  // every MMA of this thread has finished before TMEM is freed
      if (!wait_spin(drain, 0)) ok = false;
    }
    __syncwarp();
  } else if (warp >= 4) {
    // Epilogue. After a timeout a warp keeps the same control flow (the
    // ARGMAX combine synchronises the four warps of a warpgroup) but stops
    // waiting and writes nothing.
    const int ew = warp - 4, wq = warp & 3, half = ew >> 2;
    __half* stg = stg_all + ew * kStgHalves;
    pdl_wait();  // reads and writes what earlier kernels use
    int i = 0;
    for (int u = u0; u < units; u += ustep, ++i) {
      const int tile = u / nb, rb = u % nb, b = i & 1;
      if (ok) ok = wait_spin(&accf[b], (i >> 1) & 1);
      tc::tc_fence_after();
      const uint32_t tq = tb + b * bnp + ((uint32_t)(wq * 32) << 16);
      for (int c = half; c < nch; c += 2) {
        if (S > 1 && c % S == rank) continue;  // this rank's own chunks wait for the others
        float v[32];
        tc::tmem_ld32(tq + c * 32, v);
        if (S == 1) {
          tc_store_chunk<kEpi>(a, v, stg, tile, rb * bn + c * 32, min(32, bn - c * 32), wq, lane, half, ok, amx_v,
                               amx_i);
        } else if (ok) {  // partial chunk -> workspace [unit][rank][chunk][32 cols][128 rows]
          float* p = a.ws + (((size_t)u * S + rank) * nch + c) * 4096 + wq * 32 + lane;
#pragma unroll
          for (int k = 0; k < 32; ++k) __stcg(p + k * 128, v[k]);
        }
      }
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce[b]);
    }
  }
  // every role has left its loop (all waits are bounded)
  const bool any_fail = __syncthreads_or(!ok);
  if (S > 1) {
    __threadfence();
    cluster_sync();  // every rank's partials are in the workspace
    tc::tc_fence_after();
    if (warp >= 4 && u0 < units) {
      const int ew = warp - 4, wq = warp & 3, half = ew >> 2;
      const int tile = u0 / nb, rb = u0 % nb;
      const uint32_t tq = tb + ((uint32_t)(wq * 32) << 16);
      for (int c = half; c < nch; c += 2) {
        if (c % S != rank) continue;
        float acc[32];
        for (int q = 0; q < S; ++q) {
          float p[32];
          if (q == rank) {
            tc::tmem_ld32(tq + c * 32, p);
          } else {
            const float* src = a.ws + (((size_t)u0 * S + q) * nch + c) * 4096 + wq * 32 + lane;
#pragma unroll
            for (int k = 0; k < 32; ++k) p[k] = __ldcg(src + k * 128);
          }
#pragma unroll
          for (int k = 0; k < 32; ++k) acc[k] = q == 0 ? p[k] : acc[k] + p[k];
        }
        tc_store_chunk<kEpi>(a, acc, stg_all + ew * kStgHalves, tile, rb * bn + c * 32, min(32, bn - c * 32), wq,
                             lane, half, ok, amx_v, amx_i);
      }
    }
  }
  if (warp == 0 && any_fail) {
    // loads still in flight (a timeout elsewhere) land before the CTA exits;
    // without a failure the MMA issuer has consumed every stage
    if (lane == 0)
      for (int q = issued > nst ? issued - nst : 0; q < issued; ++q)
        if (!wait_spin(&full[q % nst], (q / nst) & 1)) ok = false;
    __syncwarp();
  }
  if (!ok) atomicExch(a.err, 3);
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 2) tc::tmem_dealloc(tb, 2 * bnp);
}

// ---- small batches (<= kGemvMaxB rows): CUDA-core weight streaming ---------
// One warp per output unit (a weight row, or a gate/up row pair for SWIGLU):
// lanes stream the row in 16-byte segments against the batch rows staged in
// shared memory, fp32 accumulation, then a butterfly reduction. No partial
// sums and no tensor-memory setup, which matters when the batch is tiny and
// each projection is a few microseconds of HBM time.
constexpr int kGemvMaxB = 8;
constexpr int kGemvWarps = 8;
constexpr int kGemvChunks = 4;  // 16-byte weight segments per lane and unit: k <= 1024 * wu

__device__ __forceinline__ void fma8(float& acc, uint4 w, uint4 x) {
  const __half2* wh = reinterpret_cast<const __half2*>(&w);
  const __half2* xh = reinterpret_cast<const __half2*>(&x);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 wf = __half22float2(wh[e]), xf = __half22float2(xh[e]);
    acc = fmaf(wf.x, xf.x, acc);
    acc = fmaf(wf.y, xf.y, acc);
  }
}

template <int kEpi, int kB>
__global__ void __launch_bounds__(kGemvWarps * 32) gemv_kernel(const uint4* __restrict__ W, const uint4* __restrict__ x,
                                                               GemmArgs a, int units_per_cta, int wu) {
  extern __shared__ uint4 xs[];  // [batch][k / 8]
  __shared__ float r_val[kGemvWarps][kB];
  __shared__ int r_idx[kGemvWarps][kB];
  __shared__ float red[kGemvWarps * 32];
  __shared__ float nfac;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int k8 = a.k / 8, B = a.batch;  // B <= kB
  const int units = kEpi == EPI_SWIGLU ? a.n_out / 2 : a.n_out;
  float bval[kB];
  int bidx[kB];
#pragma unroll
  for (int b = 0; b < kB; ++b) {
    bval[b] = -INFINITY;
    bidx[b] = 0x7fffffff;
  }
  // wu warps per unit split its k range; groups of wu warps take units in turn.
  // Lane chunks c = lane + 32*sub + 32*wu*i (i < kGemvChunks) cover the row.
  const int groups = kGemvWarps / wu, grp = warp / wu, sub = warp % wu;
  const int u0 = blockIdx.x * units_per_cta, u1 = min(units, u0 + units_per_cta);
  const int rounds = (units_per_cta + groups - 1) / groups;  // same for every warp: barriers below
  auto unit_of = [&](int r) { return u0 + r * groups + grp; };
  auto load_w = [&](int r, uint4 (&w)[kGemvChunks], uint4 (&w2)[kGemvChunks]) {
    const int u = unit_of(r);
    const int row = kEpi == EPI_SWIGLU ? (u >> 4) * 32 + (u & 15) : u;
    const uint4* wr = W + (size_t)row * k8;
#pragma unroll
    for (int i = 0; i < kGemvChunks; ++i) {
      const int c = lane + 32 * (sub + wu * i);
      const bool in = u < u1 && c < k8;
      w[i] = in ? __ldcs(wr + c) : make_uint4(0, 0, 0, 0);
      if constexpr (kEpi == EPI_SWIGLU) w2[i] = in ? __ldcs(wr + 16 * k8 + c) : make_uint4(0, 0, 0, 0);
    }
  };
  uint4 wc[kGemvChunks], wc2[kGemvChunks];
  load_w(0, wc, wc2);  // (issued before the activations are staged)
  pdl_wait();
  pdl_launch();
  if (a.norm_w) {
    // the rms_norm shader's arithmetic: 4 consecutive elements per thread,
    // then the stride-128..1 tree (the last five levels as warp shuffles)
    __half* xh = reinterpret_cast<__half*>(xs);
    const __half* src = reinterpret_cast<const __half*>(x);
    for (int b = 0; b < B; ++b) {
      float v[4], acc = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        v[i] = __half2float(src[(size_t)b * a.k + t * 4 + i]);
        acc = __fadd_rn(acc, __fmul_rn(v[i], v[i]));
      }
      red[t] = acc;
      __syncthreads();
      for (int stride = 128; stride >= 32; stride >>= 1) {
        if (t < stride) red[t] = __fadd_rn(red[t], red[t + stride]);
        __syncthreads();
      }
      if (t < 32) {
        float sm = red[t];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sm = __fadd_rn(sm, __shfl_down_sync(0xffffffffu, sm, o));
        if (t == 0) nfac = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sm, (float)a.k), a.eps)));
      }
      __syncthreads();
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float wv = __fadd_rn(1.0f, __half2float(a.norm_w[t * 4 + i]));
        const __half y = __float2half_rn(__fmul_rn(__fmul_rn(v[i], nfac), wv));
        xh[b * a.k + t * 4 + i] = y;
        if (a.xnorm_out && blockIdx.x == 0) a.xnorm_out[(size_t)b * a.k + t * 4 + i] = y;
      }
    }
  } else {
    for (int i = t; i < B * k8; i += blockDim.x) xs[i] = x[i];
  }
  __syncthreads();
  for (int r = 0; r < rounds; ++r) {
    const int u = unit_of(r);
    const bool live = u < u1;
    uint4 wn[kGemvChunks], wn2[kGemvChunks];
    if (r + 1 < rounds) load_w(r + 1, wn, wn2);  // next round's weights fly during this one
    float acc[kB], acc2[kB];
#pragma unroll
    for (int b = 0; b < kB; ++b) acc[b] = acc2[b] = 0.f;
#pragma unroll
    for (int i = 0; i < kGemvChunks; ++i) {
      const int c = lane + 32 * (sub + wu * i);
      if (c < k8) {
#pragma unroll
        for (int b = 0; b < kB; ++b) {
          if (b < B) {
            const uint4 xv = xs[b * k8 + c];
            fma8(acc[b], wc[i], xv);
            if constexpr (kEpi == EPI_SWIGLU) fma8(acc2[b], wc2[i], xv);
          }
        }
      }
    }
#pragma unroll
    for (int i = 0; i < kGemvChunks; ++i) {
      wc[i] = wn[i];
      if constexpr (kEpi == EPI_SWIGLU) wc2[i] = wn2[i];
    }
#pragma unroll
    for (int b = 0; b < kB; ++b) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        acc[b] += __shfl_xor_sync(0xffffffffu, acc[b], o);
        if constexpr (kEpi == EPI_SWIGLU) acc2[b] += __shfl_xor_sync(0xffffffffu, acc2[b], o);
      }
    }
    if (wu > 1) {  // sum the group's warps in order (the first warp of each group finishes)
      if (lane == 0)
#pragma unroll
        for (int b = 0; b < kB; ++b) {
          r_val[warp][b] = acc[b];
          if constexpr (kEpi == EPI_SWIGLU) red[warp * kB + b] = acc2[b];
        }
      __syncthreads();
      if (sub == 0 && lane == 0)
#pragma unroll
        for (int b = 0; b < kB; ++b) {
          for (int w = 1; w < wu; ++w) {
            acc[b] += r_val[warp + w][b];
            if constexpr (kEpi == EPI_SWIGLU) acc2[b] += red[(warp + w) * kB + b];
          }
        }
      __syncthreads();
    }
    if (live && sub == 0 && lane == 0) {
#pragma unroll
      for (int b = 0; b < kB; ++b) {
        if (b >= B) continue;
        const size_t off = (size_t)b * a.ldy + u;
        if constexpr (kEpi == EPI_F16) {
          a.y[off] = __float2half_rn(acc[b]);
        } else if constexpr (kEpi == EPI_RESIDUAL) {
          a.y[off] = __float2half_rn(__half2float(__float2half_rn(acc[b])) + __half2float(a.res[off]));
        } else if constexpr (kEpi == EPI_SWIGLU) {
          const float g16 = __half2float(__float2half_rn(acc[b]));
          const float u16 = __half2float(__float2half_rn(acc2[b]));
          const float silu = __fdiv_rn(g16, __fadd_rn(1.0f, expf(-g16)));
          a.y[off] = __float2half_rn(__fmul_rn(silu, u16));
        } else {  // ARGMAX: units visited in increasing order, so '>' keeps the lowest index
          const float v = __half2float(__float2half_rn(acc[b]));
          if (v > bval[b]) {
            bval[b] = v;
            bidx[b] = u;
          }
        }
      }
    }
  }
  if constexpr (kEpi == EPI_ARGMAX) {
    if (lane == 0)
#pragma unroll
      for (int b = 0; b < kB; ++b) {
        r_val[warp][b] = bval[b];
        r_idx[warp][b] = bidx[b];
      }
    __syncthreads();
    if (t < B) {
      float v = r_val[0][t];
      int i = r_idx[0][t];
      for (int w = 1; w < kGemvWarps; ++w)
        if (r_val[w][t] > v || (r_val[w][t] == v && r_idx[w][t] < i)) {
          v = r_val[w][t];
          i = r_idx[w][t];
        }
      a.amax_val[(size_t)blockIdx.x * B + t] = v;
      a.amax_idx[(size_t)blockIdx.x * B + t] = i;
    }
  }
}

// token[b] = index of the largest fp16 logit, lowest index among equals.
__global__ void argmax_finish_kernel(const float* __restrict__ val, const int* __restrict__ idx, int ntiles,
                                     int batch, int* __restrict__ token) {
  const int b = blockIdx.x;
  pdl_wait();
  pdl_launch();
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < ntiles; i += blockDim.x) {
    const float v = val[(size_t)i * batch + b];
    const int x = idx[(size_t)i * batch + b];
    if (v > bv || (v == bv && x < bi)) {
      bv = v;
      bi = x;
    }
  }
  __shared__ float sv[256];
  __shared__ int si[256];
  sv[threadIdx.x] = bv;
  si[threadIdx.x] = bi;
  __syncthreads();
  for (int s = blockDim.x / 2; s > 0; s >>= 1) {
    if ((int)threadIdx.x < s) {
      const float ov = sv[threadIdx.x + s];
      const int oi = si[threadIdx.x + s];
      if (ov > sv[threadIdx.x] || (ov == sv[threadIdx.x] && oi < si[threadIdx.x])) {
        sv[threadIdx.x] = ov;
        si[threadIdx.x] = oi;
      }
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) token[b] = si[0];
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_fn2() {
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

// [rows][cols] fp16 viewed as [cols / 64][rows][64]: one box brings kTcKB
// consecutive 64-wide k blocks of box_rows rows, each block a 128B-swizzled
// [box_rows][64] tile (one TMA instruction per operand per ring stage).
Status map_kb(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int box_rows) {
  EncodeTiledFn fn = encode_fn2();
  if (!fn) return Status::err(SPOCK_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {64, (cuuint64_t)rows, (cuuint64_t)(cols / 64)};
  cuuint64_t strides[2] = {(cuuint64_t)cols * 2, 128};
  cuuint32_t box[3] = {64, (cuuint32_t)box_rows, (cuuint32_t)kTcKB};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return Status::err(SPOCK_ERR_CUDA, "cuTensorMapEncodeTiled failed (gemm)");
  return Status::ok();
}

// Clusters of `split` CTAs of gemm_tc_kernel<epi> that fit on the device at
// once (cluster shapes do not tile every GPC exactly), queried once per shape.
int max_clusters(int epi, int split) {
  static std::mutex mu;
  static int cache[4][9];
  static bool init = false;
  std::lock_guard<std::mutex> g(mu);
  if (!init) {
    for (auto& r : cache)
      for (int& c : r) c = -1;
    init = true;
  }
  int& c = cache[epi & 3][split];
  if (c >= 0) return c;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(split);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = kTcSmem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = split;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  cudaError_t e = cudaErrorInvalidValue;
  switch (epi) {
    case EPI_F16: e = cudaOccupancyMaxActiveClusters(&n, gemm_tc_kernel<EPI_F16>, &cfg); break;
    case EPI_RESIDUAL: e = cudaOccupancyMaxActiveClusters(&n, gemm_tc_kernel<EPI_RESIDUAL>, &cfg); break;
    case EPI_SWIGLU: e = cudaOccupancyMaxActiveClusters(&n, gemm_tc_kernel<EPI_SWIGLU>, &cfg); break;
    default: e = cudaOccupancyMaxActiveClusters(&n, gemm_tc_kernel<EPI_ARGMAX>, &cfg); break;
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    n = 0;  // no split rather than a guess
  }
  return c = n;
}

}  // namespace

// x: [bpad][k] fp16 (rows >= batch may hold anything; any row count is one
// launch of 256-row or smaller blocks), W: [n_out][k] fp16. A K split uses
// the workspace (a.ws, a.ws_bytes) only when it fits: units * split * 128 *
// round_up(bn, 32) floats. ARGMAX partials: ceil(n_out/128) * batch.
Status launch_gemm(int epi, const void* x, const void* w, GemmArgs a, int sms, cudaStream_t st) {
  if (a.k % 64 || a.bpad % 16 || a.bpad < 16 || a.batch > a.bpad || a.batch < 1)
    return Status::err(SPOCK_ERR_UNSUPPORTED, "gemm: k % 64, bpad a multiple of 16, batch <= bpad");
  if (a.nsplit > 8 || (a.bn && (a.bn % 16 || a.bn > 256)))
    return Status::err(SPOCK_ERR_UNSUPPORTED, "gemm: at most 8 K splits, bn a multiple of 16 up to 256");
  if (((uintptr_t)x & 15) || ((uintptr_t)w & 15))
    return Status::err(SPOCK_ERR_INVALID, "gemm: operands must be 16-byte aligned");
  if (epi != EPI_ARGMAX) {
    const int outs = epi == EPI_SWIGLU ? a.n_out / 2 : a.n_out;
    if (outs % 8 || a.ldy % 8 || ((uintptr_t)a.y & 15) || ((uintptr_t)a.res & 15) ||
        (epi == EPI_SWIGLU && a.n_out % 32))
      return Status::err(SPOCK_ERR_UNSUPPORTED, "gemm: outputs and ldy must be multiples of 8, y/res 16-byte aligned");
  }
  const int ntiles = (a.n_out + 127) / 128, kbs = a.k / 64;
  if (a.batch <= kGemvMaxB && (size_t)a.batch * a.k * 2 <= 96 * 1024) {
    // ARGMAX keeps one partial per 128-row tile (what argmax_finish reads);
    // the others spread their units over a few CTAs per SM
    const int units = epi == EPI_SWIGLU ? a.n_out / 2 : a.n_out;
    if (a.k > 1024 * kGemvWarps || (epi == EPI_ARGMAX && a.k > 1024))
      return Status::err(SPOCK_ERR_UNSUPPORTED, "gemm: small-batch path needs k <= 8192 (ARGMAX: 1024)");
    if (a.norm_w && a.k != kGemvWarps * 32 * 4)
      return Status::err(SPOCK_ERR_UNSUPPORTED, "gemm: fused RMSNorm needs k == 1024");
    int per = 128, wu = 1;
    if (epi != EPI_ARGMAX) {
      // enough warps in flight to stream the weights: split short unit lists' k
      while (wu < kGemvWarps && units * wu < 16 * sms) wu *= 2;
      while (wu < kGemvWarps && a.k > 1024 * wu) wu *= 2;  // kGemvChunks segments per lane
      const int groups = kGemvWarps / wu;
      per = (units + 4 * sms - 1) / (4 * sms);
      per = ((per + groups - 1) / groups) * groups;
    }
    const int grid = (units + per - 1) / per;
    const size_t smem = (size_t)a.batch * a.k * 2;
    const uint4* w4 = (const uint4*)w;
    const uint4* x4 = (const uint4*)x;
    cudaError_t e = cudaSuccess;
    {
      static std::once_flag once;
      static Status prep;
      std::call_once(once, [] { prep = gemm_prepare(); });
      if (prep.code) return prep;
    }
    auto go = [&](auto kern) { e = launch_k(kern, dim3(grid), dim3(kGemvWarps * 32), smem, st, w4, x4, a, per, wu); };
#define SPOCK_GEMV_B(E)                                     \
  if (a.batch == 1) go(gemv_kernel<E, 1>);                  \
  else if (a.batch == 2) go(gemv_kernel<E, 2>);             \
  else if (a.batch <= 4) go(gemv_kernel<E, 4>);             \
  else go(gemv_kernel<E, 8>);
    switch (epi) {
      case EPI_F16: SPOCK_GEMV_B(EPI_F16) break;
      case EPI_RESIDUAL: SPOCK_GEMV_B(EPI_RESIDUAL) break;
      case EPI_SWIGLU: SPOCK_GEMV_B(EPI_SWIGLU) break;
      case EPI_ARGMAX: SPOCK_GEMV_B(EPI_ARGMAX) break;
      default: return Status::err(SPOCK_ERR_INVALID, "gemm: unknown epilogue");
    }
#undef SPOCK_GEMV_B
    if (e != cudaSuccess) return cuda_status(e, "gemv_kernel launch");
    SPOCK_LAUNCH_CHECK("gemv_kernel");
    return Status::ok();
  }
  if (a.norm_w) return Status::err(SPOCK_ERR_UNSUPPORTED, "gemm: fused RMSNorm only on the small-batch path");
  {
    static std::once_flag once;
    static Status prep;
    std::call_once(once, [] { prep = gemm_prepare(); });
    if (prep.code) return prep;
  }
  // Plan (bn, split) from per-launch costs measured on B200 (microseconds,
  // 2-k-block stages; the ~3 us of fixed cost per launch is common to all):
  // a 64-wide K block costs a CTA 0.24 us at bn <= 64, 0.33 at bn = 128 and
  // 0.48 at bn = 256; units beyond one per SM queue on a CTA (their
  // epilogues overlap); a split adds ~2.5 us of partial exchange and
  // reduction and needs all its clusters resident at once.
  const size_t ws_floats = a.ws ? a.ws_bytes / 4 : 0;
  int best_bn = 0, best_split = 1;
  double best = 1e30;
  for (int bn : {256, 128, 64, 32, 16, a.bpad}) {
    if (bn > 256 || bn % 16 || bn > a.bpad) continue;
    if (a.bn > 0 && bn != a.bn) continue;
    const int nb = (a.bpad + bn - 1) / bn, units = ntiles * nb, nch = (bn + 31) / 32;
    const double ckb = bn > 128 ? 0.48 : bn > 64 ? 0.33 : 0.24;
    for (int split : {1, 2, 4, 8}) {
      if (a.nsplit > 0 && split != a.nsplit) continue;
      double cost;
      if (split == 1) {
        cost = (double)((units + sms - 1) / sms) * kbs * ckb;
      } else {
        const int per = (kbs + split - 1) / split;
        if ((kbs + per - 1) / per != split || units > max_clusters(epi, split)) continue;
        if ((size_t)units * split * nch * 4096 > ws_floats) continue;
        cost = per * ckb + 2.5 + 0.1 * split;
      }
      if (cost < best - 1e-9) {
        best = cost;
        best_bn = bn;
        best_split = split;
      }
    }
  }
  if (!best_bn) return Status::err(SPOCK_ERR_INVALID, "gemm: no tile plan (workspace too small for the forced split)");
  a.bn = best_bn;
  a.nsplit = best_split;
  a.kb_per_split = (kbs + a.nsplit - 1) / a.nsplit;
  const int nb = (a.bpad + a.bn - 1) / a.bn, units = ntiles * nb;
  a.stages = std::min(kTcMaxStages, kTcRing / (kTcKB * (16384 + a.bn * 128)));
  CUtensorMap mw, mx;
  Status s = map_kb(&mw, w, a.n_out, a.k, 128);
  if (s.code) return s;
  s = map_kb(&mx, x, a.bpad, a.k, a.bn);
  if (s.code) return s;
  const dim3 grid(a.nsplit > 1 ? units * a.nsplit : std::min(units, sms));
  cudaError_t e = cudaSuccess;
#define SPOCK_GEMM_CASE(E)                                                                                     \
  case E:                                                                                                      \
    e = a.nsplit > 1 ? launch_k_cluster(gemm_tc_kernel<E>, grid, dim3(kTcThreads), dim3(a.nsplit, 1, 1),       \
                                        kTcSmem, st, mw, mx, a)                                                \
                     : launch_k(gemm_tc_kernel<E>, grid, dim3(kTcThreads), kTcSmem, st, mw, mx, a);            \
    break;
  switch (epi) {
    SPOCK_GEMM_CASE(EPI_F16)
    SPOCK_GEMM_CASE(EPI_RESIDUAL)
    SPOCK_GEMM_CASE(EPI_SWIGLU)
    SPOCK_GEMM_CASE(EPI_ARGMAX)
    default:
      return Status::err(SPOCK_ERR_INVALID, "gemm: unknown epilogue");
  }
#undef SPOCK_GEMM_CASE
  if (e != cudaSuccess) return cuda_status(e, "gemm_tc_kernel launch");
  SPOCK_LAUNCH_CHECK("gemm_tc_kernel");
  return Status::ok();
}

// Sets every GEMM variant's shared-memory limit once (before any graph capture).
Status gemm_prepare() {
  cudaError_t e = cudaSuccess;
#define SPOCK_GEMM_ATTR(E) \
  if (e == cudaSuccess) e = cudaFuncSetAttribute(gemm_tc_kernel<E>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem);
  SPOCK_GEMM_ATTR(EPI_F16)
  SPOCK_GEMM_ATTR(EPI_RESIDUAL)
  SPOCK_GEMM_ATTR(EPI_SWIGLU)
  SPOCK_GEMM_ATTR(EPI_ARGMAX)
#undef SPOCK_GEMM_ATTR
  const int gsm = 96 * 1024;  // staged activations of the small-batch path
#define SPOCK_GEMV_ATTR(E)                                                                                        \
  if (e == cudaSuccess) e = cudaFuncSetAttribute(gemv_kernel<E, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, gsm); \
  if (e == cudaSuccess) e = cudaFuncSetAttribute(gemv_kernel<E, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, gsm); \
  if (e == cudaSuccess) e = cudaFuncSetAttribute(gemv_kernel<E, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, gsm); \
  if (e == cudaSuccess) e = cudaFuncSetAttribute(gemv_kernel<E, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize, gsm);
  SPOCK_GEMV_ATTR(EPI_F16)
  SPOCK_GEMV_ATTR(EPI_RESIDUAL)
  SPOCK_GEMV_ATTR(EPI_SWIGLU)
  SPOCK_GEMV_ATTR(EPI_ARGMAX)
#undef SPOCK_GEMV_ATTR
  return cuda_status(e, "gemm_prepare");
}

Status launch_argmax_finish(const float* val, const int* idx, int ntiles, int batch, int* token, cudaStream_t st) {
  launch_k(argmax_finish_kernel, dim3(batch), dim3(256), 0, st, val, idx, ntiles, batch, token);
  SPOCK_LAUNCH_CHECK("argmax_finish_kernel");
  return Status::ok();
}

}  // namespace spock
