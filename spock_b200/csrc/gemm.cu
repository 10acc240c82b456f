// Weight-streaming projection for the decode glue: y[b][n] = sum_k x[b][k] W[n][k]
// (fp16 in, fp32 accumulate), the batched form of spock's matvec / matvec_tiled /
// lm_head_tiled shaders (shaders/matvec.comp:28-41, matvec_tiled.comp:41-83,
// lm_head_tiled.comp:40-86). Their outputs are fp16-rounded; so are these.
//
// Swap-AB tcgen05 GEMM: a 128-row slab of W is the M=128 operand (K-major, TMA,
// 128B swizzle) and a block of up to 256 activation rows is the N operand, so
// one pass over the weights serves the whole batch; decode is HBM-bound on W.
// Prefill row counts run as many such blocks in one launch.
// Accumulators live in TMEM (lane = weight row, column = batch row).
//
// Grid: (row tiles, K splits, batch blocks). Large batches are split over
// batch blocks of bn >= 32 rows first (no partial sums: the CTAs of one row
// tile share its weight slab through L2), then over K while the grid is
// shorter than the SM count (one CTA streams its slab at a bounded rate, so a
// short grid leaves HBM idle). Up to 8 K splits of a tile run as one
// thread-block cluster: ranks 1.. park their fp32 partial tile in shared
// memory and rank 0 adds them in rank order through distributed shared memory
// (deterministic, no global traffic). More splits (small batches with long K)
// add vector atomics into an L2-resident accumulator; the last CTA of a tile
// (atomic ticket) reads the sum once, clears it for the next launch and runs
// the epilogue, with the split count capped so partial traffic stays below
// the weight traffic it parallelises.
//
// The epilogue stages the fp16 tile in shared memory (TMEM lanes are weight
// rows) and writes it back, with the residual, in 16-byte row segments.
//
// Epilogues (fused):
//   F16      y = fp16(acc)
//   RESIDUAL y = fp16(fp32(fp16(acc)) + res)          (matvec + residual_add.comp)
//   SWIGLU   W rows interleaved in 16-row groups [gate g..g+15 | up g..g+15]:
//            m = fp16(silu(fp16(gate)) * fp16(up))     (2 matvecs + silu_gate.comp)
//   ARGMAX   logits = fp16(acc); per batch row the tile's (max, lowest index)
//            goes to a partials array, reduced by argmax_finish (argmax.comp)
#include <cuda.h>

#include <mutex>

#include "common.cuh"
#include "gemm.h"
#include "tc.cuh"

namespace spock {

namespace {

constexpr int kMaxStages = 12;
constexpr int kMaxCluster = 8;  // portable thread-block cluster size
constexpr int kRingBytes = 4 * (128 * 128 + 256 * 128);  // 192 KB: the ring never exceeds it
constexpr uint32_t kWaitLimit = 1u << 25;

__device__ __forceinline__ bool wait_spin(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    if (tc::mbar_try_wait(bar, parity)) return true;
    if (i >= 8) __nanosleep(64);
  }
  return false;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          tc::smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(tc::smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// Thread-block cluster helpers (distributed shared memory, no TMA).
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t map_rank(uint32_t saddr, int rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

// kKB: 64-wide k blocks per ring stage. Each stage round (TMA, MMA, commit,
// hand-off) has a fixed cost, so long unsplit K loops at prefill row counts
// take two blocks per stage; short decode loops keep one (more CTAs per SM).
template <int kEpi, int kKB>
__global__ void __launch_bounds__(128, 1)
    gemm_swapab_kernel(const __grid_constant__ CUtensorMap tmw, const __grid_constant__ CUtensorMap tmx,
                       GemmArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024u - (tc::smem_u32(smem_raw) & 1023u)) & 1023u);
  const int a_bytes = 128 * 128, b_bytes = a.bn * 128, sub_bytes = a_bytes + b_bytes, stage_bytes = kKB * sub_bytes;
  const int kStages = a.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + kStages * stage_bytes);
  uint64_t* empty = full + kMaxStages;
  uint64_t* done = empty + kMaxStages;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(done + 1);
  int* s_last = reinterpret_cast<int*>(s_tmem + 1);

  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int tile = blockIdx.x, split = blockIdx.y, n0 = blockIdx.z * a.bn;
  const int kb0 = split * a.kb_per_split;
  const int nkb = min(a.kb_per_split, a.k / 64 - kb0);
  const int nst = (nkb + kKB - 1) / kKB;  // ring stages of this CTA
  auto subs = [&](int i) { return min(kKB, nkb - i * kKB); };
  uint32_t ncols = 32;
  while ((int)ncols < a.bn) ncols <<= 1;

  const int pre = nst < kStages ? nst : kStages;
  if (t == 0) {
    for (int s = 0; s < kStages; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    tc::mbar_init(done, 1);
    tc::fence_mbar_init();
    tc::prefetch_tmap(&tmw);
    tc::prefetch_tmap(&tmx);
    // The weights do not depend on the previous kernel or on TMEM: the first
    // stages' weight tiles stream while the TMEM allocation (which may wait
    // for the previous kernel's CTA on this SM) and its dependency drain.
    for (int i = 0; i < pre; ++i) {
      tc::mbar_arrive_expect_tx(&full[i], subs(i) * sub_bytes);
      for (int j = 0; j < subs(i); ++j)
        tma_load_2d(sm + i * stage_bytes + j * sub_bytes, &tmw, &full[i], (kb0 + i * kKB + j) * 64, tile * 128);
    }
  }
  __syncwarp();
  if (warp == 0) {
    tc::tmem_alloc(s_tmem, ncols);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tb = *s_tmem;
  bool ok = true;

  if (warp == 0 && lane == 0) {  // TMA producer (the first stages' weights are in flight)
    pdl_wait();
    pdl_launch();
    for (int i = 0; i < pre; ++i)
      for (int j = 0; j < subs(i); ++j)
        tma_load_2d(sm + i * stage_bytes + j * sub_bytes + a_bytes, &tmx, &full[i], (kb0 + i * kKB + j) * 64, n0);
    for (int i = pre; i < nst && ok; ++i) {
      const int s = i % kStages;
      ok = wait_spin(&empty[s], ((i / kStages) - 1) & 1);
      if (!ok) break;
      uint8_t* st = sm + s * stage_bytes;
      tc::mbar_arrive_expect_tx(&full[s], subs(i) * sub_bytes);
      for (int j = 0; j < subs(i); ++j) {
        tma_load_2d(st + j * sub_bytes, &tmw, &full[s], (kb0 + i * kKB + j) * 64, tile * 128);
        tma_load_2d(st + j * sub_bytes + a_bytes, &tmx, &full[s], (kb0 + i * kKB + j) * 64, n0);
      }
    }
  } else if (warp == 1 && lane == 0) {  // MMA issuer
    const uint32_t idesc = tc::idesc_f16(128, a.bn, false, false);
    const uint32_t sbase = tc::smem_u32(sm);
    for (int i = 0; i < nst && ok; ++i) {
      const int s = i % kStages;
      ok = wait_spin(&full[s], (i / kStages) & 1);
      if (!ok) break;
      tc::tc_fence_after();
      for (int j = 0; j < subs(i); ++j) {
        const uint32_t st = sbase + s * stage_bytes + j * sub_bytes;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc::mma_f16(tb, tc::sdesc(st + kk * 32, 16, 1024), tc::sdesc(st + a_bytes + kk * 32, 16, 1024), idesc,
                      (i > 0 || j > 0 || kk > 0) ? 1u : 0u);
      }
      tc::mma_commit(&empty[s]);
    }
    tc::mma_commit(done);
  }
  __syncwarp();
  pdl_wait();  // the epilogue reads and writes what earlier kernels use
  if constexpr (kEpi == EPI_RESIDUAL) {
    // pull this CTA's residual rows (2 x 128 B each) into L2 while the K loop runs
    for (int j = t; j < 2 * a.bn; j += 128) {
      const int b = n0 + (j >> 1), col = tile * 128 + (j & 1) * 64;
      if (b < a.batch && col < a.n_out)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(a.res + (size_t)b * a.ldy + col));
    }
  }
  // epilogue: all 128 threads; thread t <-> weight row tile*128 + t
  if (!wait_spin(done, 0)) ok = false;
  if (__syncthreads_or(!ok)) {
    if (t == 0) atomicExch(a.err, 3);
    if (a.csplit) {  // the cluster's two barriers stay matched; the leader's result is void
      cluster_sync();
      cluster_sync();
    } else if (a.nsplit > 1) {
      // Still take part in the tile's ticket, so it returns to zero; if this
      // CTA is the last one, it clears the accumulator slice the others added
      // to (the result is void either way, but the next launch starts clean).
      __threadfence();
      __syncthreads();
      if (t == 0) {
        int* ticket_p = a.tickets + tile * gridDim.z + blockIdx.z;
        const int ticket = atomicAdd(ticket_p, 1);
        *s_last = (ticket == a.nsplit - 1);
        if (*s_last) *ticket_p = 0;
      }
      __syncthreads();
      if (*s_last) {
        float* wsp = a.ws + (size_t)(tile * 128 + t) * a.bpad + n0;
        for (int c = 0; c < a.bn; ++c) __stcg(wsp + c, 0.f);
      }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 0) tc::tmem_dealloc(tb, ncols);
    return;
  }
  tc::tc_fence_after();
  const int row = tile * 128 + t;
  const uint32_t taddr = tb + ((uint32_t)(warp * 32) << 16);

  bool finisher = true;
  // cluster split: ranks 1.. leave their fp32 partial [bn][128] in their own
  // shared memory; rank 0 adds them to its accumulator in rank order
  const float* part = reinterpret_cast<const float*>(sm);
  if (a.csplit) {
    if (blockIdx.y != 0) {
      float* mine = reinterpret_cast<float*>(sm);
      for (int c0 = 0; c0 < a.bn; c0 += 32) {
        float v[32];
        tc::tmem_ld32(taddr + c0, v);
#pragma unroll
        for (int k = 0; k < 32; ++k)
          if (c0 + k < a.bn) mine[(c0 + k) * 128 + t] = v[k];
      }
    }
    cluster_sync();
    finisher = blockIdx.y == 0;
  } else if (a.nsplit > 1) {
    // partial tile -> accumulator [row][n0 + col] (vector atomics, resolved in L2)
    float* wsp = a.ws + (size_t)row * a.bpad + n0;
    for (int c0 = 0; c0 < a.bn; c0 += 32) {
      float v[32];
      tc::tmem_ld32(taddr + c0, v);
#pragma unroll
      for (int q = 0; q < 8; ++q)
        if (c0 + 4 * q < a.bn)
          atomicAdd(reinterpret_cast<float4*>(wsp + c0) + q, make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]));
    }
    __threadfence();
    __syncthreads();
    if (t == 0) {
      int* ticket_p = a.tickets + tile * gridDim.z + blockIdx.z;
      const int ticket = atomicAdd(ticket_p, 1);
      *s_last = (ticket == a.nsplit - 1);
      if (*s_last) *ticket_p = 0;  // ready for the next launch
    }
    __syncthreads();
    finisher = *s_last != 0;
    __threadfence();
  }

  if (finisher) {
    // the pipeline's stages are idle now: fp16 staging tile [bn][width]
    __half* stg = reinterpret_cast<__half*>(sm);
    constexpr int width = 128;  // staged weight rows (SWIGLU: gate and up, 64 outputs)
    for (int c0 = 0; c0 < a.bn; c0 += 32) {
      float v[32];
      if (a.nsplit > 1 && !a.csplit) {
        float4* p = reinterpret_cast<float4*>(a.ws + (size_t)row * a.bpad + n0 + c0);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          if (c0 + 4 * q < a.bn) {
            const float4 x = __ldcg(p + q);
            v[4 * q] = x.x;
            v[4 * q + 1] = x.y;
            v[4 * q + 2] = x.z;
            v[4 * q + 3] = x.w;
            __stcg(p + q, make_float4(0.f, 0.f, 0.f, 0.f));  // cleared for the next launch
          } else {
            v[4 * q] = v[4 * q + 1] = v[4 * q + 2] = v[4 * q + 3] = 0.f;
          }
        }
      } else {
        tc::tmem_ld32(taddr + c0, v);
        if (a.csplit) {
          for (int r = 1; r < a.nsplit; ++r) {
            const uint32_t base = map_rank(tc::smem_u32(part), r);
            float pv[32];
#pragma unroll
            for (int k = 0; k < 32; ++k) pv[k] = c0 + k < a.bn ? ld_cluster_f32(base + ((c0 + k) * 128 + t) * 4) : 0.f;
#pragma unroll
            for (int k = 0; k < 32; ++k) v[k] += pv[k];
          }
        }
      }
      if constexpr (kEpi == EPI_F16 || kEpi == EPI_RESIDUAL || kEpi == EPI_SWIGLU) {
        // SWIGLU stages fp16(gate) and fp16(up) rows; the store loop pairs them
#pragma unroll
        for (int k = 0; k < 32; ++k)
          if (c0 + k < a.bn) stg[(c0 + k) * width + t] = __float2half_rn(v[k]);
      } else {  // EPI_ARGMAX: fp16 logits staged; rows past n_out as -inf
#pragma unroll
        for (int k = 0; k < 32; ++k)
          if (c0 + k < a.bn) stg[(c0 + k) * width + t] = row < a.n_out ? __float2half_rn(v[k]) : __ushort_as_half(0xfc00);
      }
    }
    __syncthreads();
    if constexpr (kEpi == EPI_ARGMAX) {
      // per batch column: max over the tile's 128 rows in row order ('>' keeps the lowest index)
      for (int bl = t; bl < a.bn; bl += 128) {
        const int b = n0 + bl;
        if (b >= a.batch) continue;
        const uint4* col = reinterpret_cast<const uint4*>(stg + bl * width);
        float val = -INFINITY;
        int idx = 0x7fffffff;
        for (int c = 0; c < width / 8; ++c) {
          const uint4 u = col[c];
          const __half* hv = reinterpret_cast<const __half*>(&u);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float f = __half2float(hv[e]);
            if (f > val) {
              val = f;
              idx = tile * 128 + 8 * c + e;
            }
          }
        }
        a.amax_val[(size_t)tile * a.batch + b] = val;
        a.amax_idx[(size_t)tile * a.batch + b] = idx;
      }
    } else {
      // 16-byte segments: batch row bl, outputs out0 + 8c .. out0 + 8c + 7
      constexpr int outs = kEpi == EPI_SWIGLU ? 64 : 128;  // outputs of this tile
      const int out0 = tile * outs;
      const int n_valid = (kEpi == EPI_SWIGLU ? a.n_out / 2 : a.n_out) - out0;
      constexpr int segs = outs / 8;
      // kU segments per thread per round: the residual loads of a round are all
      // in flight before the first add (one dependent load per segment was the
      // epilogue's critical path)
      constexpr int kU = 4;
      const int total = a.bn * segs;
      for (int i0 = t; i0 < total; i0 += 128 * kU) {
        uint4 rv[kU];
        if constexpr (kEpi == EPI_RESIDUAL) {
#pragma unroll
          for (int u = 0; u < kU; ++u) {
            const int i = i0 + u * 128, bl = i / segs, c = i % segs, b = n0 + bl;
            if (i < total && b < a.batch && 8 * c < n_valid)
              rv[u] = *reinterpret_cast<const uint4*>(a.res + (size_t)b * a.ldy + out0 + 8 * c);
          }
        }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int i = i0 + u * 128, bl = i / segs, c = i % segs, b = n0 + bl;
        if (i >= total || b >= a.batch || 8 * c >= n_valid) continue;
        uint4 val;
        if constexpr (kEpi == EPI_SWIGLU) {
          // outputs 8c..8c+7 of the tile: weight rows [gate 16 | up 16] groups of 32
          const int f = 8 * c, base = (f >> 4) * 32 + (f & 15);
          const uint4 gq = *reinterpret_cast<const uint4*>(stg + bl * width + base);
          const uint4 uq = *reinterpret_cast<const uint4*>(stg + bl * width + base + 16);
          const __half* gh = reinterpret_cast<const __half*>(&gq);
          const __half* uh = reinterpret_cast<const __half*>(&uq);
          __half* o = reinterpret_cast<__half*>(&val);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float g16 = __half2float(gh[e]), u16 = __half2float(uh[e]);
            const float silu = __fdiv_rn(g16, __fadd_rn(1.0f, expf(-g16)));
            o[e] = __float2half_rn(__fmul_rn(silu, u16));
          }
        } else {
          val = *reinterpret_cast<const uint4*>(stg + bl * width + 8 * c);
        }
        const size_t off = (size_t)b * a.ldy + out0 + 8 * c;
        if constexpr (kEpi == EPI_RESIDUAL) {
          __half2* pv = reinterpret_cast<__half2*>(&val);
          const __half2* pr = reinterpret_cast<const __half2*>(&rv[u]);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 x = __half22float2(pv[e]), y = __half22float2(pr[e]);
            pv[e] = __floats2half2_rn(x.x + y.x, x.y + y.y);
          }
        }
        *reinterpret_cast<uint4*>(a.y + off) = val;
      }
      }
    }
  }
  if (a.csplit) cluster_sync();  // partials stay in place until the leader has read them
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tb, ncols);
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

Status map2d(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int box_rows) {
  EncodeTiledFn fn = encode_fn2();
  if (!fn) return Status::err(SPOCK_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return Status::err(SPOCK_ERR_CUDA, "cuTensorMapEncodeTiled failed (gemm)");
  return Status::ok();
}

}  // namespace

// x: [bpad][k] fp16 (rows >= batch may hold anything; a prefill's row count,
// bpad > 256, is one launch of 256-row or smaller blocks), W: [n_out][k] fp16.
// Workspace needs nsplit * ceil(n_out/128) * 128 * bpad floats when nsplit > 1,
// tickets ceil(n_out/128) ints (zero), ARGMAX partials ceil(n_out/128) * batch.
Status launch_gemm(int epi, const void* x, const void* w, GemmArgs a, int sms, cudaStream_t st) {
  if (a.k % 64 || a.bpad % 16 || a.bpad < 16 || a.batch > a.bpad || a.batch < 1)
    return Status::err(SPOCK_ERR_UNSUPPORTED, "gemm: k % 64, bpad a multiple of 16, batch <= bpad");
  if (a.bpad > 256 && a.nsplit > kMaxCluster)
    return Status::err(SPOCK_ERR_UNSUPPORTED, "gemm: bpad > 256 allows at most 8 K splits");
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
  // batch blocks first (no partial sums), down to 32 rows. Prefill row counts
  // (bpad > 256) start from 256-row blocks: one launch covers every row, and
  // the weight slab of a tile is re-read by its row blocks from L2.
  const bool fixed_bn = a.bn >= 16 && a.bn <= 256 && a.bn % 16 == 0;  // caller's choice (tuning)
  if (!fixed_bn) a.bn = a.bpad > 256 ? 256 : a.bpad;
  int nb = (a.bpad + a.bn - 1) / a.bn;
  while (!fixed_bn && ntiles * nb < sms && a.bn % 32 == 0 && a.bn / 2 >= 32) {
    a.bn /= 2;
    nb = (a.bpad + a.bn - 1) / a.bn;
  }
  if (nb > 65535) return Status::err(SPOCK_ERR_UNSUPPORTED, "gemm: too many row blocks");
  CUtensorMap mw, mx;
  Status s = map2d(&mw, w, a.n_out, a.k, 128);
  if (s.code) return s;
  s = map2d(&mx, x, a.bpad, a.k, a.bn);
  if (s.code) return s;
  if (a.nsplit < 1 && nb > 1) {
    // blocked batch: split K only to fill the SMs (a CTA streams one weight
    // slab at a bounded rate), in clusters that reduce on chip
    const int want = (sms + ntiles * nb - 1) / (ntiles * nb);
    a.nsplit = want < kMaxCluster ? want : kMaxCluster;
    if (a.nsplit > kbs / 2) a.nsplit = kbs / 2 > 1 ? kbs / 2 : 1;
  }
  if (a.nsplit < 1) {  // enough CTAs to stream the weights from every SM ...
    int want = (sms + ntiles * nb - 1) / (ntiles * nb);
    // ... but no more partial-tile traffic (128 x bn fp32) than weight traffic
    const int cap = a.k / (2 * a.bn);
    want = want > cap ? cap : want;
    want = want < 1 ? 1 : want;
    a.nsplit = want > kbs ? kbs : want;
  }
  a.kb_per_split = (kbs + a.nsplit - 1) / a.nsplit;
  a.nsplit = (kbs + a.kb_per_split - 1) / a.kb_per_split;
  // up to 8 splits reduce inside a cluster (deterministic, no workspace);
  // more go through the atomic workspace
  a.csplit = a.nsplit > 1 && a.nsplit <= kMaxCluster;
  if (a.nsplit > 1 && !a.csplit && (!a.ws || !a.tickets))
    return Status::err(SPOCK_ERR_INVALID, "gemm: split-K needs a workspace");
  // Four stages by default: deeper rings cost CTAs per SM, which these short K loops need more.
  // Unsplit prefill row counts take two k blocks per stage (kKB = 2).
  const int kb_stage = a.bpad > 256 && a.nsplit == 1 ? 2 : 1;
  const int stage_bytes = kb_stage * (128 * 128 + a.bn * 128);
  if (a.stages < 1) a.stages = 4;
  if (a.stages > kMaxStages) a.stages = kMaxStages;
  while (a.stages > 2 && a.stages * stage_bytes > kRingBytes) --a.stages;
  const int smem = a.stages * stage_bytes + 2 * kMaxStages * 8 + 64 + 8 * 256 * 4 + 1024;
  dim3 grid(ntiles, a.nsplit, nb);
  {
    static std::once_flag once;
    static Status prep;
    std::call_once(once, [] { prep = gemm_prepare(); });
    if (prep.code) return prep;
  }
#define SPOCK_GEMM_CASE(E)                                                                               \
  case E: {                                                                                              \
    if (a.csplit)                                                                                        \
      launch_k_cluster(gemm_swapab_kernel<E, 1>, grid, dim3(128), dim3(1, a.nsplit, 1), smem, st, mw, mx, a); \
    else if (kb_stage == 2)                                                                              \
      launch_k(gemm_swapab_kernel<E, 2>, grid, dim3(128), smem, st, mw, mx, a);                          \
    else                                                                                                 \
      launch_k(gemm_swapab_kernel<E, 1>, grid, dim3(128), smem, st, mw, mx, a);                          \
    break;                                                                                               \
  }
  switch (epi) {
    SPOCK_GEMM_CASE(EPI_F16)
    SPOCK_GEMM_CASE(EPI_RESIDUAL)
    SPOCK_GEMM_CASE(EPI_SWIGLU)
    SPOCK_GEMM_CASE(EPI_ARGMAX)
    default:
      return Status::err(SPOCK_ERR_INVALID, "gemm: unknown epilogue");
  }
#undef SPOCK_GEMM_CASE
  SPOCK_LAUNCH_CHECK("gemm_swapab_kernel");
  return Status::ok();
}

// Sets every GEMM variant's shared-memory limit once (before any graph capture).
Status gemm_prepare() {
  const int smem = kRingBytes + 2 * kMaxStages * 8 + 64 + 8 * 256 * 4 + 1024;
  cudaError_t e = cudaSuccess;
#define SPOCK_GEMM_ATTR(E)                                                                                      \
  if (e == cudaSuccess) e = cudaFuncSetAttribute(gemm_swapab_kernel<E, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); \
  if (e == cudaSuccess) e = cudaFuncSetAttribute(gemm_swapab_kernel<E, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
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
