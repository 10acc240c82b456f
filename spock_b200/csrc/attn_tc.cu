// Causal prefill attention of the gated full-attention layers on the tcgen05
// tensor cores (the layer-major prefill's counterpart of attention_decode.comp
// :64-143, applied to every prompt row at once; reference loop:
// src/runtime/vk_session.cpp:1166-1443).
//
// One CTA takes 32 prompt rows of one sequence and the 4 query heads of one
// kv head: 128 query vectors, query vector v = (head v / 32, row v % 32) on
// TMEM lane v. Two threads serve each vector (threads v and v + 128: columns
// 0-31 / 32-63 of a score tile, O columns 0-127 / 128-255). Per 64-position
// tile of the KV cache:
//   S  = Q K^T                  tcgen05 M128 N64  K256 -> TMEM [0,64) / [64,128)
//   online softmax (scale, causal mask, row max, exp; P rounded to fp16, the
//   denominators summed from the rounded values), P written K-major with the
//   128B swizzle to shared memory; O is rescaled in TMEM when a row's max moved
//   O += P V                    tcgen05 M128 N256 K64  -> TMEM [128, 384)
// S is double-buffered: tile i+1's Q K^T runs under tile i's softmax. Q is
// staged once; K and V tiles arrive by TMA (one box of 4 x 64 positions x 64 dims
// from the cache rows, no multicast) into two buffers each, a K buffer refilled
// as soon as its S MMA has read it and a V buffer once its P V has. The output
// is fp16(O / (l + 1e-30)), then fp16(out * sigmoid(gate)), as the decode
// kernel. Every mbarrier wait is bounded; a wait that gives up sets *err and
// the CTA lets its copies and MMAs land, releases TMEM and leaves.
#include <cuda.h>

#include <mutex>

#include "common.cuh"
#include "tc.cuh"

namespace spock {
namespace {

constexpr int HD = 256, QH = 8, KVH = 2, G = QH / KVH;
constexpr int kRows = 32, kPos = 64;
constexpr uint32_t kWait = 1u << 24;

// shared memory (1024-aligned offsets)
constexpr int OFF_Q = 0;                    // 4 x [128 rows x 128 B] (64-dim blocks), 64 KB
constexpr int OFF_K = 64 * 1024;            // 2 buffers x 4 x [64 pos x 128 B], 2 x 32 KB
constexpr int OFF_V = 128 * 1024;           // 2 buffers x 4 x [64 pos x 128 B], 2 x 32 KB
constexpr int OFF_P = 192 * 1024;           // [128 rows x 128 B] P, 16 KB
constexpr int OFF_RED = 208 * 1024;         // [2][128] fp32 row exchange, 1 KB
constexpr int OFF_BAR = 209 * 1024;
constexpr int SMEM = OFF_BAR + 256 + 1024;  // + alignment slack

__device__ __forceinline__ uint32_t sw128(int row, int ch) {
  return (uint32_t)row * 128u + ((uint32_t)(ch ^ (row & 7)) << 4);
}
// One K or V tile: 4 blocks of [64 positions][64 dims] (128B-swizzled), from
// the cache viewed as [batch][64-dim block][position][64] (no multicast).
__device__ __forceinline__ void tma_tile(void* dst, const CUtensorMap* m, uint64_t* bar, int p0, int blk, int seq) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(tc::smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(tc::smem_u32(bar)), "r"(0), "r"(p0), "r"(blk), "r"(seq)
      : "memory");
}

__global__ void __launch_bounds__(256, 1)
    attn_prefill_tc_kernel(const __grid_constant__ CUtensorMap tmkv, const __half* __restrict__ q,
                           const __half* __restrict__ gate, const int* __restrict__ pos, float scale,
                           __half* __restrict__ out, int T, int* __restrict__ err) {
  extern __shared__ uint8_t at_smem_raw[];
  uint8_t* sm = at_smem_raw + ((1024u - (tc::smem_u32(at_smem_raw) & 1023u)) & 1023u);
  // [0,1] K full, [2,3] V full, [4,5] S done, [6] O done, [7] drain (failure path)
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(sm + OFF_BAR + 64);
  int* s_fail = reinterpret_cast<int*>(sm + OFF_BAR + 72);
  float* red = reinterpret_cast<float*>(sm + OFF_RED);  // [2][128] row maxima, then partial sums
  const int tiles_per_seq = (T + kRows - 1) / kRows;
  const int seq = blockIdx.x / tiles_per_seq, t0 = (blockIdx.x % tiles_per_seq) * kRows, kvh = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, half = tid >> 7, v = tid & 127;
  const int r = v & 31;  // query vector v: head v / 32 of the group, prompt row t0 + r
  if (tid == 0) {
    for (int b = 0; b < 8; ++b) tc::mbar_init(&bar[b], 1);
    *s_fail = 0;
    tc::fence_mbar_init();
    tc::prefetch_tmap(&tmkv);
  }
  if (warp == 0) {
    tc::tmem_alloc(s_tmem, 512);
    tc::tmem_relinquish();
  }
  pdl_wait();
  pdl_launch();
  const int p_base = pos[seq];
  const int rows_here = min(kRows, T - t0);
  const int Lmax = p_base + t0 + rows_here;  // positions 0 .. Lmax-1 are read
  const int ntiles = (Lmax + kPos - 1) / kPos;
  const int my_last = p_base + t0 + r;      // the last position this query attends to
  // Q tile, loaded coalesced: 16-byte chunk c of query vector u = (head w,
  // row r) goes to 64-dim block c / 8 (zeros past the prompt's rows)
#pragma unroll 4
  for (int idx = tid; idx < 128 * 32; idx += 256) {
    const int rr = idx >> 7, ww = (idx >> 5) & 3, c = idx & 31, u = ww * 32 + rr;
    const uint4 x = rr < rows_here
                        ? *reinterpret_cast<const uint4*>(q + ((size_t)(seq * T + t0 + rr) * QH + kvh * G + ww) * HD + c * 8)
                        : make_uint4(0, 0, 0, 0);
    *reinterpret_cast<uint4*>(sm + OFF_Q + (c >> 3) * 16384 + sw128(u, c & 7)) = x;
  }
  tc::fence_async_smem();
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tb = *s_tmem, tO = tb + 128;
  const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
  const uint32_t sbase = tc::smem_u32(sm);
  constexpr uint32_t ID_S = tc::idesc_f16(128, 64, false, false);
  constexpr uint32_t ID_O = tc::idesc_f16(128, 256, false, true);
  // loads and waits per full barrier (thread 0's bookkeeping for the failure drain)
  int issued[4] = {0, 0, 0, 0}, waited[4] = {0, 0, 0, 0};
  auto load_k = [&](int i) {
    const int b = i & 1;
    ++issued[b];
    tc::mbar_arrive_expect_tx(&bar[b], 4 * kPos * 128);
    tma_tile(sm + OFF_K + b * 32768, &tmkv, &bar[b], i * kPos, kvh * 4, seq);
  };
  auto load_v = [&](int i) {
    const int b = i & 1;
    ++issued[2 + b];
    tc::mbar_arrive_expect_tx(&bar[2 + b], 4 * kPos * 128);
    tma_tile(sm + OFF_V + b * 32768, &tmkv, &bar[2 + b], i * kPos, (KVH + kvh) * 4, seq);
  };
  // S(i) = Q K(i)^T into S buffer i & 1 (thread 0); false if K(i) never arrived
  auto issue_s = [&](int i) -> bool {
    const int b = i & 1;
    if (!tc::mbar_wait_bounded(&bar[b], (i >> 1) & 1, kWait)) return false;
    ++waited[b];
    tc::tc_fence_after();
#pragma unroll
    for (int ks = 0; ks < 16; ++ks) {
      const uint32_t a = sbase + OFF_Q + (ks >> 2) * 16384 + (ks & 3) * 32;
      const uint32_t kb = sbase + OFF_K + b * 32768 + (ks >> 2) * 8192 + (ks & 3) * 32;
      tc::mma_f16(tb + b * 64, tc::sdesc(a, 16, 1024), tc::sdesc(kb, 16, 1024), ID_S, ks > 0);
    }
    tc::mma_commit(&bar[4 + b]);
    return true;
  };
  if (tid == 0) {
    load_k(0);
    load_v(0);
    if (ntiles > 1) {
      load_k(1);
      load_v(1);
    }
    if (!issue_s(0)) *s_fail = 1;
  }
  float m = -INFINITY, l = 0.f;
  bool ok = true;
  for (int i = 0; i < ntiles && ok; ++i) {
    const int b = i & 1, p0 = i * kPos;
    // S(i + 1) runs under this tile's softmax (its buffer was read by tile i - 1's)
    if (tid == 0 && i + 1 < ntiles && !*s_fail && !issue_s(i + 1)) *s_fail = 1;
    ok = !*s_fail && tc::mbar_wait_bounded(&bar[4 + b], (i >> 1) & 1, kWait);
    // P V of the previous tile has completed before P and O are touched again
    if (ok && i > 0) ok = tc::mbar_wait_bounded(&bar[6], (i - 1) & 1, kWait);
    if (__syncthreads_or(!ok || *s_fail)) {
      ok = false;
      break;
    }
    tc::tc_fence_after();
    if (tid == 0) {
      // K buffer b was read by S(i): refill it with tile i + 2; V buffer of
      // tile i - 1 was read by P V(i - 1): refill it with tile i + 1
      if (i + 2 < ntiles) load_k(i + 2);
      if (i >= 1 && i + 1 < ntiles) load_v(i + 1);
    }
    // online softmax: this thread's 32 columns of its row
    float s[32];
    tc::tmem_ld32(tb + b * 64 + lane_off + half * 32, s);
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float x = (p0 + half * 32 + j <= my_last) ? s[j] * scale : -INFINITY;
      s[j] = x;
      mx = fmaxf(mx, x);
    }
    red[half * 128 + v] = mx;
    __syncthreads();
    const float mn = fmaxf(m, fmaxf(mx, red[(half ^ 1) * 128 + v]));  // finite: position 0 is in tile 0
    const float corr = __expf(m - mn);
    m = mn;
    float lt = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint32_t h2[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const __half2 hp = __floats2half2_rn(__expf(s[c * 8 + 2 * e] - mn), __expf(s[c * 8 + 2 * e + 1] - mn));
        const float2 pf = __half22float2(hp);
        lt += pf.x + pf.y;  // the denominators sum the fp16 values P V multiplies
        h2[e] = *reinterpret_cast<const uint32_t*>(&hp);
      }
      *reinterpret_cast<uint4*>(sm + OFF_P + sw128(v, half * 4 + c)) = make_uint4(h2[0], h2[1], h2[2], h2[3]);
    }
    l = l * corr + lt;
    // rescale this thread's half of O where the row's max moved (warp-collective TMEM access)
    if (i > 0 && __any_sync(0xffffffffu, corr != 1.0f)) {
#pragma unroll 1
      for (int cb = half * 4; cb < half * 4 + 4; ++cb) {
        float o[32];
        tc::tmem_ld32(tO + lane_off + cb * 32, o);
#pragma unroll
        for (int k = 0; k < 32; ++k) o[k] *= corr;
        tc::tmem_st32(tO + lane_off + cb * 32, o);
      }
      tc::tmem_st_wait();
    }
    tc::fence_async_smem();
    tc::tc_fence_before();
    __syncthreads();
    // O += P V
    if (tid == 0) {
      ok = tc::mbar_wait_bounded(&bar[2 + b], (i >> 1) & 1, kWait);
      if (ok) {
        ++waited[2 + b];
        tc::tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_f16(tO, tc::sdesc(sbase + OFF_P + ks * 32, 16, 1024),
                      tc::sdesc(sbase + OFF_V + b * 32768 + ks * 2048, 8192, 1024), ID_O, (i > 0 || ks > 0) ? 1u : 0u);
        tc::mma_commit(&bar[6]);
      } else {
        *s_fail = 1;
      }
    }
  }
  if (ok) ok = !*s_fail && tc::mbar_wait_bounded(&bar[6], (ntiles - 1) & 1, kWait);
  if (__syncthreads_or(!ok)) {
    if (tid == 0) {
      atomicExch(err, 4);
      // let this CTA's issued MMAs and TMA copies land before TMEM and shared
      // memory are released (each wait bounded)
      tc::mma_commit(&bar[7]);
      tc::mbar_wait_bounded(&bar[7], 0, kWait);
      for (int b = 0; b < 4; ++b)
        if (issued[b] > waited[b]) tc::mbar_wait_bounded(&bar[b], (issued[b] - 1) & 1, kWait);
    }
  } else {
    tc::tc_fence_after();
    red[half * 128 + v] = l;
    __syncthreads();
    const float inv = 1.0f / (red[v] + red[128 + v] + 1e-30f);
    // The K buffers are idle now: gate rows come in coalesced (16-byte chunk c
    // of query vector u at u * 512 + ((c ^ (u & 31)) << 4), conflict-free for
    // both access patterns), each thread turns its own chunks into outputs in
    // place, and the outputs leave coalesced.
    uint8_t* stg = sm + OFF_K;
    auto chunk_addr = [&](int u, int c) { return stg + u * 512 + ((c ^ (u & 31)) << 4); };
    auto gaddr = [&](int idx, int& u, int& c) -> size_t {  // idx: 16-byte chunk of the CTA's rows
      const int rr = idx >> 7, ww = (idx >> 5) & 3;
      c = idx & 31;
      u = ww * 32 + rr;
      return ((size_t)(seq * T + t0 + rr) * QH + kvh * G + ww) * HD + c * 8;
    };
#pragma unroll 4
    for (int idx = tid; idx < 128 * 32; idx += 256) {
      int u, c;
      const size_t g = gaddr(idx, u, c);
      *reinterpret_cast<uint4*>(chunk_addr(u, c)) =
          (idx >> 7) < rows_here ? *reinterpret_cast<const uint4*>(gate + g) : make_uint4(0, 0, 0, 0);
    }
    __syncthreads();
    // every lane runs the (warp-collective) TMEM loads
#pragma unroll 1
    for (int cb = half * 4; cb < half * 4 + 4; ++cb) {
      float o[32];
      tc::tmem_ld32(tO + lane_off + cb * 32, o);
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        uint4* cp = reinterpret_cast<uint4*>(chunk_addr(v, cb * 4 + cc));
        const uint4 g4 = *cp;
        const __half2* gh = reinterpret_cast<const __half2*>(&g4);
        uint4 res;
        uint32_t* rr = reinterpret_cast<uint32_t*>(&res);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 gt = __half22float2(gh[e]);
          const int k = cc * 8 + 2 * e;
          const float a0 = __half2float(__float2half_rn(o[k] * inv)), a1 = __half2float(__float2half_rn(o[k + 1] * inv));
          const __half2 hv = __floats2half2_rn(a0 * __fdividef(1.0f, 1.0f + __expf(-gt.x)), a1 * __fdividef(1.0f, 1.0f + __expf(-gt.y)));
          rr[e] = *reinterpret_cast<const uint32_t*>(&hv);
        }
        *cp = res;
      }
    }
    __syncthreads();
#pragma unroll 4
    for (int idx = tid; idx < 128 * 32; idx += 256) {
      int u, c;
      const size_t g = gaddr(idx, u, c);
      if ((idx >> 7) < rows_here) *reinterpret_cast<uint4*>(out + g) = *reinterpret_cast<const uint4*>(chunk_addr(u, c));
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tb, 512);
}

typedef CUresult (*EncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                             const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                             CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeFn encode() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qr) == cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
  });
  return fn;
}

}  // namespace

// kv: the cache of this layer for every sequence, [batch][max_seq][K|V][2][256]
// fp16 with sequence stride kv_seq_stride elements (kv points at this layer).
Status launch_attn_prefill_tc(const void* q, const void* gate, const void* kv, int64_t kv_seq_stride, int max_seq,
                              const int* pos, float scale, void* out, int batch, int T, int* err, cudaStream_t st) {
  EncodeFn fn = encode();
  if (!fn) return Status::err(SPOCK_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if (((uintptr_t)kv & 15) || (kv_seq_stride * 2) % 16)
    return Status::err(SPOCK_ERR_INVALID, "attention prefill: KV cache must be 16-byte aligned");
  CUtensorMap map;
  cuuint64_t dims[4] = {64, (cuuint64_t)max_seq, (cuuint64_t)(2 * KVH * HD / 64), (cuuint64_t)batch};
  cuuint64_t strides[3] = {(cuuint64_t)(2 * KVH * HD * 2), 128, (cuuint64_t)kv_seq_stride * 2};
  cuuint32_t box[4] = {64, kPos, 4, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult rc = fn(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(kv), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (rc != CUDA_SUCCESS) return Status::err(SPOCK_ERR_CUDA, "attention prefill: tensor map encoding failed");
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [] {
    attr = cudaFuncSetAttribute(attn_prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
  });
  if (attr != cudaSuccess) return cuda_status(attr, "attn_prefill_tc_kernel attribute");
  const int tiles = (T + kRows - 1) / kRows;
  cudaError_t e = launch_k(attn_prefill_tc_kernel, dim3(tiles * batch, KVH), dim3(256), SMEM, st, map,
                           (const __half*)q, (const __half*)gate, pos, scale, (__half*)out, T, err);
  if (e != cudaSuccess) return cuda_status(e, "attn_prefill_tc_kernel");
  SPOCK_LAUNCH_CHECK("attn_prefill_tc_kernel");
  return Status::ok();
}

}  // namespace spock
