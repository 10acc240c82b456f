// Device helpers shared by the chunk-rule kernels (serial and pipelined).
#pragma once
#include "common.cuh"

namespace spock {
namespace chunk {

constexpr int C = 64;    // chunk size
constexpr int D = 128;   // key_dim == value_dim
constexpr int LDN = 65;  // padded fp32 row stride of the 64x64 N and T matrices

// Byte offset of 16-byte chunk `ch` (0..7) of row `row` in a SWIZZLE_128B
// region whose rows are 128 bytes (the layout TMA writes and UMMA reads).
__device__ __forceinline__ uint32_t sw128(int row, int ch) {
  return (uint32_t)row * 128u + ((uint32_t)(ch ^ (row & 7)) << 4);
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ uint4 pack8(const float* x) {
  return make_uint4(pack_h2(x[0], x[1]), pack_h2(x[2], x[3]), pack_h2(x[4], x[5]),
                    pack_h2(x[6], x[7]));
}

__device__ __forceinline__ void unpack8(uint4 u, float* x) {
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __half22float2(h[i]);
    x[2 * i] = f.x;
    x[2 * i + 1] = f.y;
  }
}

// T = (I - N)^-1 for strictly lower N (64x64, fp32, row stride LDN).
// 16x16 diagonal blocks by forward substitution, then off-diagonal blocks by
// block diagonals: T_ij = T_ii * sum_{k=j}^{i-1} N_ik T_kj. Executed by
// `nthreads` threads (thread index t), `sync()` synchronises exactly them.
template <class Sync>
__device__ __forceinline__ void solve_unit_lower(const float* __restrict__ N, float* __restrict__ T,
                                                 float* __restrict__ Y, int t, int nthreads, Sync sync) {
  if (t < 64) {
    const int o = (t >> 4) * 16, j = t & 15;
    float x[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      float acc = (i == j) ? 1.f : 0.f;
#pragma unroll
      for (int m = 0; m < i; ++m) acc = fmaf(N[(o + i) * LDN + o + m], x[m], acc);
      x[i] = (i < j) ? 0.f : acc;
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) T[(o + i) * LDN + o + j] = x[i];
  }
  sync();
  for (int d = 1; d < 4; ++d) {
    const int nb = 4 - d;
    for (int e = t; e < nb * 256; e += nthreads) {
      const int jb = e >> 8, r = (e >> 4) & 15, c = e & 15, ib = jb + d;
      float acc = 0.f;
      for (int col = 16 * jb; col < 16 * ib; ++col)
        acc = fmaf(N[(16 * ib + r) * LDN + col], T[col * LDN + 16 * jb + c], acc);
      Y[jb * 256 + r * 16 + c] = acc;
    }
    sync();
    for (int e = t; e < nb * 256; e += nthreads) {
      const int jb = e >> 8, r = (e >> 4) & 15, c = e & 15, ib = jb + d;
      float acc = 0.f;
      for (int m = 0; m <= r; ++m)
        acc = fmaf(T[(16 * ib + r) * LDN + 16 * ib + m], Y[jb * 256 + m * 16 + c], acc);
      T[(16 * ib + r) * LDN + 16 * jb + c] = acc;
    }
    sync();
  }
}

// Row stride of the fp32 N and T matrices of the pipelined kernel (16-byte
// aligned rows for float4 access; 68 = 4 mod 32 keeps the mma fragment loads
// of consecutive rows on distinct banks).
constexpr int LDT = 68;

// ---- 3xTF32 warp tiles (mma.sync m16n8k8) for the blocked inverse ----------
// Each fp32 operand x is split as hi = tf32(x), lo = tf32(x - hi); the three
// products lo*hi + hi*lo + hi*hi keep about 21 bits of every product, which is
// ample next to the fp16 operands the chunk products use afterwards.
__device__ __forceinline__ uint32_t tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ void split_tf32(float x, uint32_t& hi, uint32_t& lo) {
  hi = tf32_rna(x);
  lo = tf32_rna(x - __uint_as_float(hi));
}
__device__ __forceinline__ void mma_tf32(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// D(16x8, stride ldd) = A(16 x 8kSteps, stride lda) * B(8kSteps x 8, stride ldb), one warp.
// Fragments (g = lane/4, q = lane%4): A (g|g+8, q|q+4), B (q|q+4, g), C (g|g+8, 2q|2q+1).
template <int kSteps>
__device__ __forceinline__ void tile16x8_3xtf32(const float* __restrict__ A, int lda, const float* __restrict__ B,
                                                int ldb, float* __restrict__ Dst, int ldd) {
  const int lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  float c[4] = {0.f, 0.f, 0.f, 0.f}, e[4] = {0.f, 0.f, 0.f, 0.f};  // hi*hi | correction terms
#pragma unroll
  for (int s = 0; s < kSteps; ++s) {
    const float* a = A + s * 8;
    const float* b = B + s * 8 * ldb;
    uint32_t ah[4], al[4], bh0, bl0, bh1, bl1;
    split_tf32(a[g * lda + q], ah[0], al[0]);
    split_tf32(a[(g + 8) * lda + q], ah[1], al[1]);
    split_tf32(a[g * lda + q + 4], ah[2], al[2]);
    split_tf32(a[(g + 8) * lda + q + 4], ah[3], al[3]);
    split_tf32(b[q * ldb + g], bh0, bl0);
    split_tf32(b[(q + 4) * ldb + g], bh1, bl1);
    mma_tf32(e, al, bh0, bh1);
    mma_tf32(e, ah, bl0, bl1);
    mma_tf32(c, ah, bh0, bh1);
  }
  *reinterpret_cast<float2*>(Dst + g * ldd + 2 * q) = make_float2(c[0] + e[0], c[1] + e[1]);
  *reinterpret_cast<float2*>(Dst + (g + 8) * ldd + 2 * q) = make_float2(c[2] + e[2], c[3] + e[3]);
}

// T = (I - N)^-1 for 8 warps (256 threads) in five barrier-separated phases:
//   1. the four 16x16 diagonal blocks by forward substitution, one thread per
//      column (warps 0-1): once x_m is final it updates every later row, so
//      the dependent chain is 15 FMAs and the loads of N run ahead of it;
//   2/3. T10 = T11 (N10 T00) and T32 = T33 (N32 T22), which completes the two
//      32x32 diagonal inverses A^-1 = T[0:32,0:32] and B^-1 = T[32:64,32:64];
//   4/5. T[32:64,0:32] = B^-1 (N[32:64,0:32] A^-1).
// Phases 2-5 are 16x8 warp tiles on the tensor cores (3xTF32).
// N and T: row stride LDT (N's strictly lower part is read). The strictly
// upper blocks T[0:16,16:32] and T[32:48,48:64] must hold zeros (nothing here
// writes them). Y: 32 x kLDY floats of scratch.
constexpr int kLDY = 40;
template <class Sync>
__device__ __forceinline__ void solve_unit_lower_blk(const float* __restrict__ N, float* __restrict__ T,
                                                     float* __restrict__ Y, int t, Sync sync) {
  if (t < 64) {
    const int o = (t >> 4) * 16, j = t & 15;
    const float* nb = N + o * LDT + o;
    float x[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) x[i] = (i == j) ? 1.f : 0.f;
#pragma unroll
    for (int m = 0; m < 15; ++m) {
      float c[16];
#pragma unroll
      for (int i = m + 1; i < 16; ++i) c[i] = nb[i * LDT + m];
#pragma unroll
      for (int i = m + 1; i < 16; ++i) x[i] = fmaf(c[i], x[m], x[i]);
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) T[(o + i) * LDT + o + j] = x[i];
  }
  sync();
  const int w = t >> 5;
  if (w < 4) {  // Y_b = N_{ib,jb} T_jj  (b = w/2: (ib,jb) = (1,0) | (3,2); column half w&1)
    const int jb = 2 * (w >> 1), ib = jb + 1, n8 = (w & 1) * 8;
    tile16x8_3xtf32<2>(N + 16 * ib * LDT + 16 * jb, LDT, T + 16 * jb * LDT + 16 * jb + n8, LDT,
                       Y + (w >> 1) * 16 + n8, kLDY);
  }
  sync();
  if (w < 4) {  // T_{ib,jb} = T_ii Y_b
    const int jb = 2 * (w >> 1), ib = jb + 1, n8 = (w & 1) * 8;
    tile16x8_3xtf32<2>(T + 16 * ib * LDT + 16 * ib, LDT, Y + (w >> 1) * 16 + n8, kLDY,
                       T + 16 * ib * LDT + 16 * jb + n8, LDT);
  }
  sync();
  const int mi = w >> 2, n8 = (w & 3) * 8;
  // X = N[32:64,0:32] A^-1
  tile16x8_3xtf32<4>(N + (32 + 16 * mi) * LDT, LDT, T + n8, LDT, Y + 16 * mi * kLDY + n8, kLDY);
  sync();
  // T[32:64,0:32] = B^-1 X
  tile16x8_3xtf32<4>(T + (32 + 16 * mi) * LDT + 32, LDT, Y + n8, kLDY, T + (32 + 16 * mi) * LDT + n8, LDT);
  sync();
}

template <int kOut>
__device__ __forceinline__ void store_row32(void* out, size_t idx, const float (&v)[32]) {
  if constexpr (kOut == SPOCK_F32) {
    float4* o = reinterpret_cast<float4*>(static_cast<float*>(out) + idx);
#pragma unroll
    for (int q = 0; q < 8; ++q) o[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
  } else if constexpr (kOut == SPOCK_F16) {
    uint4* o = reinterpret_cast<uint4*>(static_cast<__half*>(out) + idx);
#pragma unroll
    for (int q = 0; q < 4; ++q) o[q] = pack8(&v[8 * q]);
  } else {
    uint4* o = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(out) + idx);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint32_t w[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        __nv_bfloat162 b = __floats2bfloat162_rn(v[8 * q + 2 * k], v[8 * q + 2 * k + 1]);
        w[k] = *reinterpret_cast<uint32_t*>(&b);
      }
      o[q] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

// kPrecise (fp32 inputs): V arrives as an fp16 hi/lo pair and the products
// [T diag(beta)] V and K^T [diag(e^{gL-gc}) v_new] are carried to ~22 bits by
// adding the lo x hi cross terms, so fp32 inputs are not limited to fp16's
// 11-bit significand where it matters for the state.

}  // namespace chunk
}  // namespace spock
