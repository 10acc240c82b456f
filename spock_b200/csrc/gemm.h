// Weight-streaming projection GEMM of the decode glue (gemm.cu): interface
// shared by the kernels and the model session.
#pragma once
#include <cuda_fp16.h>

#include "common.cuh"

namespace spock {

enum GemmEpi { EPI_F16 = 0, EPI_RESIDUAL = 1, EPI_SWIGLU = 2, EPI_ARGMAX = 3 };

struct GemmArgs {
  int n_out;         // weight rows
  int k;             // inner dim, multiple of 64
  int batch;         // real batch rows
  int bpad;          // padded batch rows of x, multiple of 16
  int bn;            // activation rows per unit (MMA N, multiple of 16): 0 = launch_gemm chooses
  int kb_per_split;  // 64-wide k blocks per split; set by launch_gemm
  int nsplit;        // K splits (1, 2, 4, 8); 0 = launch_gemm chooses
  int stages;        // TMA ring depth; set by launch_gemm
  __half* y;         // [batch][ldy]; ldy % 8 == 0, 16-byte aligned
  int ldy;
  const __half* res;  // RESIDUAL: [batch][ldy]
  float* ws;          // K-split partials (L2-resident scratch, no state between launches)
  size_t ws_bytes;
  float* amax_val;    // ARGMAX partials [n_tiles][batch]
  int* amax_idx;
  int* err;
  // Small-batch path only: x is the residual stream h and the kernel applies
  // RMSNorm (x * rsqrt(mean(x^2) + eps) * (1 + norm_w), k == 1024) itself;
  // xnorm_out (nullable) receives the normed rows.
  const __half* norm_w;
  float eps;
  __half* xnorm_out;
};

Status launch_gemm(int epi, const void* x, const void* w, GemmArgs a, int sms, cudaStream_t st);
Status launch_argmax_finish(const float* val, const int* idx, int ntiles, int batch, int* token, cudaStream_t st);
Status gemm_prepare();

}  // namespace spock
