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
  int bn;            // batch rows per CTA (MMA N): 0 = launch_gemm chooses
  int kb_per_split;  // 64-wide k blocks per split; set by launch_gemm
  int nsplit;        // K splits; 0 = let launch_gemm choose
  int stages;        // TMA ring depth: 0 = launch_gemm chooses (4), capped by its 192 KB ring
  int csplit;        // set by launch_gemm: the K splits of a tile form one thread-block
                     // cluster and reduce their partials through distributed shared memory
  __half* y;         // [batch][ldy]; ldy % 8 == 0, 16-byte aligned
  int ldy;
  const __half* res;  // RESIDUAL: [batch][ldy]
  float* ws;          // split accumulator [n_tiles*128][bpad], zero between launches
  int* tickets;       // [n_tiles], zero before launch, left zero after
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
