// Decode-glue operations exposed one by one (spock_rms_norm, spock_matvec,
// spock_argmax, spock_attention_decode): the reference's DecodeSession
// dispatches these shaders individually (src/runtime/vk_session.cpp:2658-3370),
// so a caller that keeps that orchestration can swap each dispatch for one call.
// They run the same kernels as the model session; `exact` selects the
// exact-order set (exact.cu) or the fast one (gemm.cu, model_kernels.cu).
#include <cmath>
#include <vector>

#include "common.cuh"
#include "gemm.h"
#include "ops.h"

namespace spock {

Status launch_rmsnorm(const void* x, const void* w, void* y, float eps, int batch, cudaStream_t st);
Status launch_attn_prep(const void* qkv, int ld, const void* qn_w, const void* kn_w, const float* rope,
                        const int* pos, void* q_out, void* gate_out, void* kv, int64_t kv_seq_stride,
                        int64_t kv_layer_off, float eps, int rows, cudaStream_t st, int rows_per_seq = 1);
Status launch_attn_decode(const void* q, const void* gate, const void* kv, int64_t kv_seq_stride,
                          int64_t kv_layer_off, const int* pos, float scale, void* out, int rows,
                          cudaStream_t st, int rows_per_seq = 1, float* ws = nullptr, int* tickets = nullptr);
int attn_decode_splits(int rows);
Status launch_exact_proj(int epi, const void* x, int ldx, const void* w, int K, int N, int batch, void* y, int ldy,
                         const void* res, float* amax_val, int* amax_idx, cudaStream_t st);
Status launch_attn_prefill_tc(const void* q, const void* gate, const void* kv, int64_t kv_seq_stride, int max_seq,
                              const int* pos, float scale, void* out, int batch, int T, int* err, cudaStream_t st);
Status launch_exact_attn(const void* q, const void* gate, const void* kv, int64_t kv_seq_stride, int64_t kv_layer_off,
                         const int* pos, int max_seq, float scale, void* out, int rows, int rows_per_seq,
                         cudaStream_t st);

namespace {

// argmax.comp:27-62 per row of fp16 logits: the strictly greater value wins,
// so among equal maxima the lowest index does. One CTA (256 threads) per row.
__global__ void __launch_bounds__(256) argmax_rows_kernel(const __half* __restrict__ logits, int64_t n,
                                                          int32_t* __restrict__ idx) {
  const __half* row = logits + (size_t)blockIdx.x * n;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {  // ascending: '>' keeps the first
    const float v = __half2float(row[i]);
    if (v > bv) {
      bv = v;
      bi = (int)i;
    }
  }
  __shared__ float sv[256];
  __shared__ int si[256];
  sv[threadIdx.x] = bv;
  si[threadIdx.x] = bi;
  __syncthreads();
  for (int s = 128; s > 0; s >>= 1) {
    if (threadIdx.x < s) {
      const float ov = sv[threadIdx.x + s];
      const int oi = si[threadIdx.x + s];
      if (ov > sv[threadIdx.x] || (ov == sv[threadIdx.x] && oi < si[threadIdx.x])) {
        sv[threadIdx.x] = ov;
        si[threadIdx.x] = oi;
      }
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) idx[blockIdx.x] = si[0] == 0x7fffffff ? 0 : si[0];
}

Status grow(ChunkScratch& s, size_t bytes, bool zero) {
  if (bytes <= s.bytes) return Status::ok();
  cudaError_t e = s.reserve(bytes);
  if (e != cudaSuccess) return Status::err(SPOCK_ERR_ALLOC, "op scratch: device allocation failed");
  if (zero && cudaMemset(s.buf, 0, s.bytes) != cudaSuccess)
    return Status::err(SPOCK_ERR_CUDA, "op scratch: clear failed");
  return Status::ok();
}

}  // namespace

Status op_rms_norm(const void* x, const void* w, void* y, int64_t rows, int dim, float eps, cudaStream_t st) {
  if (dim != 1024) return Status::err(SPOCK_ERR_UNSUPPORTED, "spock_rms_norm: the kernel implements dim 1024");
  if (rows > 0x7fffffff) return Status::err(SPOCK_ERR_INVALID, "spock_rms_norm: too many rows");
  if (((uintptr_t)x | (uintptr_t)w | (uintptr_t)y) & 7)
    return Status::err(SPOCK_ERR_INVALID, "spock_rms_norm: x, w and y must be 8-byte aligned");
  return launch_rmsnorm(x, w, y, eps, (int)rows, st);
}

Status op_argmax(const void* logits, int64_t rows, int64_t n, int32_t* idx, cudaStream_t st) {
  if (rows > 0x7fffffff) return Status::err(SPOCK_ERR_INVALID, "spock_argmax: too many rows");
  argmax_rows_kernel<<<(unsigned)rows, 256, 0, st>>>((const __half*)logits, n, idx);
  SPOCK_LAUNCH_CHECK("argmax_rows_kernel");
  return Status::ok();
}

Status op_matvec(OpsScratch& sc, int epilogue, int exact, const void* w, int out_dim, int in_dim, const void* x,
                 int64_t rows, void* y, const void* res, int sms, cudaStream_t st) {
  const int epi = epilogue == SPOCK_MV_STORE      ? EPI_F16
                  : epilogue == SPOCK_MV_RESIDUAL ? EPI_RESIDUAL
                  : epilogue == SPOCK_MV_SILU_GATE ? EPI_SWIGLU
                                                   : EPI_ARGMAX;
  const int n_rows = epi == EPI_SWIGLU ? 2 * out_dim : out_dim;  // weight rows
  const int ntiles = (n_rows + 127) / 128;
  if (rows > (exact ? (1 << 24) : (1 << 16)))
    return Status::err(SPOCK_ERR_UNSUPPORTED, exact ? "spock_matvec: at most 2^24 rows"
                                                    : "spock_matvec: the fast path takes at most 65536 rows per call");
  Status s;
  if (epi == EPI_ARGMAX) {
    s = grow(sc.amax, (size_t)ntiles * rows * 8, false);
    if (s.code) return s;
  }
  float* av = static_cast<float*>(sc.amax.buf);
  int* ai = av ? reinterpret_cast<int*>(av + (size_t)ntiles * rows) : nullptr;
  const int ldy = epi == EPI_SWIGLU ? out_dim : out_dim;
  if (exact) {
    s = launch_exact_proj(epi, x, in_dim, w, in_dim, n_rows, (int)rows, epi == EPI_ARGMAX ? nullptr : y, ldy, res,
                          av, ai, st);
  } else {
    // the tensor-core path reads x through a tensor map of bpad (a multiple of
    // 16) rows: stage it zero-padded in the context's scratch
    const int bpad = (int)((rows + 15) / 16 * 16);
    if ((s = grow(sc.xpad, (size_t)bpad * in_dim * 2, false)).code) return s;
    if (cudaMemsetAsync(sc.xpad.buf, 0, (size_t)bpad * in_dim * 2, st) != cudaSuccess ||
        cudaMemcpyAsync(sc.xpad.buf, x, (size_t)rows * in_dim * 2, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
      return Status::err(SPOCK_ERR_CUDA, "spock_matvec: staging copy failed");
    if ((s = grow(sc.ws, (size_t)sms * 128 * 256 * 4, false)).code) return s;
    GemmArgs a{};
    a.n_out = n_rows;
    a.k = in_dim;
    a.batch = (int)rows;
    a.bpad = bpad;
    a.y = (__half*)(epi == EPI_ARGMAX ? nullptr : y);
    a.ldy = ldy;
    a.res = (const __half*)res;
    a.ws = static_cast<float*>(sc.ws.buf);
    a.ws_bytes = sc.ws.bytes;
    a.amax_val = av;
    a.amax_idx = ai;
    a.err = sc.err;
    s = launch_gemm(epi, sc.xpad.buf, w, a, sms, st);
  }
  if (s.code) return s;
  if (epi == EPI_ARGMAX) return launch_argmax_finish(av, ai, ntiles, (int)rows, static_cast<int*>(y), st);
  return Status::ok();
}

Status op_attention_decode(OpsScratch& sc, int exact, const void* proj, const void* qn, const void* kn, float eps,
                           float theta, const int32_t* pos, void* kv, int max_seq, int64_t rows, void* out,
                           cudaStream_t st, int rows_per_seq) {
  if (rows > 0x7fffffff) return Status::err(SPOCK_ERR_INVALID, "spock_attention_decode: too many rows");
  // RoPE table [max_seq][32 x (cos, sin)], built on the host with the
  // reference's formula (vk_session.cpp:333-346) and kept per (theta, max_seq)
  if (sc.rope_theta != theta || sc.rope_seq < max_seq) {
    std::vector<float> t((size_t)max_seq * 64);
    for (int p = 0; p < max_seq; ++p)
      for (int i = 0; i < 32; ++i) {
        const float inv_freq = 1.0f / std::pow(theta, 2.0f * (float)i / 64.0f);
        const float ang = (float)p * inv_freq;
        t[(size_t)p * 64 + 2 * i] = std::cos(ang);
        t[(size_t)p * 64 + 2 * i + 1] = std::sin(ang);
      }
    Status s = grow(sc.rope, t.size() * 4, false);
    if (s.code) return s;
    // ordered with every stream (the previous table may still be read)
    if (cudaDeviceSynchronize() != cudaSuccess ||
        cudaMemcpy(sc.rope.buf, t.data(), t.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
      return Status::err(SPOCK_ERR_CUDA, "spock_attention_decode: RoPE table upload failed");
    sc.rope_theta = theta;
    sc.rope_seq = max_seq;
  }
  Status s = grow(sc.qg, (size_t)rows * 2 * 2048 * 2, false);
  if (s.code) return s;
  __half* q = static_cast<__half*>(sc.qg.buf);
  __half* gate = q + (size_t)rows * 2048;
  const int64_t stride = (int64_t)max_seq * 2 * 2 * 256;  // one layer per sequence
  const float* rope = static_cast<const float*>(sc.rope.buf);
  if ((s = launch_attn_prep(proj, 5120, qn, kn, rope, pos, q, gate, kv, stride, 0, eps, (int)rows, st,
                            rows_per_seq)).code)
    return s;
  if (exact)
    return launch_exact_attn(q, gate, kv, stride, 0, pos, max_seq, 1.0f / 16.0f, out, (int)rows, rows_per_seq, st);
  if (rows_per_seq > 1)  // prompt rows: the tcgen05 prefill kernel
    return launch_attn_prefill_tc(q, gate, kv, stride, max_seq, pos, 1.0f / 16.0f, out, (int)(rows / rows_per_seq),
                                  rows_per_seq, sc.err, st);
  const int ns = attn_decode_splits((int)rows);
  if (ns > 1) {
    if ((s = grow(sc.attn_ws, (size_t)rows * 2 * ns * 1032 * 4, false)).code) return s;
    if ((s = grow(sc.attn_tk, (size_t)rows * 2 * 4, true)).code) return s;
  }
  return launch_attn_decode(q, gate, kv, stride, 0, pos, 1.0f / 16.0f, out, (int)rows, st, 1,
                            ns > 1 ? static_cast<float*>(sc.attn_ws.buf) : nullptr,
                            ns > 1 ? static_cast<int*>(sc.attn_tk.buf) : nullptr);
}

}  // namespace spock
