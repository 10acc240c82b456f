// extern "C" boundary of libspock_b200.so (declared in include/spock_b200.h).
// Argument validation and error text live here; the kernels' launchers return
// spock::Status. Nothing here throws across the ABI.
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>
#include <string>

#include "chunk_scratch.h"
#include "common.cuh"
#include "ops.h"

namespace spock {
std::atomic<uint64_t> g_launches{0};
bool& pdl_enabled() {
  static thread_local bool on = false;
  return on;
}

Status launch_decode_step(const spock_dn_layer& L, int64_t batch, void* qkv, void* conv_state,
                          float* state, const void* a, const void* b, const void* z, void* out,
                          void* core_raw, int* err, cudaStream_t stream);
Status launch_recurrent(int64_t batch, int H, int kd, int vd, const void* q, const void* k,
                        const void* v, const float* g, const float* beta, float* state, void* out, int* err,
                        cudaStream_t stream);
Status launch_chunk_prefill(ChunkScratch& scratch, const spock_chunk_desc& d, const void* q,
                            const void* k, const void* v, const float* g, const float* beta,
                            const float* init, void* out, float* final_state, int* err_flag,
                            cudaStream_t stream);
Status launch_last_to_fp16(int64_t batch, int64_t H, int64_t S, int64_t V, const float* core,
                           void* out, cudaStream_t stream);
Status launch_wait_timeout_selftest(uint32_t polls, int* err, cudaStream_t stream);
Status noalloc_err_word(int** out);
}  // namespace spock

struct spock_ctx {
  int device = 0;
  std::string err;
  int* d_err_flag = nullptr;  // device word written by kernels whose bounded waits gave up
  int sms = 148;
  spock::ChunkScratch chunk;
  spock::OpsScratch ops;
};

namespace {
std::mutex g_err_mu;
std::string g_err;  // context-less errors
}  // namespace

namespace spock {
// The context's device error word (bounded waits that gave up), shared with
// model sessions created on the context so spock_sync reports their timeouts.
int* ctx_err_word(spock_ctx* ctx) { return ctx ? ctx->d_err_flag : nullptr; }

// Records the text returned by spock_last_error(NULL) (context-less calls).
void record_global_error(const std::string& msg) {
  std::lock_guard<std::mutex> lk(g_err_mu);
  g_err = msg;
}
}  // namespace spock

namespace {

int fail(spock_ctx* ctx, int code, const std::string& msg) {
  if (ctx) {
    ctx->err = msg;
  } else {
    std::lock_guard<std::mutex> lk(g_err_mu);
    g_err = msg;
  }
  return code;
}

int finish(spock_ctx* ctx, const spock::Status& s) {
  if (s.code != SPOCK_OK) return fail(ctx, s.code, s.msg);
  return SPOCK_OK;
}

// Makes ctx's device current for the duration of a call.
struct DeviceGuard {
  int prev = -1;
  bool ok = true;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
  }
  ~DeviceGuard() {
    int cur;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

bool sm100(int dev) {
  cudaDeviceProp p;
  if (cudaGetDeviceProperties(&p, dev) != cudaSuccess) return false;
  return p.major == 10;
}
}  // namespace

extern "C" {

__attribute__((visibility("default"))) int spock_create(int device, spock_ctx** out) {
  if (!out) return fail(nullptr, SPOCK_ERR_INVALID, "spock_create: out is NULL");
  *out = nullptr;
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess)
    return fail(nullptr, SPOCK_ERR_CUDA, std::string("spock_create: ") + cudaGetErrorString(e));
  if (device < 0 || device >= n)
    return fail(nullptr, SPOCK_ERR_INVALID, "spock_create: device ordinal out of range");
  if (!sm100(device))
    return fail(nullptr, SPOCK_ERR_UNSUPPORTED, "spock_create: device is not sm_100 (B200)");
  spock_ctx* c = new (std::nothrow) spock_ctx();
  if (!c) return fail(nullptr, SPOCK_ERR_ALLOC, "spock_create: out of host memory");
  c->device = device;
  DeviceGuard g(device);
  if (!g.ok || cudaMalloc(&c->d_err_flag, sizeof(int)) != cudaSuccess ||
      cudaMemset(c->d_err_flag, 0, sizeof(int)) != cudaSuccess) {
    delete c;
    return fail(nullptr, SPOCK_ERR_ALLOC, "spock_create: device allocation failed");
  }
  c->ops.err = c->d_err_flag;
  cudaDeviceGetAttribute(&c->sms, cudaDevAttrMultiProcessorCount, device);
  *out = c;
  return SPOCK_OK;
}

__attribute__((visibility("default"))) int spock_destroy(spock_ctx* ctx) {
  if (!ctx) return SPOCK_OK;
  {
    DeviceGuard g(ctx->device);
    cudaFree(ctx->d_err_flag);
    ctx->chunk.release();
    ctx->ops.release();
  }
  delete ctx;
  return SPOCK_OK;
}

__attribute__((visibility("default"))) const char* spock_last_error(const spock_ctx* ctx) {
  if (ctx) return ctx->err.c_str();
  std::lock_guard<std::mutex> lk(g_err_mu);
  return g_err.c_str();
}

__attribute__((visibility("default"))) uint64_t spock_kernel_launch_count(void) {
  return spock::g_launches.load();
}

__attribute__((visibility("default"))) int spock_selftest_wait_timeout(spock_ctx* ctx, uint32_t polls, void* stream) {
  if (polls == 0 || polls > (1u << 20))
    return fail(ctx, SPOCK_ERR_INVALID, "spock_selftest_wait_timeout: polls must be in [1, 2^20]");
  if (!ctx) {  // the allocation-free entry point's error word, on the current device
    int* word = nullptr;
    spock::Status s = spock::noalloc_err_word(&word);
    if (!s.code) s = spock::launch_wait_timeout_selftest(polls, word, (cudaStream_t)stream);
    return finish(nullptr, s);
  }
  DeviceGuard g(ctx->device);
  return finish(ctx, spock::launch_wait_timeout_selftest(polls, ctx->d_err_flag, (cudaStream_t)stream));
}

__attribute__((visibility("default"))) int spock_sync(spock_ctx* ctx, void* stream) {
  if (!ctx) return fail(nullptr, SPOCK_ERR_INVALID, "spock_sync: ctx is NULL");
  DeviceGuard g(ctx->device);
  cudaError_t e = cudaStreamSynchronize((cudaStream_t)stream);
  if (e != cudaSuccess) return fail(ctx, SPOCK_ERR_CUDA, std::string("spock_sync: ") + cudaGetErrorString(e));
  int flag = 0;
  e = cudaMemcpy(&flag, ctx->d_err_flag, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return fail(ctx, SPOCK_ERR_CUDA, std::string("spock_sync: ") + cudaGetErrorString(e));
  if (flag) {
    cudaMemset(ctx->d_err_flag, 0, sizeof(int));
    return fail(ctx, SPOCK_ERR_TIMEOUT, "spock_sync: a kernel's bounded wait gave up (code " +
                                            std::to_string(flag) + ")");
  }
  return SPOCK_OK;
}

__attribute__((visibility("default"))) int spock_chunk_prefill(
    spock_ctx* ctx, const spock_chunk_desc* d, const void* q, const void* k, const void* v,
    const float* g, const float* beta, const float* init_state, void* core_out,
    float* final_state, void* stream) {
  if (!ctx) return fail(nullptr, SPOCK_ERR_INVALID, "spock_chunk_prefill: ctx is NULL");
  if (!d) return fail(ctx, SPOCK_ERR_INVALID, "spock_chunk_prefill: desc is NULL");
  // Same rule as the reference (deltanet_chunk.cpp:55-58): every field non-zero.
  if (d->batch <= 0 || d->num_heads <= 0 || d->seq_len <= 0 || d->key_dim <= 0 ||
      d->value_dim <= 0 || d->chunk_size <= 0)
    return fail(ctx, SPOCK_ERR_INVALID, "DeltaNet chunk config fields must be non-zero");
  if (!q || !k || !v || !g || !beta || !core_out || !final_state)
    return fail(ctx, SPOCK_ERR_INVALID, "spock_chunk_prefill: NULL tensor pointer");
  if (d->dtype_in < SPOCK_F32 || d->dtype_in > SPOCK_BF16 || d->dtype_out < SPOCK_F32 ||
      d->dtype_out > SPOCK_BF16)
    return fail(ctx, SPOCK_ERR_INVALID, "spock_chunk_prefill: unknown dtype");
  DeviceGuard dg(ctx->device);
  if (!dg.ok) return fail(ctx, SPOCK_ERR_CUDA, "spock_chunk_prefill: cannot select device");
  return finish(ctx, spock::launch_chunk_prefill(ctx->chunk, *d, q, k, v, g, beta, init_state,
                                                 core_out, final_state, ctx->d_err_flag,
                                                 (cudaStream_t)stream));
}

__attribute__((visibility("default"))) int spock_chunk_last_to_fp16(
    spock_ctx* ctx, int64_t batch, int64_t num_heads, int64_t seq_len, int64_t value_dim,
    const float* core_out, void* out, void* stream) {
  if (!ctx) return fail(nullptr, SPOCK_ERR_INVALID, "spock_chunk_last_to_fp16: ctx is NULL");
  if (batch <= 0 || num_heads <= 0 || seq_len <= 0 || value_dim <= 0 || !core_out || !out)
    return fail(ctx, SPOCK_ERR_INVALID, "spock_chunk_last_to_fp16: bad arguments");
  DeviceGuard dg(ctx->device);
  return finish(ctx, spock::launch_last_to_fp16(batch, num_heads, seq_len, value_dim, core_out,
                                                out, (cudaStream_t)stream));
}

__attribute__((visibility("default"))) int spock_deltanet_decode_step(
    spock_ctx* ctx, const spock_dn_layer* layer, int64_t batch, void* qkv, void* conv_state,
    float* state, const void* a, const void* b, const void* z, void* out, void* core_raw,
    void* stream) {
  if (!ctx) return fail(nullptr, SPOCK_ERR_INVALID, "spock_deltanet_decode_step: ctx is NULL");
  if (!layer || !qkv || !conv_state || !state || !a || !b || !z || !out || !layer->conv_weight ||
      !layer->a_log_bias || !layer->norm_weight)
    return fail(ctx, SPOCK_ERR_INVALID, "spock_deltanet_decode_step: NULL pointer");
  DeviceGuard dg(ctx->device);
  return finish(ctx, spock::launch_decode_step(*layer, batch, qkv, conv_state, state, a, b, z, out,
                                               core_raw, ctx->d_err_flag, (cudaStream_t)stream));
}

__attribute__((visibility("default"))) int spock_deltanet_recurrent(
    spock_ctx* ctx, int64_t batch, int32_t num_heads, int32_t key_dim, int32_t value_dim,
    const void* q, const void* k, const void* v, const float* g, const float* beta, float* state,
    void* out, void* stream) {
  if (!ctx) return fail(nullptr, SPOCK_ERR_INVALID, "spock_deltanet_recurrent: ctx is NULL");
  if (!q || !k || !v || !g || !beta || !state || !out)
    return fail(ctx, SPOCK_ERR_INVALID, "spock_deltanet_recurrent: NULL pointer");
  DeviceGuard dg(ctx->device);
  return finish(ctx, spock::launch_recurrent(batch, num_heads, key_dim, value_dim, q, k, v, g,
                                             beta, state, out, ctx->d_err_flag, (cudaStream_t)stream));
}

__attribute__((visibility("default"))) int spock_rms_norm(spock_ctx* ctx, const void* x, const void* w, void* y,
                                                          int64_t rows, int32_t dim, float eps, void* stream) {
  if (!ctx) return fail(nullptr, SPOCK_ERR_INVALID, "spock_rms_norm: ctx is NULL");
  if (!x || !w || !y || rows <= 0 || dim <= 0) return fail(ctx, SPOCK_ERR_INVALID, "spock_rms_norm: bad arguments");
  DeviceGuard dg(ctx->device);
  return finish(ctx, spock::op_rms_norm(x, w, y, rows, dim, eps, (cudaStream_t)stream));
}

__attribute__((visibility("default"))) int spock_matvec(spock_ctx* ctx, int32_t epilogue, int32_t exact, const void* w,
                                                        int32_t out_dim, int32_t in_dim, const void* x, int64_t rows,
                                                        void* y, const void* residual, void* stream) {
  if (!ctx) return fail(nullptr, SPOCK_ERR_INVALID, "spock_matvec: ctx is NULL");
  if (!w || !x || !y || rows <= 0 || out_dim <= 0 || in_dim <= 0 || epilogue < SPOCK_MV_STORE ||
      epilogue > SPOCK_MV_ARGMAX || (epilogue == SPOCK_MV_RESIDUAL && !residual))
    return fail(ctx, SPOCK_ERR_INVALID, "spock_matvec: bad arguments");
  if (exact ? in_dim % 16 : (in_dim % 64 || (epilogue != SPOCK_MV_ARGMAX && out_dim % 8)))
    return fail(ctx, SPOCK_ERR_UNSUPPORTED, exact ? "spock_matvec: exact path needs in_dim % 16 == 0"
                                                  : "spock_matvec: fast path needs in_dim % 64 == 0, out_dim % 8 == 0");
  if (epilogue == SPOCK_MV_SILU_GATE && out_dim % 16)
    return fail(ctx, SPOCK_ERR_UNSUPPORTED, "spock_matvec: SILU_GATE needs out_dim % 16 == 0");
  DeviceGuard dg(ctx->device);
  return finish(ctx, spock::op_matvec(ctx->ops, epilogue, exact, w, out_dim, in_dim, x, rows, y, residual, ctx->sms,
                                      (cudaStream_t)stream));
}

__attribute__((visibility("default"))) int spock_argmax(spock_ctx* ctx, const void* logits, int64_t rows, int64_t n,
                                                        int32_t* idx, void* stream) {
  if (!ctx) return fail(nullptr, SPOCK_ERR_INVALID, "spock_argmax: ctx is NULL");
  if (!logits || !idx || rows <= 0 || n <= 0) return fail(ctx, SPOCK_ERR_INVALID, "spock_argmax: bad arguments");
  DeviceGuard dg(ctx->device);
  return finish(ctx, spock::op_argmax(logits, rows, n, idx, (cudaStream_t)stream));
}

__attribute__((visibility("default"))) int spock_attention_decode(spock_ctx* ctx, int32_t exact, const void* proj,
                                                                  const void* q_norm, const void* k_norm, float eps,
                                                                  float rope_theta, const int32_t* pos, void* kv_cache,
                                                                  int32_t max_seq, int64_t rows, void* out,
                                                                  void* stream) {
  if (!ctx) return fail(nullptr, SPOCK_ERR_INVALID, "spock_attention_decode: ctx is NULL");
  if (!proj || !q_norm || !k_norm || !pos || !kv_cache || !out || rows <= 0 || max_seq <= 0)
    return fail(ctx, SPOCK_ERR_INVALID, "spock_attention_decode: bad arguments");
  DeviceGuard dg(ctx->device);
  return finish(ctx, spock::op_attention_decode(ctx->ops, exact, proj, q_norm, k_norm, eps, rope_theta, pos, kv_cache,
                                                max_seq, rows, out, (cudaStream_t)stream));
}

__attribute__((visibility("default"))) int spock_attention_prefill(spock_ctx* ctx, int32_t exact, const void* proj,
                                                                   const void* q_norm, const void* k_norm, float eps,
                                                                   float rope_theta, const int32_t* pos,
                                                                   void* kv_cache, int32_t max_seq, int64_t batch,
                                                                   int32_t len, void* out, void* stream) {
  if (!ctx) return fail(nullptr, SPOCK_ERR_INVALID, "spock_attention_prefill: ctx is NULL");
  if (!proj || !q_norm || !k_norm || !pos || !kv_cache || !out || batch <= 0 || len <= 0 || max_seq <= 0)
    return fail(ctx, SPOCK_ERR_INVALID, "spock_attention_prefill: bad arguments");
  DeviceGuard dg(ctx->device);
  return finish(ctx, spock::op_attention_decode(ctx->ops, exact, proj, q_norm, k_norm, eps, rope_theta, pos, kv_cache,
                                                max_seq, batch * len, out, (cudaStream_t)stream, len));
}

}  // extern "C"
