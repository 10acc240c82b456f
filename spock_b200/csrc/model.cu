// Full-model decode session for the Qwen3.5-0.8B layout (the B200 form of
// spock's DecodeSession, src/runtime/vk_session.{hpp,cpp}), batched over
// independent sequences. Per token and layer it follows the reference's
// default (all fast gates on) order (vk_session.cpp:2658-3370):
//   x = rmsnorm(h, input_norm)
//   DeltaNet: [qkv|z|a|b] = W_in x ; conv+L2+g/beta+recurrence+gated norm ;
//             h += W_out (mixer out)
//   attention: [q,gate|k|v] = W_qkv x ; q/k norm, RoPE, KV store ; GQA decode,
//             sigmoid gate ; h += W_o (gated)
//   x = rmsnorm(h, post_norm) ; m = silu(W_gate x) * (W_up x) ; h += W_down m
// then final rmsnorm, tied LM head and argmax (lowest index on ties). Layer i
// is attention iff i % 4 == 3 (src/model/qwen35_config.cpp:5-13).
//
// All weights stay resident (1.5 GB fp16); state per sequence: DeltaNet
// state 18 x 16 x 128 x 128 fp32, conv cache 18 x 6144 x 4 fp16, KV cache
// 6 x max_seq x 2 x 2 x 256 fp16. A step is captured once into a CUDA graph and
// replayed per token.
#include <cmath>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "../apps/json_min.h"
#include "chunk_scratch.h"
#include "common.cuh"
#include "gemm.h"

namespace {
constexpr int HID = 1024, INTER = 3584, DNH = 16, DND = 128, CONV = 6144, DN_IN = 6144 + 2048 + 32;
constexpr int QH = 8, KVH = 2, HD = 256, ATT_IN = QH * HD * 2 + 2 * KVH * HD;  // 5120
}  // namespace

namespace spock {
Status launch_embed(const int* tokens, const void* emb, void* h, int batch, cudaStream_t st);
Status launch_rmsnorm(const void* x, const void* w, void* y, float eps, int batch, cudaStream_t st);
Status launch_attn_prep(const void* qkv, int ld, const void* qn_w, const void* kn_w, const float* rope,
                        const int* pos, void* q_out, void* gate_out, void* kv, int64_t kv_seq_stride,
                        int64_t kv_layer_off, float eps, int rows, cudaStream_t st, int rows_per_seq = 1);
Status launch_attn_decode(const void* q, const void* gate, const void* kv, int64_t kv_seq_stride,
                          int64_t kv_layer_off, const int* pos, float scale, void* out, int rows,
                          cudaStream_t st, int rows_per_seq = 1, float* ws = nullptr, int* tickets = nullptr);
Status launch_attn_prefill_tc(const void* q, const void* gate, const void* kv, int64_t kv_seq_stride, int max_seq,
                              const int* pos, float scale, void* out, int batch, int T, int* err, cudaStream_t st);
Status launch_decode_step_strided(const spock_dn_layer& L, int64_t batch, void* qkv, int qkv_ld,
                                  void* conv_state, float* state, const void* a, const void* b, int ab_ld,
                                  const void* z, int z_ld, void* out, int out_ld, void* core_raw, int* err,
                                  cudaStream_t stream);

namespace {

__global__ void advance_kernel(int* pos, const int* tok_out, int* tok_in, int batch) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  pdl_wait();
  pdl_launch();
  if (b < batch) {
    pos[b] += 1;
    tok_in[b] = tok_out[b];
  }
}
// dst[b * dst_stride + dst_off] = src[b * src_stride + src_off]
__global__ void copy_col_kernel(int* dst, int dst_stride, int dst_off, const int* src, int src_stride, int src_off,
                                int batch) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < batch) dst[(size_t)b * dst_stride + dst_off] = src[(size_t)b * src_stride + src_off];
}
}  // namespace

Status gemm_prepare();
int* ctx_err_word(spock_ctx* ctx);
Status launch_exact_proj(int epi, const void* x, int ldx, const void* w, int K, int N, int batch, void* y, int ldy,
                         const void* res, float* amax_val, int* amax_idx, cudaStream_t st);
Status launch_exact_attn(const void* q, const void* gate, const void* kv, int64_t kv_seq_stride, int64_t kv_layer_off,
                         const int* pos, int max_seq, float scale, void* out, int rows, int rows_per_seq,
                         cudaStream_t st);
Status launch_exact_dn_decode(void* proj, int ld, void* conv, const void* conv_w, const float* alb, const float* norm_w,
                              float eps, float* state, void* out, int ldo, int batch, cudaStream_t st);
Status launch_exact_dn_prefill(const void* proj, int ld, int batch, int T, const void* conv_w, const void* conv_old,
                               void* conv_new, const float* alb, const float* norm_w, float eps, void* q, void* k,
                               void* v, float* g, float* beta, float* core, float* state, void* out,
                               cudaStream_t stream);
Status launch_dn_prefill_conv(const void* proj, int ld, int batch, int T, int H, const void* conv_w,
                              const void* conv_old, void* conv_new, const float* a_log_bias, void* q, void* k, void* v,
                              float* g, float* beta, cudaStream_t st);
Status launch_dn_prefill_gate(const float* core, const void* proj, int ld, int z_off, const float* norm_w, float eps,
                              int batch, int T, int H, void* out, cudaStream_t st);
Status launch_last_rows(const void* src, void* dst, int batch, int T, int width, cudaStream_t st);
Status launch_advance_pos(int* pos, int batch, int T, cudaStream_t st);
Status launch_chunk_prefill(ChunkScratch& scratch, const spock_chunk_desc& d, const void* q, const void* k,
                            const void* v, const float* g, const float* beta, const float* init, void* out,
                            float* final_state, int* err_flag, cudaStream_t stream);

struct ModelLayer {
  bool attn = false;
  void *input_norm = nullptr, *post_norm = nullptr;
  void *w_in = nullptr, *w_out = nullptr;      // DN: [8224][1024], [1024][2048]; attn: [5120][1024], [1024][2048]
  void *conv_w = nullptr;                      // DN fp16 [6144][4]
  float *a_log_bias = nullptr, *dn_norm = nullptr;
  void *q_norm = nullptr, *k_norm = nullptr;
  void *w_gu = nullptr, *w_down = nullptr;     // [7168][1024] (gate/up interleaved by 16 rows), [1024][3584]
  int dn_idx = -1, attn_idx = -1;
};

}  // namespace spock

struct spock_model {
  int device = 0, sms = 148;
  spock_model_desc d{};
  std::string err;
  std::vector<spock::ModelLayer> L;
  std::vector<void*> allocs;
  void *emb = nullptr, *final_norm = nullptr;
  float* rope = nullptr;  // [max_seq][64]
  // activations (bpad rows)
  int bpad = 16, batch = 0;
  void *h = nullptr, *x = nullptr, *proj = nullptr, *mix = nullptr, *mlp = nullptr, *q = nullptr, *gate = nullptr;
  float *ws = nullptr;
  size_t ws_bytes = 0;
  // split decode attention (few rows): partials [rows][2][splits][1032] and tickets [rows][2]
  float* attn_ws = nullptr;
  int* attn_tickets = nullptr;
  float* amax_val = nullptr;
  int* amax_idx = nullptr;
  int *tok_in = nullptr, *tok_out = nullptr, *pos = nullptr;
  int* err_flag = nullptr;      // the context's error word, else own_err
  int* own_err = nullptr;
  // state
  float* dn_state = nullptr;
  void* conv_state = nullptr;
  void* kv = nullptr;
  int64_t kv_seq_stride = 0;
  cudaGraphExec_t graph = nullptr;
  int h_pos = 0;  // tokens processed since reset (all sequences advance together)
  int graph_batch = -1;
  cudaStream_t graph_stream = nullptr;
  // layer-major prefill scratch, grown on demand (rows = batch x prompt length)
  struct Prefill {
    size_t rows = 0;  // capacity
    void* buf = nullptr;
    void *h, *x, *proj, *mix, *mlp, *q, *k, *v, *aq, *agate, *last, *conv_old;
    float *g, *beta, *core;
    int32_t* prompt;  // the replayed graph's prompt rows
  } pf;
  // prefill graph: a prompt shape (batch, length, stream) seen twice in a row
  // is captured and replayed from then on
  cudaGraphExec_t pgraph = nullptr;
  int pg_batch = -1, pg_len = -1;
  cudaStream_t pg_stream = nullptr;
  spock::ChunkScratch chunk_scratch;
};

namespace {
using spock::Status;

int mfail(spock_model* m, int code, const std::string& msg) {
  m->err = msg;
  return code;
}

template <class T>
cudaError_t dalloc(spock_model* m, T** p, size_t bytes) {
  void* v = nullptr;
  cudaError_t e = cudaMalloc(&v, bytes);
  if (e == cudaSuccess) {
    m->allocs.push_back(v);
    cudaMemset(v, 0, bytes);
  }
  *p = static_cast<T*>(v);
  return e;
}

void drop_prefill_graph(spock_model* m) {
  if (m->pgraph) cudaGraphExecDestroy(m->pgraph);
  m->pgraph = nullptr;
  m->pg_batch = m->pg_len = -1;
  m->pg_stream = nullptr;
}

int n_dn(const spock_model* m) { return (int)(m->d.num_layers - m->d.num_layers / 4); }
int n_attn(const spock_model* m) { return (int)(m->d.num_layers / 4); }

Status gemm(spock_model* m, int epi, const void* x, const void* w, int n_out, int k, void* y, int ldy,
            const void* res, cudaStream_t st, const void* norm_w = nullptr, void* xnorm_out = nullptr) {
  spock::GemmArgs a{};
  a.norm_w = (const __half*)norm_w;
  a.eps = m->d.rms_eps;
  a.xnorm_out = (__half*)xnorm_out;
  a.n_out = n_out;
  a.k = k;
  a.batch = m->batch;
  a.bpad = m->bpad;
  a.nsplit = 0;
  a.y = (__half*)y;
  a.ldy = ldy;
  a.res = (const __half*)res;
  a.ws = m->ws;
  a.ws_bytes = m->ws_bytes;
  a.amax_val = m->amax_val;
  a.amax_idx = m->amax_idx;
  a.err = m->err_flag;
  return spock::launch_gemm(epi, x, w, a, m->sms, st);
}

#define TRY(expr)                  \
  do {                             \
    Status _s = (expr);            \
    if (_s.code) return _s;        \
  } while (0)

// ---- exact order (spock_model_desc.exact) ----------------------------------
// The same per-layer sequence as the reference's decode step, every kernel in
// the shaders' reduction order (exact.cu); the RMSNorm and attention-prep
// kernels already follow it.
Status xproj(spock_model* m, int epi, const void* x, int ldx, const void* w, int K, int N, int rows, void* y,
             int ldy, const void* res, cudaStream_t st) {
  return spock::launch_exact_proj(epi, x, ldx, w, K, N, rows, y, ldy, res, m->amax_val, m->amax_idx, st);
}

Status record_step_exact(spock_model* m, cudaStream_t st) {
#ifndef SPOCK_NO_PDL
  spock::pdl_scope pdl_on;
#endif
  if (!st) spock::pdl_enabled() = false;
  const int B = m->batch;
  const float eps = m->d.rms_eps;
  TRY(spock::launch_embed(m->tok_in, m->emb, m->h, B, st));
  for (const auto& l : m->L) {
    TRY(spock::launch_rmsnorm(m->h, l.input_norm, m->x, eps, B, st));
    if (!l.attn) {
      TRY(xproj(m, spock::EPI_F16, m->x, HID, l.w_in, HID, DN_IN, B, m->proj, DN_IN, nullptr, st));
      TRY(spock::launch_exact_dn_decode(m->proj, DN_IN, (uint16_t*)m->conv_state + (size_t)l.dn_idx * B * CONV * 4,
                                        l.conv_w, l.a_log_bias, l.dn_norm, eps,
                                        m->dn_state + (size_t)l.dn_idx * B * DNH * DND * DND, m->mix, DNH * DND, B,
                                        st));
      TRY(xproj(m, spock::EPI_RESIDUAL, m->mix, DNH * DND, l.w_out, DNH * DND, HID, B, m->h, HID, m->h, st));
    } else {
      TRY(xproj(m, spock::EPI_F16, m->x, HID, l.w_in, HID, ATT_IN, B, m->proj, ATT_IN, nullptr, st));
      const int64_t layer_off = (int64_t)l.attn_idx * m->d.max_seq * 2 * KVH * HD;
      TRY(spock::launch_attn_prep(m->proj, ATT_IN, l.q_norm, l.k_norm, m->rope, m->pos, m->q, m->gate, m->kv,
                                  m->kv_seq_stride, layer_off, eps, B, st));
      TRY(spock::launch_exact_attn(m->q, m->gate, m->kv, m->kv_seq_stride, layer_off, m->pos, m->d.max_seq,
                                   1.0f / 16.0f, m->mix, B, 1, st));
      TRY(xproj(m, spock::EPI_RESIDUAL, m->mix, QH * HD, l.w_out, QH * HD, HID, B, m->h, HID, m->h, st));
    }
    TRY(spock::launch_rmsnorm(m->h, l.post_norm, m->x, eps, B, st));
    TRY(xproj(m, spock::EPI_SWIGLU, m->x, HID, l.w_gu, HID, 2 * INTER, B, m->mlp, INTER, nullptr, st));
    TRY(xproj(m, spock::EPI_RESIDUAL, m->mlp, INTER, l.w_down, INTER, HID, B, m->h, HID, m->h, st));
  }
  TRY(spock::launch_rmsnorm(m->h, m->final_norm, m->x, eps, B, st));
  TRY(xproj(m, spock::EPI_ARGMAX, m->x, HID, m->emb, HID, m->d.vocab, B, nullptr, 0, nullptr, st));
  TRY(spock::launch_argmax_finish(m->amax_val, m->amax_idx, (m->d.vocab + 127) / 128, B, m->tok_out, st));
  spock::launch_k(spock::advance_kernel, dim3((B + 127) / 128), dim3(128), 0, st, m->pos, m->tok_out, m->tok_in, B);
  SPOCK_LAUNCH_CHECK("advance_kernel");
  return Status::ok();
}

// One decode token for every sequence: tok_in -> tok_out, h holds the final normed hidden in x.
Status record_step(spock_model* m, cudaStream_t st) {
  if (m->d.exact) return record_step_exact(m, st);
#ifndef SPOCK_NO_PDL
  spock::pdl_scope pdl_on;  // every kernel of the step overlaps its predecessor's tail
#endif
  const int B = m->batch;
  TRY(spock::launch_embed(m->tok_in, m->emb, m->h, B, st));
  const float eps = m->d.rms_eps;
  // RMSNorm then projection. Up to 8 rows the small-batch projection kernel
  // normalises h itself (one launch instead of two).
  const bool fuse = B <= 8;
  auto normed = [&](int epi, const void* norm_w, const void* w, int n_out, void* y, int ldy,
                    void* xnorm_out) -> Status {
    if (fuse) return gemm(m, epi, m->h, w, n_out, HID, y, ldy, nullptr, st, norm_w, xnorm_out);
    TRY(spock::launch_rmsnorm(m->h, norm_w, m->x, eps, B, st));
    return gemm(m, epi, m->x, w, n_out, HID, y, ldy, nullptr, st);
  };
  for (const auto& l : m->L) {
    if (!l.attn) {
      TRY(normed(spock::EPI_F16, l.input_norm, l.w_in, DN_IN, m->proj, DN_IN, nullptr));
      spock_dn_layer dl{DNH, DND, DND, 4, l.conv_w, l.a_log_bias, l.dn_norm, eps, 0};
      __half* p = (__half*)m->proj;  // [batch][qkv 6144 | z 2048 | a 16 | b 16]
      // state and conv caches are [dn layer][sequence][...]
      TRY(spock::launch_decode_step_strided(
          dl, B, p, DN_IN, (uint16_t*)m->conv_state + (size_t)l.dn_idx * B * CONV * 4,
          m->dn_state + (size_t)l.dn_idx * B * DNH * DND * DND, p + CONV + 2048, p + CONV + 2048 + DNH, DN_IN,
          p + CONV, DN_IN, m->mix, DNH * DND, nullptr, m->err_flag, st));
      TRY(gemm(m, spock::EPI_RESIDUAL, m->mix, l.w_out, HID, DNH * DND, m->h, HID, m->h, st));
    } else {
      TRY(normed(spock::EPI_F16, l.input_norm, l.w_in, ATT_IN, m->proj, ATT_IN, nullptr));
      const int64_t layer_off = (int64_t)l.attn_idx * m->d.max_seq * 2 * KVH * HD;
      TRY(spock::launch_attn_prep(m->proj, ATT_IN, l.q_norm, l.k_norm, m->rope, m->pos, m->q, m->gate, m->kv,
                                  m->kv_seq_stride, layer_off, eps, B, st));
      TRY(spock::launch_attn_decode(m->q, m->gate, m->kv, m->kv_seq_stride, layer_off, m->pos, 1.0f / 16.0f,
                                    m->mix, B, st, 1, m->attn_ws, m->attn_tickets));
      TRY(gemm(m, spock::EPI_RESIDUAL, m->mix, l.w_out, HID, QH * HD, m->h, HID, m->h, st));
    }
    TRY(normed(spock::EPI_SWIGLU, l.post_norm, l.w_gu, 2 * INTER, m->mlp, INTER, nullptr));
    TRY(gemm(m, spock::EPI_RESIDUAL, m->mlp, l.w_down, HID, INTER, m->h, HID, m->h, st));
  }
  TRY(normed(spock::EPI_ARGMAX, m->final_norm, m->emb, m->d.vocab, nullptr, 0, m->x));  // x: the normed hidden
  TRY(spock::launch_argmax_finish(m->amax_val, m->amax_idx, (m->d.vocab + 127) / 128, B, m->tok_out, st));
  spock::launch_k(spock::advance_kernel, dim3((B + 127) / 128), dim3(128), 0, st, m->pos, m->tok_out, m->tok_in, B);
  SPOCK_LAUNCH_CHECK("advance_kernel");
  return Status::ok();
}

// Grows the prefill scratch to `rows` token rows (plus one 256-row GEMM block of slack).
Status reserve_prefill(spock_model* m, size_t rows) {
  if (rows <= m->pf.rows) return Status::ok();
  if (m->pf.buf) cudaFree(m->pf.buf);  // waits for the device: no queued work still reads it
  m->pf = spock_model::Prefill{};
  drop_prefill_graph(m);
  const size_t R = rows + 256, B = (size_t)m->d.max_batch;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += (bytes + 255) / 256 * 256;
    return o;
  };
  const size_t o_h = take(R * HID * 2), o_x = take(R * HID * 2), o_proj = take(R * DN_IN * 2),
               o_mix = take(R * 2048 * 2), o_mlp = take(R * INTER * 2), o_q = take(R * 2048 * 2),
               o_k = take(R * 2048 * 2), o_v = take(R * 2048 * 2), o_aq = take(R * QH * HD * 2),
               o_ag = take(R * QH * HD * 2), o_last = take(B * HID * 2), o_conv = take(B * CONV * 4 * 2),
               o_g = take(R * DNH * 4), o_b = take(R * DNH * 4), o_core = take(R * 2048 * 4),
               o_prompt = take(R * 4);
  void* buf = nullptr;
  cudaError_t e = cudaMalloc(&buf, off);
  if (e != cudaSuccess) return Status::err(SPOCK_ERR_ALLOC, "model prefill: scratch allocation failed");
  cudaMemset(buf, 0, off);
  char* c = static_cast<char*>(buf);
  auto& p = m->pf;
  p.buf = buf;
  p.rows = rows;
  p.h = c + o_h;
  p.x = c + o_x;
  p.proj = c + o_proj;
  p.mix = c + o_mix;
  p.mlp = c + o_mlp;
  p.q = c + o_q;
  p.k = c + o_k;
  p.v = c + o_v;
  p.aq = c + o_aq;
  p.agate = c + o_ag;
  p.last = c + o_last;
  p.conv_old = c + o_conv;
  p.g = reinterpret_cast<float*>(c + o_g);
  p.beta = reinterpret_cast<float*>(c + o_b);
  p.core = reinterpret_cast<float*>(c + o_core);
  p.prompt = reinterpret_cast<int32_t*>(c + o_prompt);
  return Status::ok();
}

// A projection over R token rows: row blocks of at most 256 (the GEMM's batch
// limit), no K split (the split accumulator is sized for decode batches).
Status gemm_rows(spock_model* m, int epi, const void* x, const void* w, int n_out, int k, void* y, int ldy,
                 const void* res, int R, cudaStream_t st) {
  // one launch over all R rows (the scratch holds at least R + 256 rows, so the
  // padded rows the tensor map covers are readable)
  spock::GemmArgs a{};
  a.n_out = n_out;
  a.k = k;
  a.batch = R;
  a.bpad = (R + 15) / 16 * 16;
  a.nsplit = 0;  // launch_gemm splits K (in clusters) only to fill the SMs
  a.y = (__half*)y;
  a.ldy = ldy;
  a.res = (const __half*)res;
  a.ws = m->ws;
  a.ws_bytes = m->ws_bytes;
  a.amax_val = m->amax_val;
  a.amax_idx = m->amax_idx;
  a.err = m->err_flag;
  return spock::launch_gemm(epi, x, w, a, m->sms, st);
}

// Exact-order layer-major prefill: every layer over all T prompt tokens
// (rows r = b*T + t); each DeltaNet layer walks the prompt through the
// recurrence token by token (token-serial decode semantics).
Status record_prefill_exact(spock_model* m, const int32_t* prompt, int T, cudaStream_t st) {
  spock::pdl_scope pdl_on;
  if (!st) spock::pdl_enabled() = false;
  const int B = m->batch, R = B * T;
  const float eps = m->d.rms_eps;
  auto& p = m->pf;
  TRY(spock::launch_embed(prompt, m->emb, p.h, R, st));
  for (const auto& l : m->L) {
    TRY(spock::launch_rmsnorm(p.h, l.input_norm, p.x, eps, R, st));
    if (!l.attn) {
      TRY(xproj(m, spock::EPI_F16, p.x, HID, l.w_in, HID, DN_IN, R, p.proj, DN_IN, nullptr, st));
      uint16_t* conv = (uint16_t*)m->conv_state + (size_t)l.dn_idx * B * CONV * 4;
      float* state = m->dn_state + (size_t)l.dn_idx * B * DNH * DND * DND;
      if (cudaMemcpyAsync(p.conv_old, conv, (size_t)B * CONV * 4 * 2, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
        return Status::err(SPOCK_ERR_CUDA, "model prefill: conv snapshot failed");
      TRY(spock::launch_exact_dn_prefill(p.proj, DN_IN, B, T, l.conv_w, p.conv_old, conv, l.a_log_bias, l.dn_norm, eps,
                                         p.q, p.k, p.v, p.g, p.beta, p.core, state, p.mix, st));
      TRY(xproj(m, spock::EPI_RESIDUAL, p.mix, DNH * DND, l.w_out, DNH * DND, HID, R, p.h, HID, p.h, st));
    } else {
      TRY(xproj(m, spock::EPI_F16, p.x, HID, l.w_in, HID, ATT_IN, R, p.proj, ATT_IN, nullptr, st));
      const int64_t layer_off = (int64_t)l.attn_idx * m->d.max_seq * 2 * KVH * HD;
      TRY(spock::launch_attn_prep(p.proj, ATT_IN, l.q_norm, l.k_norm, m->rope, m->pos, p.aq, p.agate, m->kv,
                                  m->kv_seq_stride, layer_off, eps, R, st, T));
      TRY(spock::launch_exact_attn(p.aq, p.agate, m->kv, m->kv_seq_stride, layer_off, m->pos, m->d.max_seq,
                                   1.0f / 16.0f, p.mix, R, T, st));
      TRY(xproj(m, spock::EPI_RESIDUAL, p.mix, QH * HD, l.w_out, QH * HD, HID, R, p.h, HID, p.h, st));
    }
    TRY(spock::launch_rmsnorm(p.h, l.post_norm, p.x, eps, R, st));
    TRY(xproj(m, spock::EPI_SWIGLU, p.x, HID, l.w_gu, HID, 2 * INTER, R, p.mlp, INTER, nullptr, st));
    TRY(xproj(m, spock::EPI_RESIDUAL, p.mlp, INTER, l.w_down, INTER, HID, R, p.h, HID, p.h, st));
  }
  TRY(spock::launch_last_rows(p.h, p.last, B, T, HID, st));
  TRY(spock::launch_rmsnorm(p.last, m->final_norm, m->x, eps, B, st));
  TRY(xproj(m, spock::EPI_ARGMAX, m->x, HID, m->emb, HID, m->d.vocab, B, nullptr, 0, nullptr, st));
  TRY(spock::launch_argmax_finish(m->amax_val, m->amax_idx, (m->d.vocab + 127) / 128, B, m->tok_out, st));
  TRY(spock::launch_advance_pos(m->pos, B, T, st));
  return Status::ok();
}

// Layer-major prefill: every layer over all T prompt tokens of every sequence
// (rows r = b*T + t), then the final norm, LM head and argmax of each
// sequence's last token. DeltaNet layers run the chunk rule over the prompt.
Status record_prefill(spock_model* m, const int32_t* prompt, int T, cudaStream_t st) {
  if (m->d.exact) return record_prefill_exact(m, prompt, T, st);
  spock::pdl_scope pdl_on;  // (the caller disables it on the legacy default stream)
  if (!st) spock::pdl_enabled() = false;
  const int B = m->batch, R = B * T;
  const float eps = m->d.rms_eps;
  auto& p = m->pf;
  TRY(spock::launch_embed(prompt, m->emb, p.h, R, st));
  for (const auto& l : m->L) {
    TRY(spock::launch_rmsnorm(p.h, l.input_norm, p.x, eps, R, st));
    if (!l.attn) {
      TRY(gemm_rows(m, spock::EPI_F16, p.x, l.w_in, DN_IN, HID, p.proj, DN_IN, nullptr, R, st));
      // the decode step's layout: [dn layer][sequence][...] with the session's batch
      uint16_t* conv = (uint16_t*)m->conv_state + (size_t)l.dn_idx * B * CONV * 4;
      float* state = m->dn_state + (size_t)l.dn_idx * B * DNH * DND * DND;
      if (cudaMemcpyAsync(p.conv_old, conv, (size_t)B * CONV * 4 * 2, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
        return Status::err(SPOCK_ERR_CUDA, "model prefill: conv snapshot failed");
      TRY(spock::launch_dn_prefill_conv(p.proj, DN_IN, B, T, DNH, l.conv_w, p.conv_old, conv, l.a_log_bias, p.q, p.k,
                                        p.v, p.g, p.beta, st));
      spock_chunk_desc cd{B, DNH, T, DND, DND, 64, SPOCK_F16, SPOCK_F32, 0, 0};
      TRY(spock::launch_chunk_prefill(m->chunk_scratch, cd, p.q, p.k, p.v, p.g, p.beta, state, p.core, state,
                                      m->err_flag, st));
      TRY(spock::launch_dn_prefill_gate(p.core, p.proj, DN_IN, CONV, l.dn_norm, eps, B, T, DNH, p.mix, st));
      TRY(gemm_rows(m, spock::EPI_RESIDUAL, p.mix, l.w_out, HID, DNH * DND, p.h, HID, p.h, R, st));
    } else {
      TRY(gemm_rows(m, spock::EPI_F16, p.x, l.w_in, ATT_IN, HID, p.proj, ATT_IN, nullptr, R, st));
      const int64_t layer_off = (int64_t)l.attn_idx * m->d.max_seq * 2 * KVH * HD;
      TRY(spock::launch_attn_prep(p.proj, ATT_IN, l.q_norm, l.k_norm, m->rope, m->pos, p.aq, p.agate, m->kv,
                                  m->kv_seq_stride, layer_off, eps, R, st, T));
      if (T > 1)  // query tiles on the tcgen05 tensor cores
        TRY(spock::launch_attn_prefill_tc(p.aq, p.agate, (const __half*)m->kv + layer_off, m->kv_seq_stride,
                                          m->d.max_seq, m->pos, 1.0f / 16.0f, p.mix, B, T, m->err_flag, st));
      else
        TRY(spock::launch_attn_decode(p.aq, p.agate, m->kv, m->kv_seq_stride, layer_off, m->pos, 1.0f / 16.0f, p.mix,
                                      R, st, T, m->attn_ws, m->attn_tickets));
      TRY(gemm_rows(m, spock::EPI_RESIDUAL, p.mix, l.w_out, HID, QH * HD, p.h, HID, p.h, R, st));
    }
    TRY(spock::launch_rmsnorm(p.h, l.post_norm, p.x, eps, R, st));
    TRY(gemm_rows(m, spock::EPI_SWIGLU, p.x, l.w_gu, 2 * INTER, HID, p.mlp, INTER, nullptr, R, st));
    TRY(gemm_rows(m, spock::EPI_RESIDUAL, p.mlp, l.w_down, HID, INTER, p.h, HID, p.h, R, st));
  }
  // each sequence's last token: final norm, LM head, argmax (the decode step's tail)
  TRY(spock::launch_last_rows(p.h, p.last, B, T, HID, st));
  TRY(spock::launch_rmsnorm(p.last, m->final_norm, m->x, eps, B, st));
  TRY(gemm_rows(m, spock::EPI_ARGMAX, m->x, m->emb, m->d.vocab, HID, nullptr, 0, nullptr, B, st));
  TRY(spock::launch_argmax_finish(m->amax_val, m->amax_idx, (m->d.vocab + 127) / 128, B, m->tok_out, st));
  TRY(spock::launch_advance_pos(m->pos, B, T, st));
  return Status::ok();
}

// Runs the layer-major prefill. On a non-default stream, the second call in a
// row with the same (batch, length, stream) captures the launch sequence as a
// graph over the scratch's own prompt buffer; later calls of that shape copy
// the prompt there and replay it. (The first call of a shape runs eagerly, so
// any lazy setup in the launchers has happened before a capture.)
Status run_prefill(spock_model* m, const int32_t* prompt, int T, cudaStream_t st) {
  if (!st) return record_prefill(m, prompt, T, st);
  const bool same = m->pg_batch == m->batch && m->pg_len == T && m->pg_stream == st;
  if (!same) {
    drop_prefill_graph(m);
    m->pg_batch = m->batch;
    m->pg_len = T;
    m->pg_stream = st;
    return record_prefill(m, prompt, T, st);
  }
  if (cudaMemcpyAsync(m->pf.prompt, prompt, (size_t)m->batch * T * 4, cudaMemcpyDefault, st) != cudaSuccess)
    return Status::err(SPOCK_ERR_CUDA, "model prefill: prompt copy failed");
  if (!m->pgraph) {
    Status prep = spock::gemm_prepare();
    if (prep.code) return prep;
    cudaGraph_t g;
    cudaError_t e = cudaStreamBeginCapture(st, cudaStreamCaptureModeRelaxed);
    if (e != cudaSuccess) return spock::cuda_status(e, "model prefill: begin capture");
    Status s = record_prefill(m, m->pf.prompt, T, st);
    e = cudaStreamEndCapture(st, &g);
    if (s.code) return s;
    if (e != cudaSuccess) return spock::cuda_status(e, "model prefill: end capture");
    e = cudaGraphInstantiate(&m->pgraph, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) {
      m->pgraph = nullptr;
      return spock::cuda_status(e, "model prefill: graph instantiate");
    }
  }
  cudaError_t e = cudaGraphLaunch(m->pgraph, st);
  return e == cudaSuccess ? Status::ok() : spock::cuda_status(e, "model prefill: graph launch");
}

Status ensure_graph(spock_model* m, cudaStream_t st) {
  if (m->graph && m->graph_batch == m->batch && m->graph_stream == st) return Status::ok();
  if (m->graph) {
    cudaGraphExecDestroy(m->graph);
    m->graph = nullptr;
  }
  cudaGraph_t g;
  Status prep = spock::gemm_prepare();
  if (prep.code) return prep;
  cudaError_t e = cudaStreamBeginCapture(st, cudaStreamCaptureModeRelaxed);
  if (e != cudaSuccess) return spock::cuda_status(e, "model: begin capture");
  Status s = record_step(m, st);
  e = cudaStreamEndCapture(st, &g);
  if (s.code) return s;
  if (e != cudaSuccess) return spock::cuda_status(e, "model: end capture");
  e = cudaGraphInstantiate(&m->graph, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) return spock::cuda_status(e, "model: graph instantiate");
  m->graph_batch = m->batch;
  m->graph_stream = st;
  return Status::ok();
}

struct Guard {
  int prev = -1;
  explicit Guard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~Guard() {
    int cur;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};
}  // namespace

extern "C" {

__attribute__((visibility("default"))) int spock_model_create(spock_ctx* ctx, const spock_model_desc* d,
                                                              spock_model** out) {
  if (!out || !d) return SPOCK_ERR_INVALID;
  *out = nullptr;
  if (d->num_layers <= 0 || d->num_layers % 4 || d->vocab <= 0 || d->max_batch <= 0 || d->max_batch > 256 ||
      d->max_seq <= 0)
    return SPOCK_ERR_INVALID;
  spock_model* m = new spock_model();
  m->d = *d;
  cudaGetDevice(&m->device);
  cudaDeviceGetAttribute(&m->sms, cudaDevAttrMultiProcessorCount, m->device);
  m->bpad = ((d->max_batch + 15) / 16) * 16;
  const int B = m->bpad;
  bool ok = true;
  auto A = [&](auto** p, size_t bytes) { ok = ok && dalloc(m, p, bytes) == cudaSuccess; };
  A(&m->emb, (size_t)d->vocab * HID * 2);
  A(&m->final_norm, HID * 2);
  A(&m->rope, (size_t)d->max_seq * 64 * 4);
  A(&m->h, (size_t)B * HID * 2);
  A(&m->x, (size_t)B * HID * 2);
  A(&m->proj, (size_t)B * DN_IN * 2);
  A(&m->mix, (size_t)B * 2048 * 2);
  A(&m->mlp, (size_t)B * INTER * 2);
  A(&m->q, (size_t)B * QH * HD * 2);
  A(&m->gate, (size_t)B * QH * HD * 2);
  // projection K-split partials: at most one 128 x 256 fp32 tile per SM
  m->ws_bytes = (size_t)m->sms * 128 * 256 * 4;
  A(&m->ws, m->ws_bytes);
  A(&m->amax_val, (size_t)((d->vocab + 127) / 128) * B * 4);
  A(&m->amax_idx, (size_t)((d->vocab + 127) / 128) * B * 4);
  A(&m->tok_in, (size_t)B * 4);
  A(&m->tok_out, (size_t)B * 4);
  A(&m->pos, (size_t)B * 4);
  A(&m->own_err, 4);
  A(&m->attn_ws, (size_t)64 * 2 * 1032 * 4);  // rows x splits <= 64 (attn_decode_splits)
  A(&m->attn_tickets, (size_t)16 * 2 * 4);
  m->err_flag = ctx ? spock::ctx_err_word(ctx) : m->own_err;
  const int ndn = n_dn(m), nat = n_attn(m);
  A(&m->dn_state, (size_t)ndn * B * DNH * DND * DND * 4);
  A(&m->conv_state, (size_t)ndn * B * CONV * 4 * 2);
  m->kv_seq_stride = (int64_t)nat * d->max_seq * 2 * KVH * HD;
  A(&m->kv, (size_t)B * m->kv_seq_stride * 2);
  m->L.resize(d->num_layers);
  int di = 0, ai = 0;
  for (int i = 0; i < d->num_layers; ++i) {
    auto& l = m->L[i];
    l.attn = (i % 4) == 3;
    A(&l.input_norm, HID * 2);
    A(&l.post_norm, HID * 2);
    A(&l.w_gu, (size_t)2 * INTER * HID * 2);
    A(&l.w_down, (size_t)HID * INTER * 2);
    if (l.attn) {
      l.attn_idx = ai++;
      A(&l.w_in, (size_t)ATT_IN * HID * 2);
      A(&l.w_out, (size_t)HID * QH * HD * 2);
      A(&l.q_norm, HD * 2);
      A(&l.k_norm, HD * 2);
    } else {
      l.dn_idx = di++;
      A(&l.w_in, (size_t)DN_IN * HID * 2);
      A(&l.w_out, (size_t)HID * 2048 * 2);
      A(&l.conv_w, (size_t)CONV * 4 * 2);
      A(&l.a_log_bias, DNH * 2 * 4);
      A(&l.dn_norm, DND * 4);
    }
  }
  if (!ok) {
    spock_model_destroy(m);
    return SPOCK_ERR_ALLOC;
  }
  // RoPE table exactly as DecodeSession builds it (vk_session.cpp:333-346): host fp32
  std::vector<float> rope((size_t)d->max_seq * 64);
  const float theta = d->rope_theta;
  for (int p = 0; p < d->max_seq; ++p)
    for (int i = 0; i < 32; ++i) {
      const float inv_freq = 1.0f / std::pow(theta, 2.0f * (float)i / 64.0f);
      const float ang = (float)p * inv_freq;
      rope[(size_t)p * 64 + 2 * i] = std::cos(ang);
      rope[(size_t)p * 64 + 2 * i + 1] = std::sin(ang);
    }
  cudaMemcpy(m->rope, rope.data(), rope.size() * 4, cudaMemcpyHostToDevice);
  *out = m;
  return SPOCK_OK;
}

__attribute__((visibility("default"))) int spock_model_destroy(spock_model* m) {
  if (!m) return SPOCK_OK;
  if (m->graph) cudaGraphExecDestroy(m->graph);
  drop_prefill_graph(m);
  for (void* p : m->allocs) cudaFree(p);
  if (m->pf.buf) cudaFree(m->pf.buf);
  m->chunk_scratch.release();
  delete m;
  return SPOCK_OK;
}

__attribute__((visibility("default"))) int spock_model_sync(spock_model* m, void* stream) {
  if (!m) return SPOCK_ERR_INVALID;
  Guard g(m->device);
  cudaError_t e = cudaStreamSynchronize((cudaStream_t)stream);
  if (e != cudaSuccess) return mfail(m, SPOCK_ERR_CUDA, std::string("spock_model_sync: ") + cudaGetErrorString(e));
  int flag = 0;
  e = cudaMemcpy(&flag, m->err_flag, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return mfail(m, SPOCK_ERR_CUDA, std::string("spock_model_sync: ") + cudaGetErrorString(e));
  if (!flag) return SPOCK_OK;
  cudaMemset(m->err_flag, 0, sizeof(int));
  return mfail(m, SPOCK_ERR_TIMEOUT,
               "spock_model_sync: a kernel's bounded wait gave up (code " + std::to_string(flag) + ")");
}

__attribute__((visibility("default"))) const char* spock_model_last_error(const spock_model* m) {
  return m ? m->err.c_str() : "";
}

// Roles as in spock's artifact (weight_loader / vk_session.cpp): "embedding",
// "final_norm", "layer.N.<input_norm|post_norm|mlp_gate|mlp_up|mlp_down|
// delta_in_proj_qkv|delta_in_proj_z|delta_in_proj_a|delta_in_proj_b|delta_conv|
// delta_norm|delta_a_log|delta_dt_bias|delta_out_proj|attn_q|attn_k|attn_v|
// attn_q_norm|attn_k_norm|attn_o>". fp16 unless noted: delta_norm and
// delta_a_log are fp32, delta_dt_bias fp16 (kept as fp32 on device).
__attribute__((visibility("default"))) int spock_model_set_weight(spock_model* m, const char* role,
                                                                  const void* host, size_t bytes) {
  if (!m || !role || !host) return SPOCK_ERR_INVALID;
  Guard g(m->device);
  const std::string r(role);
  auto put = [&](void* dst, size_t expect, size_t off = 0) -> int {
    if (bytes != expect) return mfail(m, SPOCK_ERR_INVALID, r + ": expected " + std::to_string(expect) + " bytes");
    return cudaMemcpy((char*)dst + off, host, bytes, cudaMemcpyHostToDevice) == cudaSuccess ? SPOCK_OK
                                                                                            : mfail(m, SPOCK_ERR_CUDA, "copy failed");
  };
  if (r == "embedding") return put(m->emb, (size_t)m->d.vocab * HID * 2);
  if (r == "final_norm") return put(m->final_norm, HID * 2);
  if (r.rfind("layer.", 0) != 0) return mfail(m, SPOCK_ERR_INVALID, "unknown role " + r);
  const size_t dot = r.find('.', 6);
  const int li = std::atoi(r.substr(6, dot - 6).c_str());
  if (dot == std::string::npos || li < 0 || li >= m->d.num_layers) return mfail(m, SPOCK_ERR_INVALID, "bad layer in " + r);
  const std::string n = r.substr(dot + 1);
  auto& l = m->L[li];
  if (n == "input_norm") return put(l.input_norm, HID * 2);
  if (n == "post_norm") return put(l.post_norm, HID * 2);
  if (n == "mlp_down") return put(l.w_down, (size_t)HID * INTER * 2);
  if (n == "mlp_gate" || n == "mlp_up") {
    // interleave gate/up rows in groups of 16 for the fused SwiGLU epilogue
    if (bytes != (size_t)INTER * HID * 2) return mfail(m, SPOCK_ERR_INVALID, r + ": bad size");
    std::vector<uint16_t> buf((size_t)INTER * HID);
    std::memcpy(buf.data(), host, bytes);
    const int half = n == "mlp_up" ? 16 : 0;
    for (int gidx = 0; gidx < INTER / 16; ++gidx)
      if (cudaMemcpy((char*)l.w_gu + ((size_t)(gidx * 32 + half) * HID) * 2, buf.data() + (size_t)gidx * 16 * HID,
                     (size_t)16 * HID * 2, cudaMemcpyHostToDevice) != cudaSuccess)
        return mfail(m, SPOCK_ERR_CUDA, "copy failed");
    return SPOCK_OK;
  }
  if (!l.attn) {
    if (n == "delta_in_proj_qkv") return put(l.w_in, (size_t)CONV * HID * 2, 0);
    if (n == "delta_in_proj_z") return put(l.w_in, (size_t)2048 * HID * 2, (size_t)CONV * HID * 2);
    if (n == "delta_in_proj_a") return put(l.w_in, (size_t)DNH * HID * 2, (size_t)(CONV + 2048) * HID * 2);
    if (n == "delta_in_proj_b") return put(l.w_in, (size_t)DNH * HID * 2, (size_t)(CONV + 2048 + DNH) * HID * 2);
    if (n == "delta_out_proj") return put(l.w_out, (size_t)HID * 2048 * 2);
    if (n == "delta_conv") return put(l.conv_w, (size_t)CONV * 4 * 2);
    if (n == "delta_norm") return put(l.dn_norm, DND * 4);
    if (n == "delta_a_log" || n == "delta_dt_bias") {
      std::vector<float> ab(DNH * 2);
      cudaMemcpy(ab.data(), l.a_log_bias, DNH * 2 * 4, cudaMemcpyDeviceToHost);
      if (n == "delta_a_log") {
        if (bytes != DNH * 4) return mfail(m, SPOCK_ERR_INVALID, r + ": bad size");
        for (int h = 0; h < DNH; ++h) ab[h * 2] = static_cast<const float*>(host)[h];
      } else {
        if (bytes != DNH * 2) return mfail(m, SPOCK_ERR_INVALID, r + ": bad size");
        for (int h = 0; h < DNH; ++h) {
          __half hv;
          std::memcpy(&hv, static_cast<const uint16_t*>(host) + h, 2);
          ab[h * 2 + 1] = __half2float(hv);
        }
      }
      return cudaMemcpy(l.a_log_bias, ab.data(), DNH * 2 * 4, cudaMemcpyHostToDevice) == cudaSuccess ? SPOCK_OK : SPOCK_ERR_CUDA;
    }
  } else {
    if (n == "attn_q") return put(l.w_in, (size_t)QH * HD * 2 * HID * 2, 0);
    if (n == "attn_k") return put(l.w_in, (size_t)KVH * HD * HID * 2, (size_t)QH * HD * 2 * HID * 2);
    if (n == "attn_v") return put(l.w_in, (size_t)KVH * HD * HID * 2, (size_t)(QH * HD * 2 + KVH * HD) * HID * 2);
    if (n == "attn_q_norm") return put(l.q_norm, HD * 2);
    if (n == "attn_k_norm") return put(l.k_norm, HD * 2);
    if (n == "attn_o") return put(l.w_out, (size_t)HID * QH * HD * 2);
  }
  return mfail(m, SPOCK_ERR_INVALID, "unknown role " + r);
}

// Loads the reference's repacked text artifact: <dir>/text_repack_manifest.json
// (written by tools/repack_text_weights.py:178-230, read by
// src/runtime/weight_loader.cpp:22-57) and its aligned blob. Each tensor record
// gives role_path, offset, nbytes and dtype; "global.token_embedding" and
// "global.final_norm" are the embedding and final norm, "layer.N.<role>" the
// per-layer roles above. Every role the model needs must appear exactly once.
__attribute__((visibility("default"))) int spock_model_load_artifact(spock_model* m, const char* dir) {
  if (!m || !dir) return SPOCK_ERR_INVALID;
  const std::string root(dir);
  jm::Value man;
  try {
    man = jm::read_file(root + "/text_repack_manifest.json");
  } catch (const std::exception& e) {
    return mfail(m, SPOCK_ERR_INVALID, std::string("artifact manifest: ") + e.what());
  }
  std::string blob = "text_weights.bin";
  if (const jm::Value* pk = man.get("packing"))
    if (const jm::Value* wf = pk->get("weights_file"))
      if (wf->kind == jm::Value::String) blob = wf->str;
  const jm::Value* tensors = man.get("tensors");
  if (!tensors || tensors->kind != jm::Value::Array) return mfail(m, SPOCK_ERR_INVALID, "artifact manifest: no tensors array");
  std::ifstream f(root + "/" + blob, std::ios::binary);
  if (!f) return mfail(m, SPOCK_ERR_INVALID, "artifact: cannot open " + blob);
  // the roles this model needs
  std::map<std::string, int> need;
  need["embedding"] = 0;
  need["final_norm"] = 0;
  for (int i = 0; i < m->d.num_layers; ++i) {
    const std::string p = "layer." + std::to_string(i) + ".";
    for (const char* r : {"input_norm", "post_norm", "mlp_gate", "mlp_up", "mlp_down"}) need[p + r] = 0;
    if (m->L[i].attn) {
      for (const char* r : {"attn_q", "attn_k", "attn_v", "attn_q_norm", "attn_k_norm", "attn_o"}) need[p + r] = 0;
    } else {
      for (const char* r : {"delta_in_proj_qkv", "delta_in_proj_z", "delta_in_proj_a", "delta_in_proj_b", "delta_conv",
                            "delta_norm", "delta_a_log", "delta_dt_bias", "delta_out_proj"})
        need[p + r] = 0;
    }
  }
  std::vector<char> buf;
  for (const auto& t : tensors->arr) {
    const jm::Value *rp = t.get("role_path"), *off = t.get("offset"), *nb = t.get("nbytes"), *dt = t.get("dtype");
    if (!rp || rp->kind != jm::Value::String || !off || !nb || off->kind != jm::Value::Number ||
        nb->kind != jm::Value::Number)
      return mfail(m, SPOCK_ERR_INVALID, "artifact manifest: tensor record without role_path/offset/nbytes");
    std::string role = rp->str;
    if (role == "global.token_embedding") role = "embedding";
    else if (role == "global.final_norm") role = "final_norm";
    auto it = need.find(role);
    if (it == need.end()) continue;  // roles this model does not use (e.g. other modalities)
    if (it->second++) return mfail(m, SPOCK_ERR_INVALID, "artifact: duplicate role " + rp->str);
    const bool f32_role = role.size() > 10 && (role.compare(role.size() - 10, 10, "delta_norm") == 0 ||
                                               role.compare(role.size() - 11, 11, "delta_a_log") == 0);
    if (dt && dt->kind == jm::Value::String) {
      const bool is32 = dt->str == "fp32" || dt->str == "float32" || dt->str == "f32";
      const bool is16 = dt->str == "fp16" || dt->str == "float16" || dt->str == "f16";
      if (!(f32_role ? is32 : is16))
        return mfail(m, SPOCK_ERR_INVALID, "artifact: " + rp->str + " has dtype " + dt->str);
    }
    const uint64_t o = (uint64_t)off->num, n = (uint64_t)nb->num;
    buf.resize(n);
    f.seekg((std::streamoff)o);
    f.read(buf.data(), (std::streamsize)n);
    if (!f) return mfail(m, SPOCK_ERR_INVALID, "artifact: short read for " + rp->str);
    const int rc = spock_model_set_weight(m, role.c_str(), buf.data(), n);
    if (rc != SPOCK_OK) return rc;
  }
  std::string missing;
  int n_missing = 0;
  for (const auto& kv : need)
    if (!kv.second) {
      if (n_missing++ < 4) missing += (missing.empty() ? "" : ", ") + kv.first;
    }
  if (n_missing) return mfail(m, SPOCK_ERR_INVALID, "artifact: " + std::to_string(n_missing) + " roles missing (" + missing + (n_missing > 4 ? ", ..." : "") + ")");
  return SPOCK_OK;
}

// Zeroes recurrent state, conv and KV caches and positions for `batch` sequences.
__attribute__((visibility("default"))) int spock_model_reset(spock_model* m, int32_t batch) {
  if (!m || batch < 1 || batch > m->d.max_batch) return SPOCK_ERR_INVALID;
  Guard g(m->device);
  m->batch = batch;
  m->h_pos = 0;
  const int B = m->bpad;
  // Work queued on any stream may still use the state: reset between
  // device-wide synchronisations so the clears are ordered on every stream
  // (the caller's streams need not synchronise with the legacy stream).
  cudaDeviceSynchronize();
  cudaMemset(m->dn_state, 0, (size_t)n_dn(m) * B * DNH * DND * DND * 4);
  cudaMemset(m->conv_state, 0, (size_t)n_dn(m) * B * CONV * 4 * 2);
  cudaMemset(m->pos, 0, (size_t)B * 4);
  cudaMemset(m->kv, 0, (size_t)B * m->kv_seq_stride * 2);
  cudaMemset(m->attn_tickets, 0, (size_t)16 * 2 * 4);
  cudaError_t e = cudaDeviceSynchronize();
  return e == cudaSuccess ? SPOCK_OK : mfail(m, SPOCK_ERR_CUDA, cudaGetErrorString(e));
}

// One token per sequence. tokens_in / tokens_out: device int32 [batch];
// hidden_out (nullable): device fp16 [batch][1024], the final-normed hidden.
__attribute__((visibility("default"))) int spock_model_step(spock_model* m, const int32_t* tokens_in,
                                                            int32_t* tokens_out, void* hidden_out, void* stream) {
  if (!m || !tokens_in || m->batch < 1) return SPOCK_ERR_INVALID;
  if (m->h_pos + 1 > m->d.max_seq) return mfail(m, SPOCK_ERR_INVALID, "spock_model_step: past max_seq");
  Guard g(m->device);
  cudaStream_t st = (cudaStream_t)stream;
  ++m->h_pos;
  cudaMemcpyAsync(m->tok_in, tokens_in, (size_t)m->batch * 4, cudaMemcpyDeviceToDevice, st);
  Status s = st ? ensure_graph(m, st) : Status::ok();
  if (s.code) return mfail(m, s.code, s.msg);
  if (st) {
    cudaError_t e = cudaGraphLaunch(m->graph, st);
    if (e != cudaSuccess) return mfail(m, SPOCK_ERR_CUDA, cudaGetErrorString(e));
  } else {
    s = record_step(m, st);
    if (s.code) return mfail(m, s.code, s.msg);
  }
  if (tokens_out) cudaMemcpyAsync(tokens_out, m->tok_out, (size_t)m->batch * 4, cudaMemcpyDeviceToDevice, st);
  if (hidden_out) cudaMemcpyAsync(hidden_out, m->x, (size_t)m->batch * HID * 2, cudaMemcpyDeviceToDevice, st);
  return SPOCK_OK;
}

// Layer-major prefill of prompt [batch][len] (device int32): all layers over
// all prompt tokens at once, the DeltaNet layers through the chunk rule.
// tokens_out [batch] (device int32) receives each sequence's greedy next
// token; hidden_out (nullable, device fp16 [batch][1024]) the final-normed
// hidden of its last prompt token. The session continues from there.
__attribute__((visibility("default"))) int spock_model_prefill(spock_model* m, const int32_t* prompt, int32_t len,
                                                               int32_t* tokens_out, void* hidden_out, void* stream) {
  if (!m || !prompt || len < 1 || m->batch < 1) return SPOCK_ERR_INVALID;
  if (m->h_pos + len > m->d.max_seq) return mfail(m, SPOCK_ERR_INVALID, "spock_model_prefill: past max_seq");
  if ((int64_t)m->batch * len > (1 << 24)) return mfail(m, SPOCK_ERR_INVALID, "spock_model_prefill: batch*len too large");
  Guard g(m->device);
  cudaStream_t st = (cudaStream_t)stream;
  Status s = reserve_prefill(m, (size_t)m->batch * len);
  if (!s.code) s = run_prefill(m, prompt, len, st);
  if (s.code) return mfail(m, s.code, s.msg);
  m->h_pos += len;
  if (tokens_out) cudaMemcpyAsync(tokens_out, m->tok_out, (size_t)m->batch * 4, cudaMemcpyDeviceToDevice, st);
  if (hidden_out) cudaMemcpyAsync(hidden_out, m->x, (size_t)m->batch * HID * 2, cudaMemcpyDeviceToDevice, st);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SPOCK_OK : mfail(m, SPOCK_ERR_CUDA, cudaGetErrorString(e));
}

__attribute__((visibility("default"))) int spock_model_generate(spock_model* m, const int32_t* prompt, int32_t len,
                                                                int32_t n_new, int32_t* out_tokens, void* stream) {
  if (!m || !prompt || len < 1 || n_new < 0 || m->batch < 1) return SPOCK_ERR_INVALID;
  if (m->h_pos + len + n_new > m->d.max_seq) return mfail(m, SPOCK_ERR_INVALID, "spock_model_generate: past max_seq");
  Guard g(m->device);
  cudaStream_t st = (cudaStream_t)stream;
  if (!st) return mfail(m, SPOCK_ERR_INVALID, "spock_model_generate needs a non-default stream (graph replay)");
  // layer-major prefill of the prompt, then greedy decode by graph replay
  int rc = spock_model_prefill(m, prompt, len, nullptr, nullptr, stream);
  if (rc != SPOCK_OK) return rc;
  Status s = ensure_graph(m, st);
  if (s.code) return mfail(m, s.code, s.msg);
  const int B = m->batch;
  const unsigned nb = (unsigned)((B + 127) / 128);
  spock::copy_col_kernel<<<nb, 128, 0, st>>>(m->tok_in, 1, 0, m->tok_out, 1, 0, B);  // first generated token
  for (int i = 0; i < n_new; ++i) {
    // tok_in holds generated token i: record it, then feed it back
    spock::copy_col_kernel<<<nb, 128, 0, st>>>(out_tokens, n_new, i, m->tok_in, 1, 0, B);
    if (i + 1 < n_new) {
      if (cudaGraphLaunch(m->graph, st) != cudaSuccess) return mfail(m, SPOCK_ERR_CUDA, "graph launch failed");
      ++m->h_pos;
    }
  }
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SPOCK_OK : mfail(m, SPOCK_ERR_CUDA, cudaGetErrorString(e));
}

}  // extern "C"
