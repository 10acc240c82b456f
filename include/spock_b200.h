/*
 * spock_b200 — C ABI of the B200 (sm_100a) Gated DeltaNet hot path.
 *
 * This is the drop-in boundary that replaces the Vulkan command-buffer /
 * descriptor layer behind spock's DeltaNet entry points. Every function takes
 * plain pointers and sizes, returns a status code (never throws, never aborts)
 * and enqueues its work asynchronously on the given CUDA stream (NULL = the
 * legacy default stream). All tensor pointers are DEVICE pointers owned by the
 * caller unless stated otherwise. Layouts are row-major, innermost last.
 *
 * There is no CPU fallback: a call on a machine without an sm_100 GPU returns
 * SPOCK_ERR_CUDA with the CUDA error text in spock_last_error().
 */
#ifndef SPOCK_B200_H
#define SPOCK_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. Replaces the std::runtime_error thrown by the reference
 * (src/runtime/deltanet_chunk.cpp:41-58, src/runtime/vk_device.cpp). */
typedef enum {
  SPOCK_OK = 0,
  SPOCK_ERR_INVALID = -1,     /* zero / negative field, size mismatch, NULL pointer */
  SPOCK_ERR_UNSUPPORTED = -2, /* a shape the CUDA kernels do not implement */
  SPOCK_ERR_CUDA = -3,        /* a CUDA runtime / driver call failed */
  SPOCK_ERR_ALLOC = -4,       /* device allocation failed */
  SPOCK_ERR_TIMEOUT = -5      /* a bounded device-side wait gave up */
} spock_status;

typedef enum { SPOCK_F32 = 0, SPOCK_F16 = 1, SPOCK_BF16 = 2 } spock_dtype;

/* Opaque per-GPU context: device ordinal, scratch buffers, error text.
 * Replaces spock::runtime::VulkanDevice (src/runtime/vk_device.hpp:29-117).
 * One context per GPU; calls on one context must not race from several host
 * threads (the same contract as DecodeSession, src/runtime/vk_session.hpp:27-28). */
typedef struct spock_ctx spock_ctx;

int spock_create(int device, spock_ctx** out);
int spock_destroy(spock_ctx* ctx);
/* Text of the last error on this context (or of the last context-less error
 * when ctx is NULL). Valid until the next call on the same context. */
const char* spock_last_error(const spock_ctx* ctx);
/* Blocks until the stream's work is done; returns SPOCK_ERR_TIMEOUT when a
 * kernel reported a bounded wait that gave up. */
int spock_sync(spock_ctx* ctx, void* stream);
/* Number of kernels this library has launched since load (diagnostics). */
uint64_t spock_kernel_launch_count(void);
/* Failure-detection self-test: launches one CTA that waits on a device
 * barrier nothing will complete, with the same bounded polling the chunk,
 * decode and projection kernels use, capped at `polls` polls. The wait gives
 * up, records the timeout in the context's error word and the kernel returns,
 * so the next spock_sync reports SPOCK_ERR_TIMEOUT and the context stays
 * usable. No GPU fault is involved. With ctx == NULL the wait records into the
 * error word of spock_chunk_prefill_noalloc's fixed array on the current
 * device instead, which spock_noalloc_sync then reports. */
int spock_selftest_wait_timeout(spock_ctx* ctx, uint32_t polls, void* stream);

/* ------------------------------------------------------------------------ */
/* Chunked gated delta rule (prefill).                                      */
/* ------------------------------------------------------------------------ */

/* Replaces spock::runtime::DeltaNetChunkConfig (src/runtime/deltanet_chunk.hpp:8-15),
 * extended with a batch of independent sequences and storage dtypes. */
typedef struct {
  int64_t batch;         /* independent sequences, >= 1 */
  int64_t num_heads;     /* >= 1 */
  int64_t seq_len;       /* tokens per sequence, >= 1; padded internally to chunk_size */
  int64_t key_dim;       /* 128 on the CUDA path */
  int64_t value_dim;     /* 128 on the CUDA path */
  int64_t chunk_size;    /* 64 on the CUDA path */
  int32_t dtype_in;      /* q, k, v storage: SPOCK_F32 / SPOCK_F16 / SPOCK_BF16 */
  int32_t dtype_out;     /* core_attn_out storage: SPOCK_F32 / SPOCK_F16 / SPOCK_BF16 */
  int32_t use_qk_l2norm; /* 1: L2-normalise q and k per (head, token), eps 1e-6 */
  int32_t reserved;
} spock_chunk_desc;

/*
 * Replaces run_deltanet_chunk_rule (src/runtime/deltanet_chunk.hpp:39-40,
 * src/runtime/deltanet_chunk.cpp:53-284) and the GPU dispatch of
 * deltanet_chunk_prefill_tiled.comp in
 * DecodeSession::gpu_chunk_prefill_from_gpu_collect
 * (src/runtime/vk_session.cpp:4466-4828).
 *
 *   q, k        [batch][num_heads][seq_len][key_dim]    dtype_in
 *   v           [batch][num_heads][seq_len][value_dim]  dtype_in
 *   g, beta     [batch][num_heads][seq_len]             fp32 (log-decay, write strength)
 *   init_state  [batch][num_heads][key_dim][value_dim]  fp32, NULL = zeros
 *   core_out    [batch][num_heads][seq_len][value_dim]  dtype_out
 *   final_state [batch][num_heads][key_dim][value_dim]  fp32 (may alias init_state)
 *
 * Internally the intra-chunk contractions run on tcgen05 tensor cores with
 * fp16 operands and fp32 accumulation in TMEM; the recurrent state is fp32.
 * Range: bf16 q/k/v are converted to fp16 operands, so values must lie in
 * fp16's range (|x| <= 65504; larger magnitudes become inf) and values below
 * 2^-14 lose precision as fp16 subnormals. The model's inputs (L2-normalised
 * q/k, O(1) v) are far inside it; fp32 inputs are staged as fp16 hi/lo pairs.
 * fp32 inputs, or use_qk_l2norm=1, are first staged as fp16 in the context's
 * device scratch (grown on demand with cudaMalloc).
 */
int spock_chunk_prefill(spock_ctx* ctx, const spock_chunk_desc* desc, const void* q,
                        const void* k, const void* v, const float* g, const float* beta,
                        const float* init_state, void* core_out, float* final_state,
                        void* stream);

/*
 * Allocation-free form of spock_chunk_prefill, for callers that cannot
 * allocate device memory when they call in: code running under an allocator
 * or memory budget it does not own, code that must not risk the device-wide
 * synchronisation cudaMalloc/cudaFree can cause, and plugins handed only the
 * caller's buffers with no context. It has no counterpart in the reference.
 *
 * Same arguments, layouts and results as spock_chunk_prefill, but no context:
 * the fp16 staging of q/k/v (needed for fp32 inputs or use_qk_l2norm=1) goes
 * to a fixed 24 MiB array compiled into the library, held on every GPU that
 * loads it until the process exits. Limit when staging is needed:
 * batch*num_heads*seq_len <= 16384; larger requests return SPOCK_ERR_INVALID
 * with the reason in spock_last_error(NULL). The call enqueues work on the
 * current device and calls no cudaMalloc, cudaFree or other allocating routine.
 * The first call on each device looks up the array's device address
 * (cudaGetSymbolAddress); make that first call before any stream capture.
 * Under CUDA's lazy module loading that first lookup is also when the driver
 * loads the library's device code and commits the 24 MiB array on that
 * device, so the first call (or first spock_noalloc_sync) on a device costs
 * 24 MiB of device memory once; later calls allocate nothing.
 * All calls on a device share the array, so calls whose work overlaps on the
 * GPU (different streams, no ordering between them) race and must not be made.
 *
 * A bounded device-side wait that gives up does not fail the call (the work is
 * asynchronous); it sets an error word at the head of the fixed array, which
 * stays set until spock_noalloc_sync reads it. Outputs of a call followed by
 * a SPOCK_ERR_TIMEOUT from spock_noalloc_sync are invalid.
 */
int spock_chunk_prefill_noalloc(const spock_chunk_desc* desc, const void* q, const void* k,
                                const void* v, const float* g, const float* beta,
                                const float* init_state, void* core_out, float* final_state,
                                void* stream);

/*
 * Companion of spock_chunk_prefill_noalloc (no counterpart in the reference):
 * synchronises `stream`, then reads the fixed array's error word on the
 * current device. Returns SPOCK_ERR_TIMEOUT (text in spock_last_error(NULL))
 * when a kernel of an earlier allocation-free call reported a bounded wait
 * that gave up, and clears the word only after reading it; SPOCK_OK otherwise.
 * Allocates nothing.
 */
int spock_noalloc_sync(void* stream);

/*
 * Last-token extraction of core_attn_out to fp16 by truncation with
 * flush-to-zero, as deltanet_chunk_last_to_fp16.comp:37-66 does for the
 * prefill -> decode handoff (src/runtime/vk_session.cpp:4621-4631).
 *   core_out [batch][num_heads][seq_len][value_dim] fp32 -> out [batch][num_heads*value_dim] fp16
 */
int spock_chunk_last_to_fp16(spock_ctx* ctx, int64_t batch, int64_t num_heads, int64_t seq_len,
                             int64_t value_dim, const float* core_out, void* out, void* stream);

/* ------------------------------------------------------------------------ */
/* Fused single-token DeltaNet decode step.                                 */
/* ------------------------------------------------------------------------ */

/* Per-layer constants of one Gated DeltaNet layer (Qwen3.5-0.8B: 16 heads,
 * key/value dim 128, conv width 4, conv_dim = heads*(2*key_dim+value_dim) = 6144). */
typedef struct {
  int32_t num_heads;
  int32_t key_dim;
  int32_t value_dim;
  int32_t conv_kernel;      /* depthwise conv width (4) */
  const void* conv_weight;  /* fp16 [conv_dim][conv_kernel] */
  const float* a_log_bias;  /* fp32 [num_heads][2]: (A_log, dt_bias) per head */
  const float* norm_weight; /* fp32 [value_dim]: gated RMSNorm weight */
  float eps;                /* RMSNorm epsilon (1e-6) */
  int32_t reserved;
} spock_dn_layer;

/*
 * One decode token for `batch` independent sequences through one DeltaNet
 * layer's mixer core. Replaces the fused pair deltanet_conv_l2_qk.comp
 * (:41-110) + deltanet_recurrent_gbeta_norm_gate.comp (:91-224) dispatched
 * from DecodeSession::decode (src/runtime/vk_session.cpp:2878-2883, 3213-3218),
 * fused into ONE kernel (one CTA per (sequence, head)).
 *
 *   qkv        [batch][conv_dim] fp16, in/out: raw projection in; conv+SiLU
 *              output with Q/K L2-normalised out (the reference's in-place contract)
 *   conv_state [batch][conv_dim][conv_kernel] fp16, in/out (shift + insert)
 *   state      [batch][num_heads][key_dim][value_dim] fp32, in/out
 *   a, b       [batch][num_heads] fp16 raw gate projections
 *   z          [batch][num_heads*value_dim] fp16 output gate
 *   out        [batch][num_heads*value_dim] fp16 gated, normalised mixer output
 *   core_raw   optional [batch][num_heads*value_dim] fp16: raw S^T q before the
 *              norm-gate (deltanet_recurrent.comp's output); NULL to skip
 */
int spock_deltanet_decode_step(spock_ctx* ctx, const spock_dn_layer* layer, int64_t batch,
                               void* qkv, void* conv_state, float* state, const void* a,
                               const void* b, const void* z, void* out, void* core_raw,
                               void* stream);

/*
 * Unfused recurrent update with g/beta given directly, the contract of
 * deltanet_recurrent.comp:55-125 (g and beta read from the state tail there):
 *   q, k, v  [batch][num_heads*key_dim] fp16 (q already L2-normalised, unscaled)
 *   g, beta  [batch][num_heads] fp32
 *   state    [batch][num_heads][key_dim][value_dim] fp32 in/out
 *   out      [batch][num_heads*value_dim] fp16 raw S^T (q/sqrt(key_dim))
 */
int spock_deltanet_recurrent(spock_ctx* ctx, int64_t batch, int32_t num_heads, int32_t key_dim,
                             int32_t value_dim, const void* q, const void* k, const void* v,
                             const float* g, const float* beta, float* state, void* out,
                             void* stream);

/* ------------------------------------------------------------------------ */
/* Decode-glue operations, one reference shader dispatch each.               */
/* ------------------------------------------------------------------------ */
/* For callers that keep the reference's own per-layer orchestration
 * (DecodeSession::decode, src/runtime/vk_session.cpp:2658-3370, dispatches
 * these shaders one by one). They run the kernels of the model session.
 * `exact` = 1 selects the exact-order kernels (each reduction in the shader's
 * own order: results bit-identical to the shader restatement), 0 the fast
 * ones. Device pointers, fp16 unless stated, rows contiguous. */

/* rms_norm.comp:31-70: y[r] = fp16(x[r] * 1/sqrt(mean(x[r]^2) + eps) * (1 + w)),
 * dim = 1024 (the hidden size; the only width the kernel implements). y may
 * alias x; x, w and y are 8-byte aligned (SPOCK_ERR_INVALID otherwise). */
int spock_rms_norm(spock_ctx* ctx, const void* x, const void* w, void* y, int64_t rows, int32_t dim, float eps,
                   void* stream);

typedef enum {
  SPOCK_MV_STORE = 0,     /* y[r][n] = fp16(W[n] . x[r])                                      */
  SPOCK_MV_RESIDUAL = 1,  /* y[r][n] = fp16(res[r][n] + fp16(W[n] . x[r])) (residual_add.comp) */
  SPOCK_MV_SILU_GATE = 2, /* W: 2*out_dim rows, gate and up rows interleaved in groups of 16;
                             y[r][p] = fp16(silu(fp16(gate_p . x[r])) * fp16(up_p . x[r]))
                             (silu_gate.comp)                                                  */
  SPOCK_MV_ARGMAX = 3     /* y: int32 [rows], the index of the largest fp16(W[n] . x[r]),
                             lowest index among equal maxima (lm_head_tiled + argmax.comp)     */
} spock_matvec_epilogue;

/* matvec.comp:28-41 over `rows` activation rows with a fused epilogue.
 * W [out_dim (x2 for SILU_GATE)][in_dim], x [rows][in_dim], y [rows][out_dim]
 * (ARGMAX: int32 [rows]); residual [rows][out_dim] for RESIDUAL (y may alias it).
 * Fast path (exact = 0): in_dim % 64 == 0, out_dim % 8 == 0, rows <= 65536,
 * ARGMAX at rows <= 8 needs in_dim <= 1024. Exact path: in_dim % 16 == 0.
 * Scratch (padded x, split-K workspace, argmax partials) grows in the context
 * and is shared by its calls: calls on one context whose work overlaps on the
 * GPU (different streams) must be ordered by the caller. */
int spock_matvec(spock_ctx* ctx, int32_t epilogue, int32_t exact, const void* w, int32_t out_dim, int32_t in_dim,
                 const void* x, int64_t rows, void* y, const void* residual, void* stream);

/* argmax.comp:27-62: idx[r] (int32) = the index of the largest fp16 logit of
 * row r of logits [rows][n], lowest index among equal maxima. */
int spock_argmax(spock_ctx* ctx, const void* logits, int64_t rows, int64_t n, int32_t* idx, void* stream);

/* One decode token of gated full attention (Qwen3.5 layout: 8 q heads, 2 kv
 * heads, head dim 256) for `rows` independent sequences: split_q_gate,
 * rms_norm_per_head (q_norm, k_norm: fp16 [256], (1+w) form), rope_apply
 * (rotary 64 of 256, theta), kv_cache_store, attention_decode.comp:64-143
 * (scale 1/16) and sigmoid_gate.
 *   proj     [rows][5120]: per q head [q 256 | gate 256] x 8, then k (2 x 256), v (2 x 256)
 *   pos      int32 [rows]: this token's position in each sequence (< max_seq)
 *   kv_cache [rows][max_seq][K|V][2][256], in/out (row pos is written)
 *   out      [rows][2048] gated attention output */
int spock_attention_decode(spock_ctx* ctx, int32_t exact, const void* proj, const void* q_norm, const void* k_norm,
                           float eps, float rope_theta, const int32_t* pos, void* kv_cache, int32_t max_seq,
                           int64_t rows, void* out, void* stream);

/* The same for `len` consecutive prompt tokens of each of `batch` sequences
 * (the layer-major prefill's attention, vk_session.cpp:1166-1443 in the
 * reference): proj [batch][len][5120]; pos int32 [batch] is each sequence's
 * first prompt position (token t sits at pos + t); every row's K/V is stored
 * first, then row t attends causally to positions 0 .. pos + t.
 * out [batch][len][2048]. The fast path runs the tcgen05 tile kernel. */
int spock_attention_prefill(spock_ctx* ctx, int32_t exact, const void* proj, const void* q_norm, const void* k_norm,
                            float eps, float rope_theta, const int32_t* pos, void* kv_cache, int32_t max_seq,
                            int64_t batch, int32_t len, void* out, void* stream);

/* ------------------------------------------------------------------------ */
/* Full-model decode (Qwen3.5-0.8B layout): the decode glue around the mixer. */
/* ------------------------------------------------------------------------ */

/* Replaces DecodeSession (src/runtime/vk_session.hpp:22-46) for batched,
 * independent sequences; one instance per GPU. */
typedef struct spock_model spock_model;

typedef struct {
  int32_t num_layers; /* multiple of 4; layer i is attention iff i % 4 == 3 (24) */
  int32_t vocab;      /* 248320 (LM head tied to the embedding) */
  int32_t max_batch;  /* sequences per step, <= 256 */
  int32_t max_seq;    /* KV-cache capacity, MAX_SEQ (2048) in the reference */
  float rms_eps;      /* 1e-6 */
  float rope_theta;   /* 1e7 (vk_session.cpp:335) */
  /* 0: tensor-core projections and the chunk rule in prefill (fp16-ULP parity
   *    with the CPU restatement; prefill semantics of the reference's
   *    layer_major_prefill + chunk-rule state).
   * 1: exact order: every reduction in the reference shaders' own order on
   *    CUDA cores (sequential matvec dots, two-pass attention softmax,
   *    per-column DeltaNet recurrence), prompt tokens walked through the
   *    recurrence one by one; hidden states and greedy tokens bit-identical
   *    to the CPU restatement of the shaders. */
  int32_t exact;
  int32_t reserved;
} spock_model_desc;

/* ctx (nullable) supplies the error word of the model's bounded device waits:
 * with a ctx, spock_sync(ctx, ...) reports a model kernel's timeout as well;
 * spock_model_sync reads the same word either way. */
int spock_model_create(spock_ctx* ctx, const spock_model_desc* desc, spock_model** out);
int spock_model_destroy(spock_model* m);
/* Blocks until the stream's work is done; returns SPOCK_ERR_TIMEOUT (text in
 * spock_model_last_error) when a kernel of this model's prefill, step or
 * generate reported a bounded wait that gave up, clearing the word after
 * reading it. The outputs of that work are invalid; spock_model_reset clears
 * the state and the projection workspace before the session is used again. */
int spock_model_sync(spock_model* m, void* stream);
const char* spock_model_last_error(const spock_model* m);
/* Uploads one tensor by the reference artifact's role name (weight_loader.hpp
 * find_by_role: "embedding", "final_norm", "layer.N.delta_in_proj_qkv", ...);
 * host pointer, fp16 unless the role is fp32 in the artifact. */
int spock_model_set_weight(spock_model* m, const char* role, const void* host, size_t bytes);
/* Loads every tensor the model needs from a repacked text artifact directory
 * (text_repack_manifest.json + text_weights.bin, the format
 * src/runtime/weight_loader.cpp:22-57 reads): role_path "global.token_embedding",
 * "global.final_norm" and "layer.N.<role>". SPOCK_ERR_INVALID names missing,
 * duplicate or mistyped roles. Replaces WeightArtifact::load + the per-role
 * uploads of DecodeSession (vk_session.cpp:1151-1462). */
int spock_model_load_artifact(spock_model* m, const char* repack_dir);
/* Zeroes DeltaNet/conv/KV state and positions for `batch` sequences
 * (DecodeSession::reset, vk_session.cpp:980). Synchronises the device before
 * and after the clears, so it is ordered against work on every stream. */
int spock_model_reset(spock_model* m, int32_t batch);
/* One token per sequence through all layers, final norm, LM head and argmax.
 * tokens_in/out: device int32 [batch]; hidden_out (nullable): device fp16
 * [batch][1024], the final-normed hidden. Replaces one iteration of the decode
 * loop (vk_session.cpp:2298-4190). */
int spock_model_step(spock_model* m, const int32_t* tokens_in, int32_t* tokens_out, void* hidden_out,
                     void* stream);
/* Layer-major prefill of prompt [batch][len] (device int32; the reference's
 * layer_major_prefill, vk_session.cpp:1003-2018, batched): every layer over
 * all prompt tokens at once, DeltaNet layers through the chunk rule. Writes
 * each sequence's greedy next token to tokens_out [batch] (device int32) and,
 * when non-NULL, the final-normed hidden of its last prompt token to
 * hidden_out (device fp16 [batch][1024]). Decoding continues from there. */
int spock_model_prefill(spock_model* m, const int32_t* prompt, int32_t len, int32_t* tokens_out,
                        void* hidden_out, void* stream);
/* Prefill of prompt [batch][len] (spock_model_prefill) then n_new greedy
 * tokens (graph-replayed decode steps) into out_tokens [batch][n_new]
 * (device int32). Requires a non-default stream. */
int spock_model_generate(spock_model* m, const int32_t* prompt, int32_t len, int32_t n_new,
                         int32_t* out_tokens, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* SPOCK_B200_H */
