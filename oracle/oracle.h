// C ABI of the CPU oracle (oracle/liboracle.so). Test infrastructure only.
#pragma once
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif
int oracle_chunk_rule(int64_t num_heads, int64_t seq_len, int64_t key_dim, int64_t value_dim,
                      int64_t chunk_size, int use_qk_l2norm, const float* query,
                      const float* key, const float* value, const float* g, const float* beta,
                      const float* initial_state, float* core_attn_out, float* final_state,
                      int num_threads);
int oracle_conv_l2_qk(int batch, int conv_dim, int kernel_size, int key_total, int num_heads,
                      uint16_t* qkv, uint16_t* conv_state, const uint16_t* conv_w,
                      int num_threads);
int oracle_rec_norm_gate(int batch, int num_heads, int k_dim, int v_dim, float q_scale,
                         float eps, const uint16_t* a, const uint16_t* b,
                         const float* a_log_bias, const uint16_t* qkv, float* state,
                         const uint16_t* z, const float* norm_w, uint16_t* out,
                         int num_threads);
int oracle_recurrent_raw(int num_heads, int k_dim, int v_dim, float q_scale, const uint16_t* q,
                         const uint16_t* k, const uint16_t* v, float* state_with_tail,
                         uint16_t* out);
typedef struct oracle_model oracle_model;
oracle_model* oracle_model_create(int layers, int vocab, int max_seq, float eps, float theta);
void oracle_model_destroy(oracle_model* m);
void oracle_model_set(oracle_model* m, const char* role, const void* ptr);
void oracle_model_reset(oracle_model* m, int batch);
int oracle_model_step(oracle_model* m, const int* tokens, int* out_tokens, uint16_t* hidden_out,
                      float* margin, int threads);
void oracle_matvec(const uint16_t* W, const uint16_t* x, int out, int in, uint16_t* y, int threads);
void oracle_rms_norm(const uint16_t* x, const uint16_t* w, float eps, uint16_t* y);
int oracle_argmax(const uint16_t* logits, int n);
void oracle_attention_decode(const uint16_t* proj, const uint16_t* qn_w, const uint16_t* kn_w, float eps, float theta,
                             uint16_t* cache, int pos, uint16_t* gated);
void oracle_silu_gate(int64_t n, const uint16_t* gate, const uint16_t* up, uint16_t* out);
void oracle_residual_add(int64_t n, const uint16_t* a, const uint16_t* b, uint16_t* out);
void oracle_gbeta(int H, const uint16_t* a, const uint16_t* b, const float* a_log_bias, float* g, float* beta);
void oracle_f32_to_f16(const float* x, uint16_t* y, int64_t n);
void oracle_f16_to_f32(const uint16_t* x, float* y, int64_t n);
#ifdef __cplusplus
}
#endif
