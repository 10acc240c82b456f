// Per-context scratch of the decode-glue operations (ops.cu), grown on demand.
#pragma once
#include "chunk_scratch.h"
#include "common.cuh"

namespace spock {
struct OpsScratch {
  ChunkScratch xpad;     // fast projections: x zero-padded to a multiple of 16 rows
  ChunkScratch ws;       // projection K-split partials
  ChunkScratch amax;     // argmax partials [tiles][rows] value + index
  ChunkScratch qg;       // attention: normalised / rotated q and the gate
  ChunkScratch rope;     // RoPE table [rope_seq][64]
  ChunkScratch attn_ws;  // split decode attention: partials
  ChunkScratch attn_tk;  // split decode attention: tickets (zero between launches)
  float rope_theta = 0.f;
  int rope_seq = 0;
  int* err = nullptr;    // the context's error word
  void release() {
    for (ChunkScratch* s : {&xpad, &ws, &amax, &qg, &rope, &attn_ws, &attn_tk}) s->release();
  }
};

Status op_rms_norm(const void* x, const void* w, void* y, int64_t rows, int dim, float eps, cudaStream_t st);
Status op_argmax(const void* logits, int64_t rows, int64_t n, int32_t* idx, cudaStream_t st);
Status op_matvec(OpsScratch& sc, int epilogue, int exact, const void* w, int out_dim, int in_dim, const void* x,
                 int64_t rows, void* y, const void* res, int sms, cudaStream_t st);
Status op_attention_decode(OpsScratch& sc, int exact, const void* proj, const void* qn, const void* kn, float eps,
                           float theta, const int32_t* pos, void* kv, int max_seq, int64_t rows, void* out,
                           cudaStream_t st, int rows_per_seq = 1);
}  // namespace spock
