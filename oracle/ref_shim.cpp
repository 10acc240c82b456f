// C ABI around the reference's own chunk rule, compiled from the reference's
// unmodified sources (src/runtime/deltanet_chunk.{hpp,cpp}) by oracle/Makefile
// into oracle/_ref/libref_chunk.so. Test infrastructure only: it pins the
// oracle restatement and serves as bench.py's reference arm.
#include <cstdint>
#include <cstring>
#include <exception>
#include <thread>
#include <vector>

#include "runtime/deltanet_chunk.hpp"

extern "C" int ref_chunk_rule(int64_t num_heads, int64_t seq_len, int64_t key_dim,
                              int64_t value_dim, int64_t chunk_size, int use_qk_l2norm,
                              const float* q, const float* k, const float* v, const float* g,
                              const float* beta, const float* init, float* out, float* state) {
  try {
    spock::runtime::DeltaNetChunkConfig c;
    c.num_heads = (size_t)num_heads;
    c.sequence_length = (size_t)seq_len;
    c.key_dim = (size_t)key_dim;
    c.value_dim = (size_t)value_dim;
    c.chunk_size = (size_t)chunk_size;
    c.use_qk_l2norm = use_qk_l2norm != 0;
    const size_t nq = c.num_heads * c.sequence_length * c.key_dim;
    const size_t nv = c.num_heads * c.sequence_length * c.value_dim;
    const size_t ns = c.num_heads * c.sequence_length;
    spock::runtime::DeltaNetChunkInputs in;
    in.query.assign(q, q + nq);
    in.key.assign(k, k + nq);
    in.value.assign(v, v + nv);
    in.g.assign(g, g + ns);
    in.beta.assign(beta, beta + ns);
    if (init) in.initial_state.assign(init, init + c.num_heads * c.key_dim * c.value_dim);
    auto o = spock::runtime::run_deltanet_chunk_rule(c, in);
    std::memcpy(out, o.core_attn_out.data(), o.core_attn_out.size() * sizeof(float));
    std::memcpy(state, o.final_state.data(), o.final_state.size() * sizeof(float));
    return 0;
  } catch (const std::exception&) {
    return -1;
  }
}

// Independent sequences ([batch][head][seq][dim] blocks) on a thread pool, one
// reference call per sequence; used to time the reference on all host cores.
extern "C" int ref_chunk_rule_batched(int64_t batch, int64_t num_heads, int64_t seq_len,
                                      int64_t key_dim, int64_t value_dim, int64_t chunk_size,
                                      const float* q, const float* k, const float* v,
                                      const float* g, const float* beta, float* out,
                                      float* state, int threads) {
  const size_t nq = (size_t)num_heads * seq_len * key_dim;
  const size_t nv = (size_t)num_heads * seq_len * value_dim;
  const size_t ns = (size_t)num_heads * seq_len;
  const size_t nst = (size_t)num_heads * key_dim * value_dim;
  std::vector<int> rc(batch, 0);
  auto work = [&](int t) {
    for (int64_t b = t; b < batch; b += threads)
      rc[b] = ref_chunk_rule(num_heads, seq_len, key_dim, value_dim, chunk_size, 0, q + b * nq,
                             k + b * nq, v + b * nv, g + b * ns, beta + b * ns, nullptr,
                             out + b * nv, state + b * nst);
  };
  std::vector<std::thread> th;
  for (int t = 0; t < threads; ++t) th.emplace_back(work, t);
  for (auto& x : th) x.join();
  for (int r : rc)
    if (r) return r;
  return 0;
}
