// K3 — paged chunked-prefill attention (causal over cached prefix blocks + the new chunk).
//
// Semantics: transformers 5.5.0 eager_attention_forward (models/llama/modeling_llama.py:199)
// with a causal mask, as HFBackend runs it for a multi-token step
// (src/tokenserve/backends/hf.py:71), except that the prefix comes from cached blocks of the
// paged pool (src/tokenserve/kv_cache.py:159-177) instead of being recomputed. Query row j of a
// sequence whose step ends at context_lens[s] sits at position context_lens[s] - q_len + j.
#include "common.cuh"

namespace ts {
int paged_attention_portable(void* out, const void* query, int64_t q_stride, const void* kp,
                             const void* vp, const int32_t* bt, int max_blocks,
                             const int32_t* qsl, const int32_t* cl, int num_seqs, int num_rows,
                             int hq, int hkv, int hd, int bs, int64_t nb, float scale, int dtype,
                             cudaStream_t s);
}

extern "C" int ts_paged_prefill(void* out, const void* query, int64_t query_token_stride,
                                const void* key_pool, const void* value_pool,
                                const int32_t* block_tables, int32_t max_blocks_per_seq,
                                const int32_t* query_start_loc, const int32_t* context_lens,
                                int32_t num_seqs, int32_t num_query_tokens, int32_t max_query_len,
                                int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                                int32_t block_size, int64_t num_blocks, float scale, int32_t dtype,
                                void* stream) {
  if (ts::dtype_size(dtype) == 0)
    return ts::set_error(TS_ERR_INVALID_ARGUMENT, "paged_prefill: bad dtype %d", dtype);
  if (num_seqs < 0 || num_query_tokens < 0 || max_query_len < 0 || num_q_heads <= 0 ||
      num_kv_heads <= 0 || num_q_heads % num_kv_heads || head_dim <= 0 || block_size <= 0 ||
      num_blocks <= 0 || max_blocks_per_seq <= 0)
    return ts::set_error(TS_ERR_INVALID_ARGUMENT,
                         "paged_prefill: bad sizes (seqs %d, tokens %d, heads %d/%d, head_dim "
                         "%d, block_size %d)",
                         num_seqs, num_query_tokens, num_q_heads, num_kv_heads, head_dim,
                         block_size);
  if (query_token_stride < int64_t(num_q_heads) * head_dim)
    return ts::set_error(TS_ERR_INVALID_ARGUMENT, "paged_prefill: query stride too small");
  if (num_seqs == 0 || num_query_tokens == 0) return ts::ok();
  if (!out || !query || !key_pool || !value_pool || !block_tables || !query_start_loc ||
      !context_lens)
    return ts::set_error(TS_ERR_INVALID_ARGUMENT, "paged_prefill: null pointer");
  return ts::paged_attention_portable(out, query, query_token_stride, key_pool, value_pool,
                                      block_tables, max_blocks_per_seq, query_start_loc,
                                      context_lens, num_seqs, num_query_tokens, num_q_heads,
                                      num_kv_heads, head_dim, block_size, num_blocks, scale,
                                      dtype, static_cast<cudaStream_t>(stream));
}
