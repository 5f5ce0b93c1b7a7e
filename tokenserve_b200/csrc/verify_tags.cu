// Device shadow-KV check: every position of every sequence, read back through its block table,
// must hold the token id the host expects. This is the read half of tokenserve's
// SimulatedBackend._write_and_verify (src/tokenserve/backends/simulated.py:161-169), run on the
// int32 tag pool that ts_reshape_and_cache fills next to the K/V rows.
#include "common.cuh"

namespace {

// One CTA per sequence; mismatch_pos[b] = smallest mismatching position, or -1.
__global__ void __launch_bounds__(256) verify_tags_kernel(
    const int32_t* __restrict__ tag_pool, const int32_t* __restrict__ block_tables,
    int max_blocks, const int32_t* __restrict__ context_lens,
    const int64_t* __restrict__ expected_offsets, const int32_t* __restrict__ expected,
    int block_size, int64_t num_blocks, int32_t* __restrict__ mismatch_pos) {
  const int b = blockIdx.x;
  __shared__ int first;
  if (threadIdx.x == 0) first = 0x7fffffff;
  __syncthreads();
  int ctx = context_lens[b];
  if (ctx > max_blocks * block_size) {
    ctx = max_blocks * block_size;
    if (threadIdx.x == 0) atomicMin(&first, ctx);  // table too short for the context
  }
  const int32_t* table = block_tables + int64_t(b) * max_blocks;
  const int32_t* want = expected + expected_offsets[b];
  for (int p = threadIdx.x; p < ctx; p += blockDim.x) {
    const int64_t blk = table[p / block_size];
    const bool ok = blk >= 0 && blk < num_blocks &&
                    tag_pool[blk * block_size + p % block_size] == want[p];
    if (!ok) atomicMin(&first, p);
  }
  __syncthreads();
  if (threadIdx.x == 0) mismatch_pos[b] = first == 0x7fffffff ? -1 : first;
}

}  // namespace

extern "C" int ts_verify_tags(const int32_t* tag_pool, const int32_t* block_tables,
                              int32_t max_blocks_per_seq, const int32_t* context_lens,
                              const int64_t* expected_offsets, const int32_t* expected_tokens,
                              int32_t batch, int32_t block_size, int64_t num_blocks,
                              int32_t* mismatch_pos, void* stream) {
  if (batch < 0 || block_size <= 0 || num_blocks <= 0 || max_blocks_per_seq <= 0)
    return ts::set_error(TS_ERR_INVALID_ARGUMENT, "verify_tags: bad sizes");
  if (batch == 0) return ts::ok();
  if (!tag_pool || !block_tables || !context_lens || !expected_offsets || !expected_tokens ||
      !mismatch_pos)
    return ts::set_error(TS_ERR_INVALID_ARGUMENT, "verify_tags: null pointer");
  verify_tags_kernel<<<batch, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      tag_pool, block_tables, max_blocks_per_seq, context_lens, expected_offsets,
      expected_tokens, block_size, num_blocks, mismatch_pos);
  return ts::launch_status("verify_tags");
}
