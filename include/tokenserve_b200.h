/*
 * tokenserve_b200 — C ABI of the B200 paged-KV execution kernels.
 *
 * These entry points are what a tokenserve `Backend` (src/tokenserve/backends/base.py:48-65)
 * needs to execute one engine step on a paged KV cache. In the reference the same work is
 * done by pure Python: the slot mapping and the shadow-KV write of SimulatedBackend
 * (src/tokenserve/backends/base.py:40-45, src/tokenserve/backends/simulated.py:147-169) and
 * the contiguous per-sequence attention of HFBackend (src/tokenserve/backends/hf.py:57-75,
 * which runs transformers' eager_attention_forward). The reference binds no native code, so
 * each function below names the Python code it replaces; the Python side binds them with
 * ctypes (tokenserve_b200/ops.py).
 *
 * Conventions
 *   - Every pointer argument is a DEVICE pointer unless its comment says otherwise. Tensors
 *     stay owned by the caller; nothing here allocates device memory.
 *   - `stream` is a cudaStream_t passed as void* (NULL = the legacy default stream). All work
 *     is enqueued asynchronously on it; no call synchronises the device.
 *   - Return value: 0 on success; a negative TS_ERR_* code when an argument is invalid
 *     (nothing was launched); a positive cudaError_t when a launch failed. ts_last_error()
 *     returns a message for the last failure on the calling thread.
 *   - KV pool layout per layer: key_pool and value_pool are each
 *     [num_blocks][num_kv_heads][block_size][head_dim] in `dtype`, contiguous. Physical slot
 *     s = block_id * block_size + offset addresses row (s / block_size, h, s % block_size).
 *   - Query head q uses KV head q / (num_q_heads / num_kv_heads) (grouped-query attention,
 *     the head order of transformers' repeat_kv).
 */
#ifndef TOKENSERVE_B200_H
#define TOKENSERVE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TS_ABI_VERSION 1

/* Element types of queries, keys, values and attention outputs. */
enum ts_dtype { TS_FLOAT32 = 0, TS_FLOAT16 = 1, TS_BFLOAT16 = 2 };

/* Negative status codes (argument errors detected on the host before any launch). */
enum ts_status {
  TS_OK = 0,
  TS_ERR_INVALID_ARGUMENT = -1,
  TS_ERR_UNSUPPORTED = -2,
  TS_ERR_WORKSPACE_TOO_SMALL = -3,
  TS_ERR_MISALIGNED = -4,
};

/* ABI version of the loaded library (TS_ABI_VERSION it was built with). */
int ts_version(void);

/* Message for the most recent failing call on this thread ("" if none). Host pointer, valid
 * until the next call on this thread. */
const char* ts_last_error(void);

/*
 * K1 — write the KV of the step's new tokens into the paged pool (reshape_and_cache).
 *
 * Replaces: the slot mapping of BatchItem.slot_mapping (src/tokenserve/backends/base.py:40-45)
 * and the write half of SimulatedBackend._write_and_verify
 * (src/tokenserve/backends/simulated.py:156-160), here carrying real K/V rows instead of
 * token ids.
 *
 * key, value:   [num_tokens][num_kv_heads][head_dim] in dtype; token t's row starts at
 *               key + t * key_token_stride elements (heads contiguous, stride head_dim).
 * slot_mapping: [num_tokens] int64; slot < 0 skips the token (padding).
 * token_tags:   optional int32 [num_tokens] (NULL = off); when set, tag_pool (int32
 *               [num_blocks * block_size]) receives token_tags[t] at slot_mapping[t]. This is
 *               the device shadow of SimulatedBackend's shadow array (simulated.py:101).
 * error_flag:   optional int32 device word (NULL = off). A slot >= num_blocks * block_size is
 *               skipped and sets *error_flag to 1; nothing outside the pool is written.
 */
int ts_reshape_and_cache(const void* key, const void* value, int64_t key_token_stride,
                         int64_t value_token_stride, void* key_pool, void* value_pool,
                         const int64_t* slot_mapping, int64_t num_tokens, int32_t num_kv_heads,
                         int32_t head_dim, int32_t block_size, int64_t num_blocks, int32_t dtype,
                         const int32_t* token_tags, int32_t* tag_pool, int32_t* error_flag,
                         void* stream);

/* Bytes of device workspace ts_paged_decode needs for these sizes (0 is possible). */
size_t ts_paged_decode_workspace_size(int32_t batch, int32_t num_q_heads, int32_t num_kv_heads,
                                      int32_t head_dim, int32_t max_blocks_per_seq,
                                      int32_t block_size, int32_t dtype);

/*
 * K2 — paged decode attention: one query token per sequence attends to its whole context.
 *
 * Replaces: transformers 5.5.0 eager_attention_forward (models/llama/modeling_llama.py:199,
 * with repeat_kv :187) as called by HFBackend._execute (src/tokenserve/backends/hf.py:71)
 * for a decode step, over a contiguous per-sequence cache.
 *
 * out:          [batch][num_q_heads][head_dim] in dtype, contiguous.
 * query:        [batch][num_q_heads][head_dim]; sequence b's row starts at
 *               query + b * query_token_stride elements.
 * block_tables: int32 [batch][max_blocks_per_seq] (row-major); entries past the context are
 *               ignored.
 * context_lens: int32 [batch]; tokens 0..context_lens[b]-1 (the new token included) are
 *               attended. 0 writes zeros.
 * scale:        softmax scale (head_dim ** -0.5 for Llama).
 * workspace:    device scratch of at least ts_paged_decode_workspace_size(...) bytes, 256-byte
 *               aligned, with no initial contents required (every call resets the counters it
 *               uses). Calls that overlap on the GPU must not share a workspace.
 */
int ts_paged_decode(void* out, const void* query, int64_t query_token_stride,
                    const void* key_pool, const void* value_pool, const int32_t* block_tables,
                    int32_t max_blocks_per_seq, const int32_t* context_lens, int32_t batch,
                    int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                    int32_t block_size, int64_t num_blocks, float scale, int32_t dtype,
                    void* workspace, size_t workspace_bytes, void* stream);

/*
 * K2 that reuses the work plan an earlier ts_paged_decode left in `workspace` (a model's later
 * layers in one decode step: every layer has the same block tables and context lengths).
 *
 * Replaces: the same eager attention as ts_paged_decode (one call per layer in
 * src/tokenserve/backends/hf.py:71); the plan reuse itself has no counterpart in the reference.
 * ts_paged_decode runs a one-CTA prep kernel (partition descriptors, claim order, prefix sums)
 * before the decode kernel; this call launches the decode kernel alone. Arguments as
 * ts_paged_decode. Preconditions: the earlier call, ordered before this one on the GPU, used
 * the same workspace, block_tables contents, context_lens contents, batch, num_kv_heads and
 * max_blocks_per_seq, and took the tensor-core path (same dtype, head_dim, block_size and
 * pointer alignment as here). A plan made for another batch, head count, table width or grid
 * is detected on the device: nothing is written and the workspace's status word (int32 at
 * byte 4) is set to 4. Changed table or length contents are not detected.
 */
int ts_paged_decode_planned(void* out, const void* query, int64_t query_token_stride,
                            const void* key_pool, const void* value_pool,
                            const int32_t* block_tables, int32_t max_blocks_per_seq,
                            const int32_t* context_lens, int32_t batch, int32_t num_q_heads,
                            int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                            int64_t num_blocks, float scale, int32_t dtype, void* workspace,
                            size_t workspace_bytes, void* stream);

/* Size of the device scratch built into the library for ts_paged_decode_no_alloc (32 MiB). */
#define TS_NO_ALLOC_SCRATCH_BYTES (32u << 20)

/*
 * K2 without a workspace argument. No counterpart in the reference: tokenserve has no native
 * code at all; this entry point exists only for callers of this library that cannot allocate.
 *
 * Some callers cannot hand ts_paged_decode a workspace: a C or FFI caller embedded in a
 * process whose device memory is owned by another allocator (a framework's caching allocator
 * that has reserved the HBM, so a cudaMalloc next to it fails or fragments it), or a caller on
 * a latency-critical path that must not call cudaMalloc/cudaFree, which can synchronise the
 * device. This variant takes the same arguments minus the workspace and allocates nothing:
 * its scratch is a TS_NO_ALLOC_SCRATCH_BYTES array inside the library's device image, which
 * every GPU that loads the library holds until the process exits.
 *
 *   - Sizes whose scratch (ts_paged_decode_workspace_size) exceeds TS_NO_ALLOC_SCRATCH_BYTES
 *     are rejected with TS_ERR_WORKSPACE_TOO_SMALL before anything is launched.
 *   - The first call on each device looks up the scratch's device address with that device
 *     current and keeps it for the life of the process; make that first call before any
 *     stream capture. A cudaDeviceReset invalidates that address (and the kernel attributes
 *     the library sets once per device): calls after a reset of the device are unsupported.
 *   - All calls on a device share the one scratch array and each call clears the parts that
 *     must start at zero. Calls whose kernels overlap on the GPU (different streams without
 *     ordering between them) race on it and give wrong results: order them.
 */
int ts_paged_decode_no_alloc(void* out, const void* query, int64_t query_token_stride,
                             const void* key_pool, const void* value_pool,
                             const int32_t* block_tables, int32_t max_blocks_per_seq,
                             const int32_t* context_lens, int32_t batch, int32_t num_q_heads,
                             int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                             int64_t num_blocks, float scale, int32_t dtype, void* stream);

/*
 * K3 — paged chunked-prefill attention (causal): each sequence's new chunk of queries
 * attends to its cached prefix blocks plus the chunk itself, all read through the block
 * table (the chunk's K/V must already be in the pool, written by ts_reshape_and_cache).
 *
 * Replaces: the same eager_attention_forward path for a multi-token step with a causal mask
 * (HFBackend recomputes from position 0 when it holds no cache, hf.py:62-65; here the
 * cached prefix is reused).
 *
 * out, query:      [num_query_tokens][num_q_heads][head_dim]; query token i of the batch
 *                  starts at query + i * query_token_stride elements; out is contiguous.
 * query_start_loc: int32 [num_seqs + 1]; sequence s owns query rows
 *                  query_start_loc[s] .. query_start_loc[s+1]-1.
 * context_lens:    int32 [num_seqs]; total tokens of sequence s after this step. Query row j
 *                  of sequence s sits at position context_lens[s] - q_len + j and attends to
 *                  positions 0..that position.
 * max_query_len:   an upper bound of the per-sequence query lengths.
 */
int ts_paged_prefill(void* out, const void* query, int64_t query_token_stride,
                     const void* key_pool, const void* value_pool, const int32_t* block_tables,
                     int32_t max_blocks_per_seq, const int32_t* query_start_loc,
                     const int32_t* context_lens, int32_t num_seqs, int32_t num_query_tokens,
                     int32_t max_query_len, int32_t num_q_heads, int32_t num_kv_heads,
                     int32_t head_dim, int32_t block_size, int64_t num_blocks, float scale,
                     int32_t dtype, void* stream);

/*
 * K4 — batched block copy (preemption swap-in / copy-on-write).
 *
 * Replaces: nothing in the reference, which preempts by recompute
 * (src/tokenserve/scheduler.py:215-225) and shares only full blocks
 * (src/tokenserve/kv_cache.py:179-199); it is validated against an index copy.
 *
 * pool_base:          start of num_planes equally sized planes (e.g. [layers][2] pools).
 * plane_stride_bytes: distance between planes; block b of plane p starts at
 *                     pool_base + p * plane_stride_bytes + b * block_bytes.
 * src_dst:            int64 [num_pairs][2] of (source block, destination block). Sources
 *                     and destinations must be disjoint sets.
 * num_blocks:         blocks per plane (for bounds checking); an out-of-range pair is
 *                     skipped and sets *error_flag (optional, may be NULL).
 */
int ts_copy_blocks(void* pool_base, int64_t num_planes, int64_t plane_stride_bytes,
                   int64_t block_bytes, int64_t num_blocks, const int64_t* src_dst,
                   int64_t num_pairs, int32_t* error_flag, void* stream);

/*
 * K4 swap form — the same block copy between two arenas of one plane layout, for swap-to-host
 * preemption: swap-out copies pool blocks into a pinned host arena, swap-in copies them back
 * (into any free blocks). The kernel reads or writes the host side directly through its
 * device-mapped address.
 *
 * Replaces: nothing in the reference (recompute-only preemption, src/tokenserve/scheduler.py:
 * 215-225; swap-to-host is listed as future work in its README, "What a GPU run would add").
 *
 * dst_base / src_base: arenas of num_planes planes; block b of plane p of an arena starts at
 *                      base + p * plane_stride_bytes + b * block_bytes. Each must be memory of
 *                      the current device or pinned (page-locked) host memory; anything else
 *                      (pageable host memory, another device's memory) returns
 *                      TS_ERR_INVALID_ARGUMENT before any launch. src_dst and error_flag too.
 * src_dst:             int64 [num_pairs][2] of (block in src arena, block in dst arena); a
 *                      pair out of either arena's range is skipped and sets *error_flag.
 */
int ts_swap_blocks(void* dst_base, int64_t dst_plane_stride_bytes, int64_t dst_num_blocks,
                   const void* src_base, int64_t src_plane_stride_bytes, int64_t src_num_blocks,
                   int64_t num_planes, int64_t block_bytes, const int64_t* src_dst,
                   int64_t num_pairs, int32_t* error_flag, void* stream);

/*
 * Shadow-KV verification of the token tags written by ts_reshape_and_cache: for each
 * sequence, every position 0..context_lens[b]-1 read back through its block table must hold
 * expected_tokens (concatenated per sequence at expected_offsets[b]). The first mismatch per
 * sequence is reported in mismatch_pos[b] (-1 = none; host reads it after the stream syncs).
 *
 * Replaces: the read half of SimulatedBackend._write_and_verify
 * (src/tokenserve/backends/simulated.py:161-169).
 */
int ts_verify_tags(const int32_t* tag_pool, const int32_t* block_tables,
                   int32_t max_blocks_per_seq, const int32_t* context_lens,
                   const int64_t* expected_offsets, const int32_t* expected_tokens,
                   int32_t batch, int32_t block_size, int64_t num_blocks,
                   int32_t* mismatch_pos, void* stream);

/*
 * K2 of one rank of a KV-head-sharded model, fused with the all-gather of its output.
 *
 * Replaces: the per-layer all-gather of attention outputs in the sharded configuration (the
 * reference runs a single process; the sharded layout is this backend's: rank r of `world`
 * holds KV heads [r*Hkv/world, (r+1)*Hkv/world) and their query heads, under replicated block
 * tables). Arguments as ts_paged_decode for this rank's heads (num_q_heads / num_kv_heads are the
 * rank's counts), except the output: each of dst_outs[0..world) is a rank's full output
 * [batch][world * num_q_heads][head_dim], and this rank's rows land at head offset
 * rank * num_q_heads in every one of them (stores over NVLink for the peers). The grid's last
 * CTA then writes `epoch` (non-zero, increasing per call) into signals[r][rank] for every r;
 * with batch 0 nothing is decoded and one small kernel publishes the epoch the same way, so the
 * other ranks' waits still end. dst_outs and signals are device arrays of device pointers (peer buffers mapped with
 * ts_ipc_open); the tensor-core decode path is required (TS_ERR_UNSUPPORTED otherwise).
 * reuse_plan = 1 skips the prep kernel and runs the plan an earlier call left in `workspace`,
 * under the preconditions of ts_paged_decode_planned.
 */
int ts_paged_decode_peer(void* const* dst_outs, int32_t world, int32_t rank,
                         int32_t* const* signals, uint32_t epoch, const void* query,
                         int64_t query_token_stride, const void* key_pool, const void* value_pool,
                         const int32_t* block_tables, int32_t max_blocks_per_seq,
                         const int32_t* context_lens, int32_t batch, int32_t num_q_heads,
                         int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                         int64_t num_blocks, float scale, int32_t dtype, void* workspace,
                         size_t workspace_bytes, int32_t reuse_plan, void* stream);

/*
 * The pull form of the same exchange: this rank's rows go into its own buffer only
 * (dst_outs[rank], at head offset rank * num_q_heads, fast local stores), and the grid's last
 * CTA publishes `epoch` into signals[r][rank] for every r as above; each rank then fetches the
 * others' rows with ts_gather_peers. Arguments as ts_paged_decode_peer.
 *
 * Replaces: the same eager attention per KV-head shard; the exchange has no counterpart in the
 * reference, which runs on one CPU process.
 */
int ts_paged_decode_publish(void* const* dst_outs, int32_t world, int32_t rank,
                            int32_t* const* signals, uint32_t epoch, const void* query,
                            int64_t query_token_stride, const void* key_pool,
                            const void* value_pool, const int32_t* block_tables,
                            int32_t max_blocks_per_seq, const int32_t* context_lens,
                            int32_t batch, int32_t num_q_heads, int32_t num_kv_heads,
                            int32_t head_dim, int32_t block_size, int64_t num_blocks,
                            float scale, int32_t dtype, void* workspace, size_t workspace_bytes,
                            int32_t reuse_plan, void* stream);

/*
 * Completes a pull exchange on this rank: waits on the device (bounded, about a second) until
 * local_signals[r] >= epoch for every r < world, then copies every other rank's
 * [batch][heads_per_rank][head_dim] slice from that rank's buffer fulls[r] (read over NVLink)
 * into the same rows and head offset of fulls[rank]. fulls is a device array of world pointers
 * (each rank's [batch][world * heads_per_rank][head_dim] buffer as mapped here). On a timeout
 * nothing is copied by the CTAs that gave up and *status (device int32) is set to 3.
 * heads_per_rank * head_dim * element size must be a multiple of 16 bytes.
 */
int ts_gather_peers(void* const* fulls, int32_t world, int32_t rank,
                    const int32_t* local_signals, uint32_t epoch, int32_t batch,
                    int32_t heads_per_rank, int32_t head_dim, int32_t dtype, int32_t* status,
                    void* stream);

/*
 * Waits on the device until local_signals[r] >= epoch for every r < world (every rank's
 * ts_paged_decode_peer of that epoch has finished writing into this rank's buffer). The wait
 * is bounded (about a second); on timeout *status (device int32) is set to 3 and the kernel
 * returns, leaving the context usable.
 */
int ts_wait_peers(const int32_t* local_signals, int32_t world, uint32_t epoch, int32_t* status,
                  void* stream);

/* Device buffers shared between the ranks' processes, and their CUDA IPC handles (64 bytes). */
int ts_peer_alloc(size_t bytes, void** ptr);
int ts_peer_free(void* ptr);
int ts_ipc_get_handle(const void* ptr, void* handle);
int ts_ipc_open(const void* handle, void** ptr);
int ts_ipc_close(void* ptr);

/*
 * Fused element-wise parts of a Llama decoder layer used by the paged model runner. They
 * replace transformers 5.5.0 modules (models/llama/modeling_llama.py) that tokenserve's
 * HFBackend runs per sequence (src/tokenserve/backends/hf.py:71), with the same rounding points.
 *
 * ts_add_rmsnorm: residual[r] += x[r] in dtype (x may be NULL: no add), then
 *   out[r] = weight * dtype(residual[r] * rsqrt(mean(residual[r]^2) + eps))   (LlamaRMSNorm :53-70)
 *   out, residual, x: [num_rows][hidden]; weight: [hidden]; all of `dtype`.
 */
int ts_add_rmsnorm(void* out, void* residual, const void* x, const void* weight,
                   int64_t num_rows, int32_t hidden, float eps, int32_t dtype, void* stream);

/*
 * ts_rope_and_cache: for each token t of a fused projection qkv[t] = [q heads | k heads | v heads]
 * (head_dim each, rows qkv_token_stride elements apart): rotary embedding of q and k at
 * positions[t] (apply_rotary_pos_emb :146-168, cos/sin of positions[t] * inv_freq[i] in fp32
 * rounded to dtype), rotated q to q_out [num_tokens][num_q_heads][head_dim], rotated k and v
 * written to the pool slot slot_mapping[t] exactly like ts_reshape_and_cache (slot < 0 skipped,
 * slot past the pool skipped and flagged). inv_freq: fp32 [head_dim / 2].
 */
int ts_rope_and_cache(const void* qkv, int64_t qkv_token_stride, void* q_out, void* key_pool,
                      void* value_pool, const int64_t* slot_mapping, const int64_t* positions,
                      const float* inv_freq, int64_t num_tokens, int32_t num_q_heads,
                      int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                      int64_t num_blocks, int32_t dtype, int32_t* error_flag, void* stream);

/*
 * ts_silu_mul: out[r][c] = dtype(dtype(silu(gate_up[r][c])) * gate_up[r][intermediate + c])
 * (LlamaMLP act_fn(gate) * up, :184); gate_up: [num_rows][2 * intermediate].
 */
int ts_silu_mul(void* out, const void* gate_up, int64_t num_rows, int32_t intermediate,
                int32_t dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TOKENSERVE_B200_H */
