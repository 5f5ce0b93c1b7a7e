// K2 — paged decode attention (bf16 / fp16 KV, block_size 16, head_dim 64 or 128).
//
// Semantics: transformers 5.5.0 eager_attention_forward (models/llama/modeling_llama.py:199)
// with repeat_kv (:187) for one query token per sequence over its whole context, which is what
// tokenserve's HFBackend runs for a decode step (src/tokenserve/backends/hf.py:71), except that
// the context is read through the block table of KVCacheManager (src/tokenserve/kv_cache.py:141)
// instead of a private contiguous cache.
//
// Design (HBM-bound: every K/V byte is read exactly once):
//   * Work item = partition of one (sequence b, KV head h): up to 64 consecutive blocks. All
//     G = Hq/Hkv query heads of h are packed into the N dimension of the tensor-core tiles, so a
//     KV byte serves every query head that uses it (GQA packing).
//   * A one-CTA prep kernel plans the step into the workspace: small steps get a static even
//     split of the (sequence, head, block) units over the grid's warps, cut into partitions at
//     sequence ends and every 64 blocks; large steps get partitions of 64 / 32 / 16 blocks
//     claimed from a counter in a sorted order. The plan depends only on the block tables and
//     context lengths, so a model's later layers in the same step reuse it
//     (ts_paged_decode_planned) and launch the decode kernel alone.
//   * Every warp is an independent pipeline over its partitions: it fetches its next item a few
//     blocks before the current one ends, and lane 0 streams the blocks with 2-D TMA loads
//     (128-byte swizzle, no multicast) into a private ring of kStages stages, each holding one
//     block's K and V tile for head h.
//   * S^T = K Q^T and O^T += V^T P^T on mma.sync m16n8k16 (fp32 accumulate). P is split into a
//     hi and a lo half-precision part so the PV product keeps ~16 mantissa bits.
//   * Online softmax in fp32 (exp2 domain) per block; partitions of one (b, h) are merged by the
//     last warp to finish one (log-sum-exp merge in fixed partition order), tracked with an
//     arrival counter.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace {

// Tuning knobs (compile-time).
#ifndef TS_DECODE_WARPS
#define TS_DECODE_WARPS 8  // independent warp pipelines per CTA (one CTA per SM)
#endif
#ifndef TS_DECODE_PART_BLOCKS
#define TS_DECODE_PART_BLOCKS 64  // largest work item, in blocks
#endif
#ifndef TS_DECODE_STATIC_MAX_BLOCKS
#define TS_DECODE_STATIC_MAX_BLOCKS 64  // static split while a group's range is at most this
#endif
#ifndef TS_DECODE_STAGES_D128
#define TS_DECODE_STAGES_D128 3  // ring stages per warp at head_dim 128
#endif
#ifndef TS_DECODE_MIN_ITEMS_PER_WARP
#define TS_DECODE_MIN_ITEMS_PER_WARP 2  // dynamic claiming: the item size gives every warp this many
#endif
#ifndef TS_DECODE_PREFETCH_BLOCKS
#define TS_DECODE_PREFETCH_BLOCKS 4  // the next item is fetched this many blocks before the end
#endif
#ifndef TS_DECODE_HEAVY_PARTS
#define TS_DECODE_HEAVY_PARTS 4  // dynamic claiming: sequences with this many partitions go first (0: none)
#endif
#ifndef TS_DECODE_ONE_BOX
#define TS_DECODE_ONE_BOX 0  // 1: one 4 KiB TMA box per 128-dim tile instead of two 2 KiB
#endif

constexpr int kWarps = TS_DECODE_WARPS;
constexpr int kBlock = 16;                          // tokens per KV block
// Work is split statically and evenly. The grid's warps form NG = min(G / H, WB) groups of H
// (one warp per KV head); group g takes blocks [floor(g WB / NG), floor((g + 1) WB / NG)) of
// the step's WB blocks (all sequences' blocks in order) and warp (g, h) attends head h over
// them, cut into partitions of at most kPartBlocks blocks wherever a sequence or the range
// ends. Every warp streams the same number of blocks (+-1) whatever the batch, so small
// batches keep all warps busy to the end, and the H warps of a group (neighbours in one CTA)
// read the H heads of the same blocks, which sit next to each other in the pool.
//
// Large steps instead use dynamic claiming (the split above would cut more sequences and leave
// the partition merges unevenly spread): partitions of pb blocks (64 / 32 / 16, the largest that
// gives every warp two), claimed from a counter in the order prep_dynamic describes. The prep
// kernel picks the static split below kStaticMaxBlocksPerWarp blocks per warp on average.
constexpr int kPartBlocks = TS_DECODE_PART_BLOCKS;
constexpr int kMinPartBlocks = 16;
constexpr int kStaticMaxBlocksPerWarp = TS_DECODE_STATIC_MAX_BLOCKS;
constexpr int kMinItemsPerWarp = TS_DECODE_MIN_ITEMS_PER_WARP;
constexpr int kHeavyParts = TS_DECODE_HEAVY_PARTS;
static_assert(kPartBlocks >= 2 && kPartBlocks <= 64, "a work item's table fits two registers per lane");
// Upper bound of the grid's warps (SMs x warps per CTA), used to size the workspace.
constexpr int kMaxGridWarps = 8192;
constexpr float kLog2e = 1.4426950408889634f;

struct DecodeArgs {
  // Output rows: sequence b, query head j (of this call's num_q_heads) goes to
  // dst + b * out_row_stride + (out_head0 + j) * head_dim for dst = out, or, with n_out > 0,
  // for every dst in outs[0..n_out) (the ranks' full buffers of a KV-head-sharded model).
  void* out;
  void* const* outs;  // device array of n_out pointers, or nullptr
  int n_out;
  int64_t out_row_stride;  // elements
  int out_head0;
  // Completion signal (n_signals > 0): the grid's last CTA stores `epoch` into
  // signals[r][signal_index] for every r < n_signals, after every CTA's output stores.
  int n_signals;
  int* const* signals;
  int remote_out;  // 1: output rows were stored into other GPUs' memory (push exchange)
  int signal_index;
  unsigned epoch;
  const void* query;
  int64_t q_stride;
  const int32_t* block_tables;
  const int32_t* context_lens;
  int max_blocks;
  int batch;
  int num_q_heads;
  int num_kv_heads;
  int group;  // query heads per KV head
  int64_t num_blocks;
  float scale_log2;
  // [0] claim counter, [1] status, [2] 1 = dynamic claiming, [3] items to claim (dynamic) or
  // groups (static), [4] CTAs finished, [6..9] the plan's batch, KV heads, table width and grid
  // warps. The main kernel's last CTA re-zeroes [0] and [4], so a later launch can run the
  // same plan (block tables and context lengths unchanged) without the prep kernel.
  int* header;
  int reuse_plan;  // 1: the workspace holds the prep kernel's plan from an earlier launch
  int grid_warps;  // warps of the main kernel's grid
  // [batch + 1] partitions of one head before sequence b; sequence b's partition k of head h
  // writes partial slot chunk_prefix[b] * H + h * parts_b + k, so a (sequence, head)'s partials
  // are consecutive for the merge
  int* chunk_prefix;
  // [partition] = {(sequence, first block, blocks, index k in its sequence),
  //                (chunk_prefix[sequence], partitions of the sequence, context length, 0)}
  int4* part_info;
  int* group_first;  // [groups + 1] first partition of each group (static split)
  int* arrive;  // [batch * num_kv_heads]
  float* part_o;   // [partition][head_dim][NT * 8]
  float2* part_ml;  // [partition][NT * 8]
};

// Workspace layout (byte offsets), shared by the size query and the launcher.
struct WsLayout {
  size_t chunk_prefix, part_info, group_first, arrive, part_o, part_ml, total;
};

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

int num_sms();

// grid_warps: warps of the decode grid on the device the call runs on (its SMs x kWarps).
WsLayout ws_layout(int batch, int hkv, int hd, int max_blocks, int nt, int grid_warps) {
  WsLayout w;
  // A sequence is cut at most once per kPartBlocks blocks and once per group boundary; each cut
  // gives one partition per head (groups x heads <= grid warps).
  const size_t bh = size_t(batch) * size_t(hkv);
  const size_t slots = std::max(
      bh * size_t((max_blocks + kPartBlocks - 1) / kPartBlocks + 1) + size_t(grid_warps),
      bh * size_t((max_blocks + kMinPartBlocks - 1) / kMinPartBlocks));
  w.chunk_prefix = 256;
  w.part_info = w.chunk_prefix + align256(sizeof(int) * (size_t(batch) + 1));
  w.group_first = w.part_info + align256(2 * sizeof(int4) * slots);
  w.arrive = w.group_first + align256(sizeof(int) * (size_t(grid_warps) + 1));
  w.part_o = w.arrive + align256(sizeof(int) * bh);
  w.part_ml = w.part_o + align256(sizeof(float) * slots * hd * nt * 8);
  w.total = w.part_ml + align256(sizeof(float2) * slots * nt * 8);
  return w;
}

// --------------------------------------------------------------------------- prep kernel

// Block-wide exclusive scan (1 CTA); returns the exclusive prefix and sets *total.
__device__ __forceinline__ int block_exclusive_scan(int v, int* total, int* warp_sums) {
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int x = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += x;
  }
  __syncthreads();
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = lane < (int)(blockDim.x / 32) ? warp_sums[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int x = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += x;
    }
    warp_sums[lane] = w;  // inclusive over warps
  }
  __syncthreads();
  *total = warp_sums[blockDim.x / 32 - 1];
  return incl - v + (warp > 0 ? warp_sums[warp - 1] : 0);
}


__device__ __forceinline__ int blocks_of(int ctx) { return (ctx + kBlock - 1) / kBlock; }

// The step's WB blocks in NG groups (0 < NG <= WB < 2^31): the first WB % NG groups hold
// WB / NG + 1 blocks, the others WB / NG. 32-bit arithmetic only.
struct GroupSplit {
  int q, r;  // WB / NG, WB % NG
  __device__ __forceinline__ GroupSplit(int WB, int NG) : q(WB / NG), r(WB % NG) {}
  __device__ __forceinline__ int start(int g) const { return g * q + min(g, r); }
  __device__ __forceinline__ int group_of(int u) const {
    const int big = r * (q + 1);
    return u < big ? u / (q + 1) : r + (u - big) / q;
  }
};

// Calls f(group, group start, first block, end block) for every partition of blocks [u0, u1):
// its pieces inside one group's range, each cut into kPartBlocks-block partitions, in order.
template <typename F>
__device__ __forceinline__ void for_each_chunk(int u0, int u1, const GroupSplit& gsp, F&& f) {
  const int g0 = gsp.group_of(u0), g1 = gsp.group_of(u1 - 1);
  int gs = gsp.start(g0);
  for (int g = g0; g <= g1; ++g) {
    const int gn = gsp.start(g + 1);
    const int lo = max(u0, gs), hi = min(u1, gn);
    for (int c = lo; c < hi; c += kPartBlocks) f(g, gs, c, min(hi, c + kPartBlocks));
    gs = gn;
  }
}

constexpr int kPrepThreads = 1024;

// Sequence b's context length, clamped to its block table.
__device__ __forceinline__ int ctx_of(const DecodeArgs& a, int b) {
  const int ctx = __ldg(a.context_lens + b), cap = a.max_blocks * kBlock;
  return ctx < 0 ? 0 : (ctx > cap ? cap : ctx);
}

// Static split (small steps): groups of H warps, see kPartBlocks. run0: blocks before this
// thread's first sequence b0; nblk: its cnt sequences' blocks.
__device__ void prep_static(DecodeArgs& a, int* warp_sums, long long WB, int run0, int cnt,
                            int b0) {
  const int B = a.batch;
  const int NG = int(min((long long)(a.grid_warps / a.num_kv_heads), WB));
  const GroupSplit gsp(int(WB), NG > 0 ? NG : 1);
  // A group spans at most kPartBlocks blocks (the prep kernel's choice of split), so each
  // group a sequence overlaps holds exactly one of its partitions: the count is the number of
  // groups its blocks [u, u + n) touch.
  int c = 0;
  int u = run0;
  for (int i = 0; i < cnt; ++i) {
    const int n = blocks_of(ctx_of(a, b0 + i));
    if (n > 0) c += gsp.group_of(u + n - 1) - gsp.group_of(u) + 1;
    u += n;
  }
  int total = 0;
  int runc = block_exclusive_scan(c, &total, warp_sums);
  if (B <= int(blockDim.x)) {
    // One sequence per thread (b0 = thread, cnt <= 1). The partitions are written in parallel,
    // thread t taking partitions t, t + T, ...: a long sequence's tens of partitions would
    // otherwise be one thread's serial loop, the prep's critical path. Partition p belongs to
    // the last sequence b with s_runc[b] <= p (binary search; empty sequences share the next
    // one's prefix) and is its k-th, k = p - s_runc[b], covering group group_of(u_b) + k.
    __shared__ int s_runc[kPrepThreads + 1], s_u[kPrepThreads], s_ctx[kPrepThreads];
    if (cnt > 0) {
      s_runc[b0] = runc;
      s_u[b0] = run0;
      s_ctx[b0] = ctx_of(a, b0);
      a.chunk_prefix[b0] = runc;
    }
    if (threadIdx.x == 0) s_runc[B] = total;
    __syncthreads();
    for (int p = threadIdx.x; p < total; p += blockDim.x) {
      int lo = 0, hi = B;  // s_runc[lo] <= p < s_runc[hi]
      while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (s_runc[mid] <= p) lo = mid; else hi = mid;
      }
      const int b = lo, k = p - s_runc[b], ub = s_u[b], ctx = s_ctx[b];
      const int g = gsp.group_of(ub) + k, gs = gsp.start(g);
      const int blk_lo = max(ub, gs), blk_hi = min(ub + blocks_of(ctx), gsp.start(g + 1));
      a.part_info[2 * p] = make_int4(b, blk_lo - ub, blk_hi - blk_lo, k);
      a.part_info[2 * p + 1] = make_int4(s_runc[b], s_runc[b + 1] - s_runc[b], ctx, 0);
      if (blk_lo == gs) a.group_first[g] = p;  // the partition that opens group g
    }
  } else {
    u = run0;
    for (int i = 0; i < cnt; ++i) {
      const int b = b0 + i;
      a.chunk_prefix[b] = runc;
      const int ctx = ctx_of(a, b), n = blocks_of(ctx);
      int k = 0;
      if (n > 0)
        for_each_chunk(u, u + n, gsp, [&](int g, int gs, int lo, int hi) {
          a.part_info[2 * (runc + k)] = make_int4(b, lo - u, hi - lo, k);
          if (lo == gs) a.group_first[g] = runc + k;  // the partition that opens group g
          ++k;
        });
      for (int m = 0; m < k; ++m) a.part_info[2 * (runc + m) + 1] = make_int4(runc, k, ctx, 0);
      runc += k;
      u += n;
    }
  }
  if (threadIdx.x == 0) {
    a.chunk_prefix[B] = total;
    a.group_first[NG] = total;
    a.header[2] = 0;
    a.header[3] = NG;
  }
}

// Dynamic claiming (large steps): partitions of pb blocks of every (sequence, head), pb the
// largest of 64 / 32 / 16 that gives every warp kMinItemsPerWarp. Claim order, by counting sort:
//   1. every partition of the sequences with at least kHeavyParts partitions, sequence by
//      sequence, most partitions first — their merges (the last warp to finish one of them reads
//      all its partials) then run while the other warps still stream, not in the kernel's tail;
//   2. the full partitions of the other sequences;
//   3. the remaining partial partitions, longest first, so the tail is made of the shortest items.
// The order only decides which warp runs a partition; every partition's partial result and
// every merge (fixed partition order) are the same whatever the order, so outputs are too.
constexpr int kPartsCap = 512;  // sequences with more partitions share the first bucket
constexpr int kClassFull = kPartsCap + 1;
constexpr int kSortBuckets = kClassFull + 1 + kPartBlocks;

__device__ void prep_dynamic(DecodeArgs& a, int* warp_sums, int cnt, int b0) {
  __shared__ int bucket[kSortBuckets];  // counts, then cursors
  const int B = a.batch, H = a.num_kv_heads;
  for (int i = threadIdx.x; i < kSortBuckets; i += blockDim.x) bucket[i] = 0;
  // pb: the largest candidate with kMinItemsPerWarp items per warp; its partition scan is kept.
  int pb = kMinPartBlocks, run_p = 0, total_parts = 0;
  for (int cand = kPartBlocks; cand >= kMinPartBlocks; cand /= 2) {
    int n = 0;
    for (int i = 0; i < cnt; ++i) n += (blocks_of(ctx_of(a, b0 + i)) + cand - 1) / cand;
    int total = 0;
    const int run = block_exclusive_scan(n, &total, warp_sums);
    if (cand == kMinPartBlocks || int64_t(total) * H >= kMinItemsPerWarp * int64_t(a.grid_warps)) {
      pb = cand;
      run_p = run;
      total_parts = total;
      break;
    }
  }
  // Bucket of a sequence of n blocks (np partitions): heavy ones by partition count, descending;
  // the full partitions of the others in one bucket; their partial partitions by size, descending.
  auto heavy = [&](int np) { return kHeavyParts > 0 && np >= kHeavyParts; };
  auto heavy_bucket = [&](int np) { return kPartsCap - min(np, kPartsCap); };
  auto partial_bucket = [&](int n) { return kClassFull + 1 + (pb - n % pb); };
  for (int i = 0; i < cnt; ++i) {
    const int n = blocks_of(ctx_of(a, b0 + i)), np = (n + pb - 1) / pb;
    if (heavy(np)) {
      atomicAdd(&bucket[heavy_bucket(np)], np);
    } else {
      if (n / pb) atomicAdd(&bucket[kClassFull], n / pb);
      if (n % pb) atomicAdd(&bucket[partial_bucket(n)], 1);
    }
  }
  __syncthreads();
  // Counts -> cursors (exclusive prefix in bucket order); thread i owns a contiguous run of
  // buckets, so any block size covers them.
  int sorted = 0;
  const int per_b = (kSortBuckets + blockDim.x - 1) / blockDim.x;
  const int bk0 = min(kSortBuckets, int(threadIdx.x) * per_b);
  const int bk1 = min(kSortBuckets, bk0 + per_b);
  int run_sum = 0;
  for (int k = bk0; k < bk1; ++k) run_sum += bucket[k];
  int first = block_exclusive_scan(run_sum, &sorted, warp_sums);  // every count was read above
  for (int k = bk0; k < bk1; ++k) {
    const int c = bucket[k];
    bucket[k] = first;
    first += c;
  }
  __syncthreads();
  // Partition p of sequence b -> claim position q (items q * H + h, one per head).
  auto put = [&](int q, int b, int p, int n, int c0, int ctx) {
    a.part_info[2 * q] = make_int4(b, p * pb, min(pb, n - p * pb), p);
    a.part_info[2 * q + 1] = make_int4(c0, (n + pb - 1) / pb, ctx, 0);
  };
  for (int i = 0; i < cnt; ++i) {
    const int b = b0 + i, ctx = ctx_of(a, b), n = blocks_of(ctx), np = (n + pb - 1) / pb;
    a.chunk_prefix[b] = run_p;
    if (heavy(np)) {
      const int q = atomicAdd(&bucket[heavy_bucket(np)], np);
      for (int p = 0; p < np; ++p) put(q + p, b, p, n, run_p, ctx);
    } else {
      if (n / pb) {
        const int q = atomicAdd(&bucket[kClassFull], n / pb);
        for (int p = 0; p < n / pb; ++p) put(q + p, b, p, n, run_p, ctx);
      }
      if (n % pb) put(atomicAdd(&bucket[partial_bucket(n)], 1), b, n / pb, n, run_p, ctx);
    }
    run_p += np;
  }
  if (threadIdx.x == 0) {
    a.chunk_prefix[B] = total_parts;
    a.header[2] = 1;
    a.header[3] = total_parts * H;
  }
}

// One CTA (up to kPrepThreads threads, as many as the batch needs): chooses the split (static below kStaticMaxBlocksPerWarp blocks per
// warp, dynamic above), writes the partition descriptors and the per-sequence partition
// prefixes that place each (sequence, head)'s partial results, zeroes the claim counter, status
// word and arrival counters, and writes the output rows of empty contexts.
template <typename T>
__global__ void __launch_bounds__(kPrepThreads) decode_prep_kernel(DecodeArgs a, int row_elems) {
  // The decode grid may launch now (it waits for this grid before reading anything); this grid
  // itself waits for the work before it on the stream (e.g. the K/V append) to be complete.
  ts::allow_dependents();
  ts::wait_prior_grid();
  __shared__ int warp_sums[32];
  const int B = a.batch, H = a.num_kv_heads;
  const int per = (B + blockDim.x - 1) / blockDim.x;
  const int b0 = threadIdx.x * per;
  const int cnt = max(0, min(per, B - b0));
  int sum = 0;
  for (int i = 0; i < cnt; ++i) sum += blocks_of(ctx_of(a, b0 + i));
  // The step's total blocks (one reduction) decide the split; only the static split needs each
  // thread's exclusive prefix.
  __shared__ int total_smem;
  if (threadIdx.x == 0) {
    total_smem = 0;
    a.header[0] = 0;
    a.header[1] = 0;
    a.header[4] = 0;
    a.header[6] = a.batch;
    a.header[7] = a.num_kv_heads;
    a.header[8] = a.max_blocks;
    a.header[9] = a.grid_warps;
  }
  __syncthreads();
  const int wsum = __reduce_add_sync(0xffffffffu, unsigned(sum));
  if (threadIdx.x % 32 == 0 && wsum) atomicAdd(&total_smem, wsum);
  __syncthreads();
  const long long WB = total_smem;
  // Static split while every group of the split spans at most min(kStaticMaxBlocksPerWarp,
  // kPartBlocks) blocks (ceil(WB / NG)); dynamic claiming above.
  const long long NG = min((long long)(a.grid_warps / H), WB);
  if (NG <= 0 || (WB + NG - 1) / NG > (long long)min(kStaticMaxBlocksPerWarp, kPartBlocks)) {
    prep_dynamic(a, warp_sums, cnt, b0);
  } else {
    int total_blocks = 0;
    const int run0 = block_exclusive_scan(sum, &total_blocks, warp_sums);
    prep_static(a, warp_sums, WB, run0, cnt, b0);
  }
  for (int i = 0; i < cnt; ++i)
    if (ctx_of(a, b0 + i) == 0)
      for (int o = 0; o < (a.n_out > 0 ? a.n_out : 1); ++o) {
        T* dst = static_cast<T*>(a.n_out > 0 ? a.outs[o] : a.out) +
                 int64_t(b0 + i) * a.out_row_stride + int64_t(a.out_head0) * (row_elems / a.num_q_heads);
        for (int e = 0; e < row_elems; ++e) dst[e] = ts::from_float<T>(0.f);
      }
  for (int i = threadIdx.x; i < B * H; i += blockDim.x) a.arrive[i] = 0;
}

// Output row (sequence b, query head j) in destination o (< max(n_out, 1)).
template <typename T, int D>
__device__ __forceinline__ T* out_row(const DecodeArgs& a, int o, int b, int j) {
  T* base = static_cast<T*>(a.n_out == 0 ? a.out : a.outs[o]);
  return base + int64_t(b) * a.out_row_stride + int64_t(a.out_head0 + j) * D;
}

// --------------------------------------------------------------------------- main kernel

// Packs two floats and transposes the 8x8 half-precision matrix they belong to across the warp.
template <typename Mma>
__device__ __forceinline__ uint32_t movmatrix_pack(float lo, float hi) {
  return ts::movmatrix_trans(Mma::pack(lo, hi));
}

template <int D>
struct Geometry {
  static constexpr int kHalves = D / 64;              // 64-column TMA boxes per row
  static constexpr int kTileBytes = kBlock * D * 2;   // one block's K (or V) for one head
  static constexpr int kStageBytes = 2 * kTileBytes;  // K tile then V tile
  static constexpr int kStages = D == 128 ? TS_DECODE_STAGES_D128 : 6;
  static constexpr bool kOneBox = TS_DECODE_ONE_BOX && D == 128;
  static constexpr int kRingBytes = kStages * kStageBytes;
  // ring, then one mbarrier (8 B) and one item descriptor (32 B) per stage, + alignment slack
  static constexpr int kBarBytes = (kWarps * kStages * 8 + 15) / 16 * 16;
  static constexpr int kSmemBytes = kWarps * kRingBytes + kBarBytes + kWarps * kStages * 32 + 1024;
};

// Byte offset of 16-byte chunk `cg` (dims 8cg..8cg+7) of token `t` inside a K or V tile in
// shared memory, as the 128-byte-swizzled TMA boxes lay it out: either two 64-dim boxes of
// 16 rows (row t of box cg / 8), or one box of 32 128-byte rows (row 2t + cg / 8).
template <int D>
__device__ __forceinline__ uint32_t tile_off(int t, int cg) {
  if constexpr (Geometry<D>::kOneBox) {
    const int r = 2 * t + (cg >> 3);
    return r * 128 + (((cg & 7) ^ (r & 7)) << 4);
  } else {
    return (cg >> 3) * 2048 + t * 128 + (((cg & 7) ^ (t & 7)) << 4);
  }
}

struct ItemInfo {
  int b, h, blk0, nparts, ctx, nblk, part_global, slot0;
};

template <typename T, int D, int NT>
__global__ void __launch_bounds__(kWarps * 32, 1)
    paged_decode_kernel(const __grid_constant__ CUtensorMap kmap,
                        const __grid_constant__ CUtensorMap vmap, const DecodeArgs a) {
  using G = Geometry<D>;
  using Mma = ts::MmaOp<T>;
  constexpr int S = G::kStages;
  constexpr int KSTEPS = D / 16;
  constexpr int MTILES = D / 16;
  constexpr int NT8 = NT * 8;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = ts::smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023) & ~1023u) - raw);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int g = lane >> 2, t = lane & 3;
  // Launched programmatically after the prep kernel (or after the caller's previous kernel when
  // the plan is reused): everything below reads the plan, the tables, the query or the pool, so
  // wait until the grid before this one has completed and its writes are visible.
  ts::wait_prior_grid();
  // A pull gather launched programmatically after this grid may now become resident: it only
  // polls the ranks' epochs until this grid (and the peers') publish, and it waits for this
  // grid to complete before it exits.
  if (a.n_signals > 0 && !a.remote_out) ts::allow_dependents();
  if (a.reuse_plan) {
    // The plan must have been made for this batch, head count, table width and grid.
    if (__ldg(a.header + 6) != a.batch || __ldg(a.header + 7) != a.num_kv_heads ||
        __ldg(a.header + 8) != a.max_blocks || __ldg(a.header + 9) != a.grid_warps) {
      if (blockIdx.x == 0 && threadIdx.x == 0) atomicExch(a.header + 1, 4);
      return;
    }
    // Rows of empty contexts (no partition writes them): zeros, as the prep kernel writes them.
    if (blockIdx.x == 0)
      for (int b = threadIdx.x; b < a.batch; b += blockDim.x)
        if (ctx_of(a, b) == 0)
          for (int o = 0; o < (a.n_out > 0 ? a.n_out : 1); ++o)
            for (int j = 0; j < a.num_q_heads; ++j) {
              T* row = out_row<T, D>(a, o, b, j);
              for (int e = 0; e < D; ++e) row[e] = ts::from_float<T>(0.f);
            }
  }
  uint8_t* ring = smem + warp * G::kRingBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kWarps * G::kRingBytes) + warp * S;
  // Per stage: {partition, block | invalid flag, sequence, first block}, {first slot of its
  // (sequence, head), partitions of that (sequence, head) | KV head << 16, context length,
  // slot of the partition}.
  int4* meta =
      reinterpret_cast<int4*>(smem + kWarps * G::kRingBytes + G::kBarBytes) + warp * S * 2;

  if (lane == 0) {
    for (int s = 0; s < S; ++s) ts::mbar_init(&bars[s], 1);
    ts::fence_mbar_init();
  }
  __syncwarp();

  // This warp's work: items claimed from the counter (item = partition * H + head), or its
  // group's partitions for its head (static split: warp gw = group * H + head).
  const bool dynamic = __ldg(a.header + 2) != 0;
  const int gw = blockIdx.x * kWarps + warp;
  const int H = a.num_kv_heads;
  int nxt = 0, part_end = 0, my_h = 0;
  if (dynamic) {
    part_end = __ldg(a.header + 3);
  } else if (gw / H < __ldg(a.header + 3)) {
    my_h = gw % H;
    nxt = __ldg(a.group_first + gw / H);
    part_end = __ldg(a.group_first + gw / H + 1);
  }

  // ---- producer state (warp-uniform except the tables, one table entry per lane)
  constexpr int TABW = (kPartBlocks + 31) / 32;  // table entries per lane
  int p_item = -1, p_blk = 0, p_nblk = 0;
  ItemInfo p_it{};
  int p_table[TABW];
  bool p_done = false;

  // The next item is fetched by a chain of dependent loads (claim counter, descriptor, table
  // row), advanced one step per produce() call once at most kPrefetchBlocks blocks of the
  // current item remain to be issued: the latencies hide behind the current item's last
  // blocks, and a dynamic claim is made only shortly before the warp can start it, so no warp
  // holds a claimed item while other warps run out of work.
  constexpr int kPrefetchBlocks = TS_DECODE_PREFETCH_BLOCKS;
  int f_state = 0;  // 0 idle, 1 claim issued, 2 descriptor loads issued, 3 ready, -1 no more work
  int f_claim = 0, f_h = 0, f_item = 0;
  int4 f_d = make_int4(0, 0, 0, 0), f_e = make_int4(0, 0, 0, 0);
  ItemInfo f_it{};
  int f_table[TABW];
  auto issue_descriptor = [&](int part, int h, int item) {
    f_h = h;
    f_item = item;
    f_d = __ldg(a.part_info + 2 * part);
    f_e = __ldg(a.part_info + 2 * part + 1);
    f_state = 2;
  };
  auto fetch_step = [&]() {
    if (f_state == 0) {
      if (dynamic) {
        if (lane == 0) f_claim = atomicAdd(a.header, 1);
        f_state = 1;
      } else if (nxt < part_end) {
        issue_descriptor(nxt, my_h, nxt * H + my_h);
        ++nxt;
      } else {
        f_state = -1;
      }
    } else if (f_state == 1) {
      const int c = __shfl_sync(0xffffffffu, f_claim, 0);
      if (c < part_end) {
        issue_descriptor(c / H, c % H, c);
      } else {
        f_state = -1;
      }
    } else if (f_state == 2) {
      // (partition, KV head) -> blocks to read and the partial-result slots of its
      // (sequence, head)
      f_it.b = f_d.x;
      f_it.h = f_h;
      f_it.blk0 = f_d.y;
      f_it.nblk = f_d.z;
      f_it.nparts = f_e.y;
      f_it.slot0 = f_e.x * a.num_kv_heads + f_h * f_it.nparts;
      f_it.part_global = f_it.slot0 + f_d.w;
      f_it.ctx = f_e.z;
      const int32_t* row = a.block_tables + int64_t(f_it.b) * a.max_blocks + f_it.blk0;
#pragma unroll
      for (int w = 0; w < TABW; ++w)
        f_table[w] = lane + 32 * w < f_it.nblk ? __ldg(row + lane + 32 * w) : 0;
      f_state = 3;
    }
  };

  auto produce = [&](int s) {
    if (!p_done && p_blk == p_nblk) {
      while (f_state >= 0 && f_state < 3) fetch_step();  // first item, or a short one
      if (f_state < 0) {
        p_done = true;
      } else {
        p_it = f_it;
        p_item = f_item;
#pragma unroll
        for (int w = 0; w < TABW; ++w) p_table[w] = f_table[w];
        p_nblk = p_it.nblk;
        p_blk = 0;
        f_state = 0;
      }
    }
    if (p_done) {
      if (lane == 0) {
        meta[2 * s] = make_int4(-1, 0, 0, 0);
        ts::mbar_arrive(&bars[s]);
      }
      return;
    }
    const int tab = TABW == 1 || p_blk < 32 ? p_table[0] : p_table[TABW - 1];
    const int phys = __shfl_sync(0xffffffffu, tab, p_blk & 31);
    const bool valid = phys >= 0 && int64_t(phys) < a.num_blocks;
    if (lane == 0) {
      meta[2 * s] = make_int4(p_item, valid ? p_blk : (p_blk | 0x40000000), p_it.b, p_it.blk0);
      meta[2 * s + 1] = make_int4(p_it.slot0, p_it.nparts | (p_it.h << 16), p_it.ctx,
                                  p_it.part_global);  // nparts < 2^16, h < 2^15
      if (valid) {
        ts::mbar_arrive_expect_tx(&bars[s], G::kStageBytes);
        const int row = (phys * a.num_kv_heads + p_it.h) * kBlock;
        uint8_t* st = ring + s * G::kStageBytes;
        if constexpr (G::kOneBox) {
          ts::tma_load_2d(st, &kmap, &bars[s], 0, 2 * row);
          ts::tma_load_2d(st + G::kTileBytes, &vmap, &bars[s], 0, 2 * row);
        } else {
#pragma unroll
          for (int hf = 0; hf < G::kHalves; ++hf) {
            ts::tma_load_2d(st + hf * 2048, &kmap, &bars[s], hf * 64, row);
            ts::tma_load_2d(st + G::kTileBytes + hf * 2048, &vmap, &bars[s], hf * 64, row);
          }
        }
      } else {
        atomicExch(a.header + 1, 2);  // block id outside the pool: flagged, block skipped
        ts::mbar_arrive(&bars[s]);
      }
    }
    ++p_blk;
    if (f_state >= 0 && f_state < 3 && p_nblk - p_blk <= kPrefetchBlocks) fetch_step();
  };

#pragma unroll 1
  for (int s = 0; s < S; ++s) produce(s);

  // ---- consumer state
  int cur_item = -1;
  ItemInfo it{};
  uint32_t qf[NT][KSTEPS][2];
  float oacc[NT][MTILES][4];
  float m_run[NT][2], l_run[NT][2];

  auto start_item = [&](const int4& m0, const int4& m1) {
    cur_item = m0.x;
    it.b = m0.z;
    it.blk0 = m0.w;
    it.slot0 = m1.x;
    it.nparts = m1.y & 0xffff;
    it.h = m1.y >> 16;
    it.ctx = m1.z;
    it.part_global = m1.w;
    const T* qb = static_cast<const T*>(a.query) + int64_t(it.b) * a.q_stride;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int head = nt * 8 + g;
      const bool hv = head < a.group;
      const uint32_t* qrow =
          reinterpret_cast<const uint32_t*>(qb + int64_t(it.h * a.group + head) * D);
#pragma unroll
      for (int ks = 0; ks < KSTEPS; ++ks) {
        qf[nt][ks][0] = hv ? __ldg(qrow + (ks * 16 + 2 * t) / 2) : 0u;
        qf[nt][ks][1] = hv ? __ldg(qrow + (ks * 16 + 8 + 2 * t) / 2) : 0u;
      }
#pragma unroll
      for (int mt = 0; mt < MTILES; ++mt)
#pragma unroll
        for (int j = 0; j < 4; ++j) oacc[nt][mt][j] = 0.f;
      m_run[nt][0] = m_run[nt][1] = -INFINITY;
      l_run[nt][0] = l_run[nt][1] = 0.f;
    }
  };

  // Output destinations, one per lane (n_out <= 64): lane o holds destination o and lane o
  // destination o + 32, so a finished item finds each base with a shuffle instead of a
  // dependent global load per destination.
  unsigned long long dst_lo = 0, dst_hi = 0;
  if (a.n_out > 0) {
    if (lane < a.n_out) dst_lo = reinterpret_cast<unsigned long long>(a.outs[lane]);
    if (lane + 32 < a.n_out) dst_hi = reinterpret_cast<unsigned long long>(a.outs[lane + 32]);
  } else {
    dst_lo = reinterpret_cast<unsigned long long>(a.out);
  }
  const int n_dst = a.n_out > 0 ? a.n_out : 1;
  // Row (sequence b, query head j) of destination o, and whether its rows take 16-byte stores.
  auto dst_row = [&](int o, int b, int j, bool& vec) -> T* {
    const unsigned long long base = __shfl_sync(0xffffffffu, o < 32 ? dst_lo : dst_hi, o & 31);
    vec = ((base | (unsigned long long)(a.out_row_stride * sizeof(T))) & 15) == 0;
    return reinterpret_cast<T*>(base) + int64_t(b) * a.out_row_stride + int64_t(a.out_head0 + j) * D;
  };

  auto finish_item = [&]() {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        float l = l_run[nt][j];
        l += __shfl_xor_sync(0xffffffffu, l, 4);
        l += __shfl_xor_sync(0xffffffffu, l, 8);
        l += __shfl_xor_sync(0xffffffffu, l, 16);
        l_run[nt][j] = l;
      }
    if (it.nparts == 1) {
      // After the transpose lane (g, t) holds, for head nt * 8 + g, the words of dims
      // 16 mt + 2t (lo) and 16 mt + 8 + 2t (hi): a quad covers 16-byte chunk c = 2 mt (+1 for
      // hi). Each chunk is gathered into lane t = c % 4 of its quad and stored as one vector.
      constexpr int NCH = 2 * MTILES;  // 16-byte chunks per head row
      uint32_t pw[NT][MTILES][2];
      uint4 ch[NT][NCH / 4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const float i0 = l_run[nt][0] > 0.f ? 1.f / l_run[nt][0] : 0.f;
        const float i1 = l_run[nt][1] > 0.f ? 1.f / l_run[nt][1] : 0.f;
#pragma unroll
        for (int mt = 0; mt < MTILES; ++mt) {
          pw[nt][mt][0] = movmatrix_pack<Mma>(oacc[nt][mt][0] * i0, oacc[nt][mt][1] * i1);
          pw[nt][mt][1] = movmatrix_pack<Mma>(oacc[nt][mt][2] * i0, oacc[nt][mt][3] * i1);
        }
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
          uint32_t v[4];
#pragma unroll
          for (int w = 0; w < 4; ++w) v[w] = __shfl_sync(0xffffffffu, pw[nt][c / 2][c % 2], (g << 2) | w);
          if (t == c % 4) ch[nt][c / 4] = make_uint4(v[0], v[1], v[2], v[3]);
        }
      }
#pragma unroll 1
      for (int o = 0; o < n_dst; ++o) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const int head = nt * 8 + g;  // after the transpose a lane owns one head
          bool vec;
          T* orow = dst_row(o, it.b, it.h * a.group + head, vec);
          if (head >= a.group) continue;
          if (vec) {
#pragma unroll
            for (int j = 0; j < NCH / 4; ++j)
              *reinterpret_cast<uint4*>(orow + 8 * (4 * j + t)) = ch[nt][j];
          } else {
            uint32_t* w32 = reinterpret_cast<uint32_t*>(orow);
#pragma unroll
            for (int mt = 0; mt < MTILES; ++mt) {
              w32[(mt * 16 + 2 * t) / 2] = pw[nt][mt][0];
              w32[(mt * 16 + 8 + 2 * t) / 2] = pw[nt][mt][1];
            }
          }
        }
      }
      return;
    }
    // Partial result of one partition: unnormalised O^T, running max and sum.
    const int64_t slot = it.part_global;
    float* po = a.part_o + slot * D * NT8;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int mt = 0; mt < MTILES; ++mt) {
        *reinterpret_cast<float2*>(po + (mt * 16 + g) * NT8 + nt * 8 + 2 * t) =
            make_float2(oacc[nt][mt][0], oacc[nt][mt][1]);
        *reinterpret_cast<float2*>(po + (mt * 16 + 8 + g) * NT8 + nt * 8 + 2 * t) =
            make_float2(oacc[nt][mt][2], oacc[nt][mt][3]);
      }
    if (g == 0) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        a.part_ml[slot * NT8 + nt * 8 + 2 * t] = make_float2(m_run[nt][0], l_run[nt][0]);
        a.part_ml[slot * NT8 + nt * 8 + 2 * t + 1] = make_float2(m_run[nt][1], l_run[nt][1]);
      }
    }
    __threadfence();
    __syncwarp();
    int old = 0;
    if (lane == 0) old = atomicAdd(a.arrive + it.b * a.num_kv_heads + it.h, 1);
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old != it.nparts - 1) return;
    __threadfence();
    // Last partition of (b, h) to finish: merge all of them. A long sequence has tens of
    // partitions and its merge can run in the kernel's tail, so the loads of several
    // partitions are kept in flight at once (the sums still run in partition order).
    const int hd = lane % NT8;  // fixed head per lane in the [D][NT8] layout
    const int64_t slot0 = it.slot0;
    const int np = it.nparts;
    // Running max: the lanes of one head split the partitions (32 / NT8 per pass, four passes'
    // loads in flight), then reduce across those lanes.
    constexpr int kLanesPerHead = 32 / NT8;
    float mx = -INFINITY;
    for (int p0 = lane / NT8; p0 < np; p0 += 4 * kLanesPerHead) {
      float v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int p = p0 + u * kLanesPerHead;
        v[u] = p < np ? __ldcg(&a.part_ml[(slot0 + p) * NT8 + hd].x) : -INFINITY;
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) mx = fmaxf(mx, v[u]);
    }
#pragma unroll
    for (int o = NT8; o < 32; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    constexpr int PER = D * NT8 / 32;
    float acc[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) acc[i] = 0.f;
    float lsum = 0.f;
    int p = 0;
    for (; p + 1 < np; p += 2) {  // two partitions' loads in flight
      const int64_t s0 = slot0 + p, s1 = s0 + 1;
      const float2 ml0 = __ldcg(&a.part_ml[s0 * NT8 + hd]);
      const float2 ml1 = __ldcg(&a.part_ml[s1 * NT8 + hd]);
      const float* src0 = a.part_o + s0 * D * NT8;
      const float* src1 = a.part_o + s1 * D * NT8;
      float x0[PER], x1[PER];
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        x0[i] = __ldcg(src0 + lane + 32 * i);
        x1[i] = __ldcg(src1 + lane + 32 * i);
      }
      const float w0 = ml0.x == -INFINITY ? 0.f : exp2f(ml0.x - mx);
      const float w1 = ml1.x == -INFINITY ? 0.f : exp2f(ml1.x - mx);
      lsum += w0 * ml0.y;
      lsum += w1 * ml1.y;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        acc[i] += w0 * x0[i];
        acc[i] += w1 * x1[i];
      }
    }
    if (p < np) {
      const int64_t sl = slot0 + p;
      const float2 ml = __ldcg(&a.part_ml[sl * NT8 + hd]);
      const float w = ml.x == -INFINITY ? 0.f : exp2f(ml.x - mx);
      lsum += w * ml.y;
      const float* src = a.part_o + sl * D * NT8;
#pragma unroll
      for (int i = 0; i < PER; ++i) acc[i] += w * __ldcg(src + lane + 32 * i);
    }
    const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
    // Lane (hd, kq = lane / NT8) holds dims kq + LPH * i of head hd. Gather each 16-byte chunk
    // (8 consecutive dims) of a head into lane kq = chunk % LPH and store it as one vector.
    constexpr int LPH = 32 / NT8;     // lanes per head
    constexpr int NCH = D / 8;        // 16-byte chunks per head row
    const int kq = lane / NT8;
    uint4 mch[NCH / LPH];
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      float f[8];
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        const int dim = 8 * c + m;
        f[m] = __shfl_sync(0xffffffffu, acc[dim / LPH], hd + NT8 * (dim % LPH)) * inv;
      }
      if (kq == c % LPH)
        mch[c / LPH] = make_uint4(Mma::pack(f[0], f[1]), Mma::pack(f[2], f[3]), Mma::pack(f[4], f[5]),
                                  Mma::pack(f[6], f[7]));
    }
#pragma unroll 1
    for (int o = 0; o < n_dst; ++o) {
      bool vec;
      T* orow = dst_row(o, it.b, it.h * a.group + hd, vec);  // every lane takes the shuffle
      if (hd >= a.group) continue;
      if (vec) {
#pragma unroll
        for (int j = 0; j < NCH / LPH; ++j)
          *reinterpret_cast<uint4*>(orow + 8 * (j * LPH + kq)) = mch[j];
      } else {
#pragma unroll
        for (int i = 0; i < PER; ++i) orow[(lane + 32 * i) / NT8] = ts::from_float<T>(acc[i] * inv);
      }
    }
    if (lane == 0) a.arrive[it.b * a.num_kv_heads + it.h] = 0;
  };

  uint32_t k = 0;
  bool failed = false;
#pragma unroll 1
  while (true) {
    const int s = k % S;
    const uint32_t ph = (k / S) & 1;
    if (!ts::mbar_wait_bounded(&bars[s], ph)) {
      failed = true;
      break;
    }
    const int4 md = meta[2 * s];
    if (md.x < 0) break;
    if (md.x != cur_item) {
      if (cur_item >= 0) finish_item();
      start_item(md, meta[2 * s + 1]);
    }
    if ((md.y & 0x40000000) == 0) {
      const uint32_t kb = ts::smem_u32(ring + s * G::kStageBytes);
      const uint32_t vb = kb + G::kTileBytes;
      const int tok0 = (it.blk0 + md.y) * kBlock;
      const int nvalid = it.ctx - tok0;

      // S^T[token][head] = K Q^T
      float sacc[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int j = 0; j < 4; ++j) sacc[nt][j] = 0.f;
      {
        const int row = (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
        for (int ks = 0; ks < KSTEPS; ++ks) {
          uint32_t af[4];
          ts::ldmatrix_x4(af, kb + tile_off<D>(row, ks * 2 + (lane >> 4)));
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) Mma::run(sacc[nt], af, qf[nt][ks][0], qf[nt][ks][1]);
        }
      }
      // Online softmax per head (column); lanes sharing t hold the same two heads.
      uint32_t pb[NT][4];  // movmatrix'd B fragments: hi(tok 0-7), hi(8-15), lo(0-7), lo(8-15)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        float s00 = sacc[nt][0] * a.scale_log2, s01 = sacc[nt][1] * a.scale_log2;
        float s10 = sacc[nt][2] * a.scale_log2, s11 = sacc[nt][3] * a.scale_log2;
        if (g >= nvalid) s00 = s01 = -INFINITY;
        if (g + 8 >= nvalid) s10 = s11 = -INFINITY;
        float bm0 = fmaxf(s00, s10), bm1 = fmaxf(s01, s11);
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
          bm0 = fmaxf(bm0, __shfl_xor_sync(0xffffffffu, bm0, o));
          bm1 = fmaxf(bm1, __shfl_xor_sync(0xffffffffu, bm1, o));
        }
        const float mn0 = fmaxf(m_run[nt][0], bm0), mn1 = fmaxf(m_run[nt][1], bm1);
        const float c0 = exp2f(m_run[nt][0] - mn0), c1 = exp2f(m_run[nt][1] - mn1);
        m_run[nt][0] = mn0;
        m_run[nt][1] = mn1;
        const float p00 = exp2f(s00 - mn0), p01 = exp2f(s01 - mn1);
        const float p10 = exp2f(s10 - mn0), p11 = exp2f(s11 - mn1);
        l_run[nt][0] = l_run[nt][0] * c0 + p00 + p10;
        l_run[nt][1] = l_run[nt][1] * c1 + p01 + p11;
#pragma unroll
        for (int mt = 0; mt < MTILES; ++mt) {
          oacc[nt][mt][0] *= c0;
          oacc[nt][mt][1] *= c1;
          oacc[nt][mt][2] *= c0;
          oacc[nt][mt][3] *= c1;
        }
        const uint32_t h0 = Mma::pack(p00, p01), h1 = Mma::pack(p10, p11);
        const float2 f0 = Mma::unpack(h0), f1 = Mma::unpack(h1);
        const uint32_t l0 = Mma::pack(p00 - f0.x, p01 - f0.y);
        const uint32_t l1 = Mma::pack(p10 - f1.x, p11 - f1.y);
        pb[nt][0] = ts::movmatrix_trans(h0);
        pb[nt][1] = ts::movmatrix_trans(h1);
        pb[nt][2] = ts::movmatrix_trans(l0);
        pb[nt][3] = ts::movmatrix_trans(l1);
      }
      // O^T[dim][head] += V^T P^T
      {
        const int vtok = (lane & 7) + (lane >> 4) * 8;
#pragma unroll
        for (int mt = 0; mt < MTILES; ++mt) {
          uint32_t af[4];
          ts::ldmatrix_x4_trans(af, vb + tile_off<D>(vtok, mt * 2 + ((lane >> 3) & 1)));
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            Mma::run(oacc[nt][mt], af, pb[nt][0], pb[nt][1]);
            Mma::run(oacc[nt][mt], af, pb[nt][2], pb[nt][3]);
          }
        }
      }
    }
    __syncwarp();
    ts::fence_proxy_async_smem();
    produce(s);
    ++k;
  }
  if (failed) {
    if (lane == 0) atomicExch(a.header + 1, 1);
    // Let copies still in flight land before the CTA's shared memory is released.
    for (int j = 1; j < S; ++j) {
      const uint32_t kk = k + j;
      ts::mbar_wait_bounded(&bars[kk % S], (kk / S) & 1);
    }
  } else if (cur_item >= 0) {
    finish_item();
  }
  // With peer outputs, every thread's output stores (local and peer) are made visible
  // system-wide before its CTA counts itself done; the last CTA then publishes the epoch to
  // every rank. The last CTA also re-zeroes the claim counter and this counter: every CTA has
  // stopped claiming, and the next launch on the stream may reuse the plan.
  // Before the CTA counts itself done, its output stores must be ordered before the last CTA's
  // system-scope release of the epoch. Stores into another GPU's memory (push) are fenced at
  // system scope by every thread; local stores (pull) only need the CTA barrier and one
  // GPU-scope fence by the counting thread, whose release chain (fence, done counter, the last
  // CTA's fence.sc.sys and st.release.sys) covers the whole CTA's writes.
  if (a.n_signals > 0 && a.remote_out) __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    if (a.n_signals > 0 && !a.remote_out) __threadfence();
    const int done = atomicAdd(a.header + 4, 1);
    if (done == int(gridDim.x) - 1) {
      if (a.n_signals > 0) {
        __threadfence_system();
        for (int r = 0; r < a.n_signals; ++r) {
          int* flag = a.signals[r] + a.signal_index;
          asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(flag), "r"(a.epoch) : "memory");
        }
      }
      a.header[0] = 0;
      a.header[4] = 0;
    }
  }
}

// An empty batch still takes part in the exchange: the epoch is published to every rank, so
// their waits for it end.
__global__ void publish_epoch_kernel(int* const* signals, int world, int index, unsigned epoch) {
  const int r = threadIdx.x;
  if (r >= world) return;
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(signals[r] + index), "r"(epoch)
               : "memory");
}

// Waits until every rank has published `epoch` into signals[0..world) (this rank's signal
// array, written by the ranks' decode kernels), with a bounded spin: on timeout *status = 3.
__global__ void wait_peers_kernel(const int* signals, int world, unsigned epoch, int* status) {
  const int r = threadIdx.x;
  if (r >= world) return;
  for (long long i = 0; i < (1LL << 20); ++i) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(signals + r) : "memory");
    if (int(v - epoch) >= 0) return;
    __nanosleep(256);
  }
  atomicExch(status, 3);
}

// --------------------------------------------------------------------------- host side

PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (cached[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

bool make_pool_map(CUtensorMap* map, const void* pool, int64_t rows, int hd, int dtype) {
  auto encode = get_encode();
  if (encode == nullptr) return false;
  // One box per 4 KiB tile views each 256-byte token row as two 128-byte rows.
  const bool one_box = TS_DECODE_ONE_BOX && hd == 128;
  const cuuint64_t dims[2] = {one_box ? 64 : cuuint64_t(hd),
                              one_box ? cuuint64_t(rows) * 2 : cuuint64_t(rows)};
  const cuuint64_t strides[1] = {one_box ? 128 : cuuint64_t(hd) * 2};
  const cuuint32_t box[2] = {64, one_box ? 2 * kBlock : cuuint32_t(kBlock)};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = encode(
      map, dtype == TS_BFLOAT16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
      2, const_cast<void*>(pool), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <typename T, int D, int NT>
int launch_fast(DecodeArgs a, const CUtensorMap& km, const CUtensorMap& vm, cudaStream_t s,
                bool plan = true) {
  using G = Geometry<D>;
  auto kern = paged_decode_kernel<T, D, NT>;
  // Once per device: later calls may be captured into a CUDA graph.
  static bool attr_done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_done[dev]) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, G::kSmemBytes);
    if (dev >= 0 && dev < 64) attr_done[dev] = true;
  }
  a.reuse_plan = plan ? 0 : 1;
  // Both kernels are launched with programmatic stream serialization: each may be scheduled
  // while the kernel before it still runs and waits on the device (griddepcontrol.wait) before
  // reading its inputs, so the decode grid's launch overlaps the prep kernel.
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (plan) {
    // One thread per sequence up to kPrepThreads (fewer threads: cheaper block-wide barriers
    // and scans, the prep kernel's critical path at small batches).
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(std::min(kPrepThreads, std::max(64, (a.batch + 31) / 32 * 32)));
    cfg.dynamicSmemBytes = 0;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, decode_prep_kernel<T>, a, a.num_q_heads * D);
    if (e != cudaSuccess) return ts::set_error(static_cast<int>(e), "paged_decode: prep launch: %s",
                                               cudaGetErrorString(e));
  }
  cfg.gridDim = dim3(num_sms());
  cfg.blockDim = dim3(kWarps * 32);
  cfg.dynamicSmemBytes = G::kSmemBytes;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, km, vm, a);
  if (e != cudaSuccess)
    return ts::set_error(static_cast<int>(e), "paged_decode: launch: %s", cudaGetErrorString(e));
  return ts::launch_status("paged_decode");
}

// Whether the tensor-core decode kernel covers these arguments.
bool fast_path(int hq, int hkv, int hd, int bs, int dtype, int64_t num_blocks, const void* kp,
               const void* vp, const void* q, int64_t q_stride, const void* out) {
  if (dtype != TS_BFLOAT16 && dtype != TS_FLOAT16) return false;
  if (bs != kBlock || (hd != 64 && hd != 128)) return false;
  if (hkv <= 0 || hq % hkv != 0 || hq / hkv > 16) return false;
  if (hkv > num_sms() * kWarps) return false;  // one warp per KV head in a group
  if (num_blocks * hkv * kBlock >= (int64_t(1) << 31)) return false;
  if ((reinterpret_cast<uint64_t>(kp) | reinterpret_cast<uint64_t>(vp)) % 16) return false;
  if ((reinterpret_cast<uint64_t>(q) | reinterpret_cast<uint64_t>(out)) % 4 || q_stride % 2)
    return false;
  return get_encode() != nullptr;
}

}  // namespace

namespace ts {
int paged_attention_portable(void* out, const void* query, int64_t q_stride, const void* kp,
                             const void* vp, const int32_t* bt, int max_blocks,
                             const int32_t* qsl, const int32_t* cl, int num_seqs, int num_rows,
                             int hq, int hkv, int hd, int bs, int64_t nb, float scale, int dtype,
                             cudaStream_t s);
}

extern "C" size_t ts_paged_decode_workspace_size(int32_t batch, int32_t num_q_heads,
                                                 int32_t num_kv_heads, int32_t head_dim,
                                                 int32_t max_blocks_per_seq, int32_t block_size,
                                                 int32_t dtype) {
  if (batch <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads != 0) return 0;
  if ((dtype != TS_BFLOAT16 && dtype != TS_FLOAT16) || block_size != kBlock ||
      (head_dim != 64 && head_dim != 128) || num_q_heads / num_kv_heads > 16)
    return 0;
  const int nt = num_q_heads / num_kv_heads > 8 ? 2 : 1;
  return ws_layout(batch, num_kv_heads, head_dim, max_blocks_per_seq, nt, num_sms() * kWarps).total;
}

namespace {

int paged_decode_call(void* out, const void* query, int64_t query_token_stride,
                      const void* key_pool, const void* value_pool, const int32_t* block_tables,
                      int32_t max_blocks_per_seq, const int32_t* context_lens, int32_t batch,
                      int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                      int32_t block_size, int64_t num_blocks, float scale, int32_t dtype,
                      void* workspace, size_t workspace_bytes, void* stream, bool plan) {
  if (ts::dtype_size(dtype) == 0)
    return ts::set_error(TS_ERR_INVALID_ARGUMENT, "paged_decode: bad dtype %d", dtype);
  if (batch < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads ||
      head_dim <= 0 || block_size <= 0 || num_blocks <= 0 || max_blocks_per_seq <= 0)
    return ts::set_error(TS_ERR_INVALID_ARGUMENT,
                         "paged_decode: bad sizes (batch %d, heads %d/%d, head_dim %d, "
                         "block_size %d, blocks %lld, max_blocks %d)",
                         batch, num_q_heads, num_kv_heads, head_dim, block_size,
                         (long long)num_blocks, max_blocks_per_seq);
  if (query_token_stride < int64_t(num_q_heads) * head_dim)
    return ts::set_error(TS_ERR_INVALID_ARGUMENT, "paged_decode: query stride too small");
  if (batch == 0) return ts::ok();
  if (!out || !query || !key_pool || !value_pool || !block_tables || !context_lens)
    return ts::set_error(TS_ERR_INVALID_ARGUMENT, "paged_decode: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (!fast_path(num_q_heads, num_kv_heads, head_dim, block_size, dtype, num_blocks, key_pool,
                 value_pool, query, query_token_stride, out))
    return ts::paged_attention_portable(out, query, query_token_stride, key_pool, value_pool,
                                        block_tables, max_blocks_per_seq, nullptr, context_lens,
                                        batch, batch, num_q_heads, num_kv_heads, head_dim,
                                        block_size, num_blocks, scale, dtype, s);
  if (batch > 8192)
    return ts::set_error(TS_ERR_UNSUPPORTED, "paged_decode: batch %d above 8192", batch);
  if (int64_t(batch) * max_blocks_per_seq >= (int64_t(1) << 31) ||
      max_blocks_per_seq > (1 << 20) || num_sms() * kWarps > kMaxGridWarps)
    return ts::set_error(TS_ERR_UNSUPPORTED, "paged_decode: batch x max_blocks or grid too large");
  const int group = num_q_heads / num_kv_heads;
  const int nt = group > 8 ? 2 : 1;
  const WsLayout w = ws_layout(batch, num_kv_heads, head_dim, max_blocks_per_seq, nt, num_sms() * kWarps);
  if (workspace == nullptr || workspace_bytes < w.total)
    return ts::set_error(TS_ERR_WORKSPACE_TOO_SMALL,
                         "paged_decode: workspace of %zu bytes, need %zu", workspace_bytes,
                         w.total);
  if (reinterpret_cast<uint64_t>(workspace) % 256)
    return ts::set_error(TS_ERR_MISALIGNED, "paged_decode: workspace not 256-byte aligned");
  CUtensorMap km, vm;
  const int64_t rows = num_blocks * num_kv_heads * kBlock;
  if (!make_pool_map(&km, key_pool, rows, head_dim, dtype) ||
      !make_pool_map(&vm, value_pool, rows, head_dim, dtype))
    return ts::set_error(TS_ERR_INVALID_ARGUMENT, "paged_decode: cannot encode TMA map of pool");
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  DecodeArgs a;
  a.out = out;
  a.outs = nullptr;
  a.n_out = 0;
  a.out_row_stride = int64_t(num_q_heads) * head_dim;
  a.out_head0 = 0;
  a.n_signals = 0;
  a.remote_out = 0;
  a.signals = nullptr;
  a.signal_index = 0;
  a.epoch = 0;
  a.query = query;
  a.q_stride = query_token_stride;
  a.block_tables = block_tables;
  a.context_lens = context_lens;
  a.max_blocks = max_blocks_per_seq;
  a.batch = batch;
  a.num_q_heads = num_q_heads;
  a.num_kv_heads = num_kv_heads;
  a.group = group;
  a.num_blocks = num_blocks;
  a.scale_log2 = scale * kLog2e;
  a.grid_warps = num_sms() * kWarps;
  a.header = reinterpret_cast<int*>(ws);
  a.chunk_prefix = reinterpret_cast<int*>(ws + w.chunk_prefix);
  a.part_info = reinterpret_cast<int4*>(ws + w.part_info);
  a.group_first = reinterpret_cast<int*>(ws + w.group_first);
  a.arrive = reinterpret_cast<int*>(ws + w.arrive);
  a.part_o = reinterpret_cast<float*>(ws + w.part_o);
  a.part_ml = reinterpret_cast<float2*>(ws + w.part_ml);
#define TS_FAST(T)                                                             \
  if (head_dim == 128)                                                         \
    return nt == 1 ? launch_fast<T, 128, 1>(a, km, vm, s, plan)                \
                   : launch_fast<T, 128, 2>(a, km, vm, s, plan);               \
  return nt == 1 ? launch_fast<T, 64, 1>(a, km, vm, s, plan)                   \
                 : launch_fast<T, 64, 2>(a, km, vm, s, plan);
  if (dtype == TS_BFLOAT16) {
    TS_FAST(__nv_bfloat16)
  }
  TS_FAST(__half)
#undef TS_FAST
}

}  // namespace

extern "C" int ts_paged_decode(void* out, const void* query, int64_t query_token_stride,
                               const void* key_pool, const void* value_pool,
                               const int32_t* block_tables, int32_t max_blocks_per_seq,
                               const int32_t* context_lens, int32_t batch, int32_t num_q_heads,
                               int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                               int64_t num_blocks, float scale, int32_t dtype, void* workspace,
                               size_t workspace_bytes, void* stream) {
  return paged_decode_call(out, query, query_token_stride, key_pool, value_pool, block_tables,
                           max_blocks_per_seq, context_lens, batch, num_q_heads, num_kv_heads,
                           head_dim, block_size, num_blocks, scale, dtype, workspace,
                           workspace_bytes, stream, true);
}

extern "C" int ts_paged_decode_planned(void* out, const void* query, int64_t query_token_stride,
                                       const void* key_pool, const void* value_pool,
                                       const int32_t* block_tables, int32_t max_blocks_per_seq,
                                       const int32_t* context_lens, int32_t batch,
                                       int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                                       int32_t block_size, int64_t num_blocks, float scale,
                                       int32_t dtype, void* workspace, size_t workspace_bytes,
                                       void* stream) {
  return paged_decode_call(out, query, query_token_stride, key_pool, value_pool, block_tables,
                           max_blocks_per_seq, context_lens, batch, num_q_heads, num_kv_heads,
                           head_dim, block_size, num_blocks, scale, dtype, workspace,
                           workspace_bytes, stream, false);
}

// --------------------------------------------------------------------------- no-alloc variant
//
// ts_paged_decode_no_alloc runs the same decode kernels as ts_paged_decode, but its scratch
// (partition partials, prefix sums, counters) lives in the file-scope device array below
// instead of a caller-provided workspace. It exists for callers that cannot allocate device
// memory for a workspace. The array is part of this library's device image, so every GPU
// that loads the library holds kStaticScratchBytes until the process exits.

namespace {

constexpr size_t kStaticScratchBytes = size_t(TS_NO_ALLOC_SCRATCH_BYTES);
static __device__ __align__(256) uint8_t g_decode_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_decode_scratch on the current device. In host code the array's name is
// only a host-side stand-in, so the real address is looked up once per device (with that
// device current) and cached.
int static_scratch(void** ptr) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return ts::set_error(static_cast<int>(e), "paged_decode_no_alloc: cudaGetDevice: %s",
                         cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices)
    return ts::set_error(TS_ERR_UNSUPPORTED, "paged_decode_no_alloc: device %d", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess || p == nullptr)
      return ts::set_error(static_cast<int>(e == cudaSuccess ? cudaErrorInvalidSymbol : e),
                           "paged_decode_no_alloc: cudaGetSymbolAddress: %s",
                           cudaGetErrorString(e));
    g_scratch_ptr[dev] = p;
  }
  *ptr = g_scratch_ptr[dev];
  return TS_OK;
}

}  // namespace

extern "C" int ts_paged_decode_no_alloc(void* out, const void* query, int64_t query_token_stride,
                                        const void* key_pool, const void* value_pool,
                                        const int32_t* block_tables, int32_t max_blocks_per_seq,
                                        const int32_t* context_lens, int32_t batch,
                                        int32_t num_q_heads, int32_t num_kv_heads,
                                        int32_t head_dim, int32_t block_size, int64_t num_blocks,
                                        float scale, int32_t dtype, void* stream) {
  if (ts::dtype_size(dtype) == 0)
    return ts::set_error(TS_ERR_INVALID_ARGUMENT, "paged_decode_no_alloc: bad dtype %d", dtype);
  if (batch < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads ||
      head_dim <= 0 || block_size <= 0 || num_blocks <= 0 || max_blocks_per_seq <= 0)
    return ts::set_error(TS_ERR_INVALID_ARGUMENT,
                         "paged_decode_no_alloc: bad sizes (batch %d, heads %d/%d, head_dim %d, "
                         "block_size %d, blocks %lld, max_blocks %d)",
                         batch, num_q_heads, num_kv_heads, head_dim, block_size,
                         (long long)num_blocks, max_blocks_per_seq);
  if (query_token_stride < int64_t(num_q_heads) * head_dim)
    return ts::set_error(TS_ERR_INVALID_ARGUMENT, "paged_decode_no_alloc: query stride too small");
  if (batch == 0) return ts::ok();
  if (!out || !query || !key_pool || !value_pool || !block_tables || !context_lens)
    return ts::set_error(TS_ERR_INVALID_ARGUMENT, "paged_decode_no_alloc: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (!fast_path(num_q_heads, num_kv_heads, head_dim, block_size, dtype, num_blocks, key_pool,
                 value_pool, query, query_token_stride, out))
    return ts::paged_attention_portable(out, query, query_token_stride, key_pool, value_pool,
                                        block_tables, max_blocks_per_seq, nullptr, context_lens,
                                        batch, batch, num_q_heads, num_kv_heads, head_dim,
                                        block_size, num_blocks, scale, dtype, s);
  if (batch > 8192)
    return ts::set_error(TS_ERR_UNSUPPORTED, "paged_decode_no_alloc: batch %d above 8192", batch);
  if (int64_t(batch) * max_blocks_per_seq >= (int64_t(1) << 31) ||
      max_blocks_per_seq > (1 << 20) || num_sms() * kWarps > kMaxGridWarps)
    return ts::set_error(TS_ERR_UNSUPPORTED,
                         "paged_decode_no_alloc: batch x max_blocks or grid too large");
  const int group = num_q_heads / num_kv_heads;
  const int nt = group > 8 ? 2 : 1;
  const WsLayout w = ws_layout(batch, num_kv_heads, head_dim, max_blocks_per_seq, nt, num_sms() * kWarps);
  if (w.total > kStaticScratchBytes)
    return ts::set_error(TS_ERR_WORKSPACE_TOO_SMALL,
                         "paged_decode_no_alloc: these sizes need %zu bytes of scratch but the "
                         "built-in scratch holds %zu; lower batch or max_blocks_per_seq, or call "
                         "ts_paged_decode with a workspace",
                         w.total, kStaticScratchBytes);
  void* scratch = nullptr;
  if (const int rc = static_scratch(&scratch); rc != TS_OK) return rc;
  CUtensorMap km, vm;
  const int64_t rows = num_blocks * num_kv_heads * kBlock;
  if (!make_pool_map(&km, key_pool, rows, head_dim, dtype) ||
      !make_pool_map(&vm, value_pool, rows, head_dim, dtype))
    return ts::set_error(TS_ERR_INVALID_ARGUMENT,
                         "paged_decode_no_alloc: cannot encode TMA map of pool");
  // The prep kernel zeroes the work counter, status word and arrival counters at the start of
  // every call; the partial-result slots are always written before they are read.
  uint8_t* ws = static_cast<uint8_t*>(scratch);
  DecodeArgs a;
  a.out = out;
  a.outs = nullptr;
  a.n_out = 0;
  a.out_row_stride = int64_t(num_q_heads) * head_dim;
  a.out_head0 = 0;
  a.n_signals = 0;
  a.remote_out = 0;
  a.signals = nullptr;
  a.signal_index = 0;
  a.epoch = 0;
  a.query = query;
  a.q_stride = query_token_stride;
  a.block_tables = block_tables;
  a.context_lens = context_lens;
  a.max_blocks = max_blocks_per_seq;
  a.batch = batch;
  a.num_q_heads = num_q_heads;
  a.num_kv_heads = num_kv_heads;
  a.group = group;
  a.num_blocks = num_blocks;
  a.scale_log2 = scale * kLog2e;
  a.grid_warps = num_sms() * kWarps;
  a.header = reinterpret_cast<int*>(ws);
  a.chunk_prefix = reinterpret_cast<int*>(ws + w.chunk_prefix);
  a.part_info = reinterpret_cast<int4*>(ws + w.part_info);
  a.group_first = reinterpret_cast<int*>(ws + w.group_first);
  a.arrive = reinterpret_cast<int*>(ws + w.arrive);
  a.part_o = reinterpret_cast<float*>(ws + w.part_o);
  a.part_ml = reinterpret_cast<float2*>(ws + w.part_ml);
#define TS_FAST_NA(T)                                                          \
  if (head_dim == 128)                                                         \
    return nt == 1 ? launch_fast<T, 128, 1>(a, km, vm, s)                      \
                   : launch_fast<T, 128, 2>(a, km, vm, s);                     \
  return nt == 1 ? launch_fast<T, 64, 1>(a, km, vm, s) : launch_fast<T, 64, 2>(a, km, vm, s);
  if (dtype == TS_BFLOAT16) {
    TS_FAST_NA(__nv_bfloat16)
  }
  TS_FAST_NA(__half)
#undef TS_FAST_NA
}

// --------------------------------------------------------------------------- peer variant
//
// ts_paged_decode_peer: the decode of one rank of a KV-head-sharded model, fused with the
// all-gather of the attention output. The rank's output rows go straight into every rank's
// full output buffer (peer stores over NVLink, no staging copy and no collective kernel), and
// the grid's last CTA publishes `epoch` into every rank's signal array; ts_wait_peers then
// waits, on the device and with a bounded spin, until all ranks have done so.

namespace {

// Whether `p` is memory of the current device (the kernel dereferences these arrays).
bool on_current_device(const void* p) {
  cudaPointerAttributes attr{};
  if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
    (void)cudaGetLastError();
    return false;
  }
  int dev = -1;
  return cudaGetDevice(&dev) == cudaSuccess && attr.type == cudaMemoryTypeDevice &&
         attr.device == dev;
}

}  // namespace

namespace {

int paged_decode_exchange(bool pull, void* const* dst_outs, int32_t world, int32_t rank,
                          int32_t* const* signals, uint32_t epoch, const void* query,
                          int64_t query_token_stride, const void* key_pool,
                          const void* value_pool, const int32_t* block_tables,
                          int32_t max_blocks_per_seq, const int32_t* context_lens, int32_t batch,
                          int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                          int32_t block_size, int64_t num_blocks, float scale, int32_t dtype,
                          void* workspace, size_t workspace_bytes, int32_t reuse_plan,
                          void* stream) {
  if (world < 1 || world > 64 || rank < 0 || rank >= world || epoch == 0)
    return ts::set_error(TS_ERR_INVALID_ARGUMENT,
                         "paged_decode_peer: bad world %d / rank %d / epoch %u", world, rank, epoch);
  if (ts::dtype_size(dtype) == 0)
    return ts::set_error(TS_ERR_INVALID_ARGUMENT, "paged_decode_peer: bad dtype %d", dtype);
  if (batch < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads ||
      head_dim <= 0 || block_size <= 0 || num_blocks <= 0 || max_blocks_per_seq <= 0)
    return ts::set_error(TS_ERR_INVALID_ARGUMENT, "paged_decode_peer: bad sizes");
  if (query_token_stride < int64_t(num_q_heads) * head_dim)
    return ts::set_error(TS_ERR_INVALID_ARGUMENT, "paged_decode_peer: query stride too small");
  if (!dst_outs || !signals || !query || !key_pool || !value_pool || !block_tables ||
      !context_lens)
    return ts::set_error(TS_ERR_INVALID_ARGUMENT, "paged_decode_peer: null pointer");
  if (!fast_path(num_q_heads, num_kv_heads, head_dim, block_size, dtype, num_blocks, key_pool,
                 value_pool, query, query_token_stride, query))
    return ts::set_error(TS_ERR_UNSUPPORTED,
                         "paged_decode_peer: needs the tensor-core decode path (bf16/fp16, block "
                         "16, head_dim 64/128, <= 16 query heads per KV head)");
  if (!on_current_device(dst_outs) || !on_current_device(signals))
    return ts::set_error(TS_ERR_INVALID_ARGUMENT,
                         "paged_decode_peer: dst_outs and signals must be arrays in the memory of "
                         "the current device");
  if (batch > 8192 || int64_t(batch) * max_blocks_per_seq >= (int64_t(1) << 31) ||
      max_blocks_per_seq > (1 << 20) || num_sms() * kWarps > kMaxGridWarps)
    return ts::set_error(TS_ERR_UNSUPPORTED, "paged_decode_peer: sizes too large");
  if (batch == 0) {
    publish_epoch_kernel<<<1, 64, 0, static_cast<cudaStream_t>(stream)>>>(
        reinterpret_cast<int* const*>(signals), world, rank, epoch);
    return ts::launch_status("paged_decode_peer");
  }
  const int group = num_q_heads / num_kv_heads;
  const int nt = group > 8 ? 2 : 1;
  const WsLayout w =
      ws_layout(batch, num_kv_heads, head_dim, max_blocks_per_seq, nt, num_sms() * kWarps);
  if (workspace == nullptr || workspace_bytes < w.total)
    return ts::set_error(TS_ERR_WORKSPACE_TOO_SMALL,
                         "paged_decode_peer: workspace of %zu bytes, need %zu", workspace_bytes,
                         w.total);
  if (reinterpret_cast<uint64_t>(workspace) % 256)
    return ts::set_error(TS_ERR_MISALIGNED, "paged_decode_peer: workspace not 256-byte aligned");
  CUtensorMap km, vm;
  const int64_t rows = num_blocks * num_kv_heads * kBlock;
  if (!make_pool_map(&km, key_pool, rows, head_dim, dtype) ||
      !make_pool_map(&vm, value_pool, rows, head_dim, dtype))
    return ts::set_error(TS_ERR_INVALID_ARGUMENT, "paged_decode_peer: cannot encode TMA map of pool");
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  DecodeArgs a;
  a.out = nullptr;
  // push: this rank's rows go into every rank's buffer; pull: into its own buffer only, and
  // the other ranks fetch them (ts_gather_peers).
  a.outs = pull ? dst_outs + rank : dst_outs;
  a.n_out = pull ? 1 : world;
  a.out_row_stride = int64_t(world) * num_q_heads * head_dim;
  a.out_head0 = rank * num_q_heads;
  a.n_signals = world;
  a.remote_out = pull ? 0 : 1;
  a.signals = reinterpret_cast<int* const*>(signals);
  a.signal_index = rank;
  a.epoch = epoch;
  a.query = query;
  a.q_stride = query_token_stride;
  a.block_tables = block_tables;
  a.context_lens = context_lens;
  a.max_blocks = max_blocks_per_seq;
  a.batch = batch;
  a.num_q_heads = num_q_heads;
  a.num_kv_heads = num_kv_heads;
  a.group = group;
  a.num_blocks = num_blocks;
  a.scale_log2 = scale * kLog2e;
  a.grid_warps = num_sms() * kWarps;
  a.header = reinterpret_cast<int*>(ws);
  a.chunk_prefix = reinterpret_cast<int*>(ws + w.chunk_prefix);
  a.part_info = reinterpret_cast<int4*>(ws + w.part_info);
  a.group_first = reinterpret_cast<int*>(ws + w.group_first);
  a.arrive = reinterpret_cast<int*>(ws + w.arrive);
  a.part_o = reinterpret_cast<float*>(ws + w.part_o);
  a.part_ml = reinterpret_cast<float2*>(ws + w.part_ml);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool plan = reuse_plan == 0;
#define TS_FAST_PEER(T)                                                        \
  if (head_dim == 128)                                                         \
    return nt == 1 ? launch_fast<T, 128, 1>(a, km, vm, s, plan)                \
                   : launch_fast<T, 128, 2>(a, km, vm, s, plan);               \
  return nt == 1 ? launch_fast<T, 64, 1>(a, km, vm, s, plan)                   \
                 : launch_fast<T, 64, 2>(a, km, vm, s, plan);
  if (dtype == TS_BFLOAT16) {
    TS_FAST_PEER(__nv_bfloat16)
  }
  TS_FAST_PEER(__half)
#undef TS_FAST_PEER
}

}  // namespace

extern "C" int ts_paged_decode_peer(void* const* dst_outs, int32_t world, int32_t rank,
                                    int32_t* const* signals, uint32_t epoch, const void* query,
                                    int64_t query_token_stride, const void* key_pool,
                                    const void* value_pool, const int32_t* block_tables,
                                    int32_t max_blocks_per_seq, const int32_t* context_lens,
                                    int32_t batch, int32_t num_q_heads, int32_t num_kv_heads,
                                    int32_t head_dim, int32_t block_size, int64_t num_blocks,
                                    float scale, int32_t dtype, void* workspace,
                                    size_t workspace_bytes, int32_t reuse_plan, void* stream) {
  return paged_decode_exchange(false, dst_outs, world, rank, signals, epoch, query,
                               query_token_stride, key_pool, value_pool, block_tables,
                               max_blocks_per_seq, context_lens, batch, num_q_heads, num_kv_heads,
                               head_dim, block_size, num_blocks, scale, dtype, workspace,
                               workspace_bytes, reuse_plan, stream);
}

extern "C" int ts_paged_decode_publish(void* const* dst_outs, int32_t world, int32_t rank,
                                       int32_t* const* signals, uint32_t epoch,
                                       const void* query, int64_t query_token_stride,
                                       const void* key_pool, const void* value_pool,
                                       const int32_t* block_tables, int32_t max_blocks_per_seq,
                                       const int32_t* context_lens, int32_t batch,
                                       int32_t num_q_heads, int32_t num_kv_heads,
                                       int32_t head_dim, int32_t block_size, int64_t num_blocks,
                                       float scale, int32_t dtype, void* workspace,
                                       size_t workspace_bytes, int32_t reuse_plan, void* stream) {
  return paged_decode_exchange(true, dst_outs, world, rank, signals, epoch, query,
                               query_token_stride, key_pool, value_pool, block_tables,
                               max_blocks_per_seq, context_lens, batch, num_q_heads, num_kv_heads,
                               head_dim, block_size, num_blocks, scale, dtype, workspace,
                               workspace_bytes, reuse_plan, stream);
}

// Waits (bounded) until every rank has published `epoch` into signals[0..world), then copies
// every other rank's [batch][heads_per_rank][head_dim] slice out of that rank's full buffer (read
// over NVLink) into the same place of this rank's buffer, 16 bytes a thread. On a timeout the
// CTA copies nothing and sets *status = 3.
__global__ void __launch_bounds__(256) gather_peers_kernel(uint8_t* const* fulls, int world,
                                                           int rank, const int* signals,
                                                           unsigned epoch, int batch,
                                                           int64_t row_bytes, int64_t slice_bytes,
                                                           int* status) {
  // Launched programmatically, the grid is resident while this rank's decode still runs, but it
  // polls nothing until that grid has completed: hundreds of CTAs polling the signal words would
  // keep one L2 slice busy under the decode's own traffic. Completing after it, this grid also
  // orders later work on the stream behind both.
  ts::wait_prior_grid();
  __shared__ int ready;
  if (threadIdx.x == 0) ready = 1;
  __syncthreads();
  if (threadIdx.x < world) {
    bool ok = false;
    for (long long i = 0; i < (1LL << 20) && !ok; ++i) {
      unsigned v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(signals + threadIdx.x)
                   : "memory");
      ok = int(v - epoch) >= 0;
      if (!ok) __nanosleep(256);
    }
    if (!ok) {
      ready = 0;
      atomicExch(status, 3);
    }
  }
  __syncthreads();
  if (!ready) return;
  uint8_t* mine = fulls[rank];
  const int64_t chunks = slice_bytes / 16;        // per row of one rank
  const int64_t per_rank = int64_t(batch) * chunks;
  const int64_t total = int64_t(world - 1) * per_rank;
  for (int64_t c = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; c < total;
       c += int64_t(gridDim.x) * blockDim.x) {
    const int rr = int(c / per_rank);
    const int r = rr < rank ? rr : rr + 1;
    const int64_t rem = c - int64_t(rr) * per_rank;
    const int64_t b = rem / chunks, k = rem - b * chunks;
    const int64_t off = b * row_bytes + int64_t(r) * slice_bytes + k * 16;
    *reinterpret_cast<uint4*>(mine + off) = *reinterpret_cast<const uint4*>(fulls[r] + off);
  }
}

extern "C" int ts_gather_peers(void* const* fulls, int32_t world, int32_t rank,
                               const int32_t* local_signals, uint32_t epoch, int32_t batch,
                               int32_t heads_per_rank, int32_t head_dim, int32_t dtype,
                               int32_t* status, void* stream) {
  const int es = ts::dtype_size(dtype);
  if (world < 1 || world > 64 || rank < 0 || rank >= world || epoch == 0 || batch < 0 ||
      heads_per_rank <= 0 || head_dim <= 0 || es == 0 || !fulls || !local_signals || !status)
    return ts::set_error(TS_ERR_INVALID_ARGUMENT, "gather_peers: bad arguments");
  const int64_t slice_bytes = int64_t(heads_per_rank) * head_dim * es;
  if (slice_bytes % 16)
    return ts::set_error(TS_ERR_UNSUPPORTED, "gather_peers: a rank's row slice is not 16-byte sized");
  if (!on_current_device(fulls) || !on_current_device(local_signals))
    return ts::set_error(TS_ERR_INVALID_ARGUMENT,
                         "gather_peers: fulls and signals must be in the current device's memory");
  const int64_t chunks = int64_t(world - 1) * batch * (slice_bytes / 16);
  const int grid = int(std::max<int64_t>(1, std::min<int64_t>(2 * num_sms(), (chunks + 255) / 256)));
  // Programmatic launch: resident (its launch latency hidden) while the decode before it finishes.
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(256);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(
      &cfg, gather_peers_kernel, reinterpret_cast<uint8_t* const*>(fulls), int(world), int(rank),
      reinterpret_cast<const int*>(local_signals), unsigned(epoch), int(batch),
      int64_t(slice_bytes * world), int64_t(slice_bytes), reinterpret_cast<int*>(status));
  if (e != cudaSuccess)
    return ts::set_error(static_cast<int>(e), "gather_peers: launch: %s", cudaGetErrorString(e));
  return ts::launch_status("gather_peers");
}

extern "C" int ts_wait_peers(const int32_t* local_signals, int32_t world, uint32_t epoch,
                             int32_t* status, void* stream) {
  if (world < 1 || world > 64 || epoch == 0 || !local_signals || !status)
    return ts::set_error(TS_ERR_INVALID_ARGUMENT, "wait_peers: bad arguments");
  wait_peers_kernel<<<1, 64, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const int*>(local_signals), world, epoch, reinterpret_cast<int*>(status));
  return ts::launch_status("wait_peers");
}

// Buffers shared between the ranks' processes: a plain device allocation (its own base, so its
// IPC handle maps exactly it) and CUDA IPC handles to map a peer's.
extern "C" int ts_peer_alloc(size_t bytes, void** ptr) {
  if (bytes == 0 || ptr == nullptr)
    return ts::set_error(TS_ERR_INVALID_ARGUMENT, "peer_alloc: bad arguments");
  const cudaError_t e = cudaMalloc(ptr, bytes);
  if (e != cudaSuccess)
    return ts::set_error(static_cast<int>(e), "peer_alloc: %s", cudaGetErrorString(e));
  return ts::ok();
}

extern "C" int ts_peer_free(void* ptr) {
  const cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return ts::set_error(static_cast<int>(e), "peer_free: %s", cudaGetErrorString(e));
  return ts::ok();
}

extern "C" int ts_ipc_get_handle(const void* ptr, void* handle) {
  if (ptr == nullptr || handle == nullptr)
    return ts::set_error(TS_ERR_INVALID_ARGUMENT, "ipc_get_handle: null pointer");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
  if (e != cudaSuccess)
    return ts::set_error(static_cast<int>(e), "ipc_get_handle: %s", cudaGetErrorString(e));
  memcpy(handle, &h, sizeof(h));
  return ts::ok();
}

extern "C" int ts_ipc_open(const void* handle, void** ptr) {
  if (ptr == nullptr || handle == nullptr)
    return ts::set_error(TS_ERR_INVALID_ARGUMENT, "ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess)
    return ts::set_error(static_cast<int>(e), "ipc_open: %s", cudaGetErrorString(e));
  return ts::ok();
}

extern "C" int ts_ipc_close(void* ptr) {
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) return ts::set_error(static_cast<int>(e), "ipc_close: %s", cudaGetErrorString(e));
  return ts::ok();
}
