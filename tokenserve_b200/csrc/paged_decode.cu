// K2 — paged decode attention (bf16 / fp16 KV, block_size 16, head_dim 64 or 128).
//
// Semantics: transformers 5.5.0 eager_attention_forward (models/llama/modeling_llama.py:199)
// with repeat_kv (:187) for one query token per sequence over its whole context, which is what
// tokenserve's HFBackend runs for a decode step (src/tokenserve/backends/hf.py:71), except that
// the context is read through the block table of KVCacheManager (src/tokenserve/kv_cache.py:141)
// instead of a private contiguous cache.
//
// Design (HBM-bound: every K/V byte is read exactly once):
//   * Work item = (sequence b, partition p of kPartBlocks blocks, KV head h). All G = Hq/Hkv
//     query heads of h are packed into the N dimension of the tensor-core tiles, so a KV byte
//     serves every query head that uses it (GQA packing).
//   * Every warp is an independent pipeline: it claims items from a global counter, and its
//     lane 0 streams the item's blocks with 2-D TMA loads (128-byte swizzle, no multicast) into
//     a private ring of kStages stages, each holding one block's K and V tile for head h.
//   * S^T = K Q^T and O^T += V^T P^T on mma.sync m16n8k16 (fp32 accumulate). P is split into a
//     hi and a lo half-precision part so the PV product keeps ~16 mantissa bits.
//   * Online softmax in fp32 (exp2 domain) per block; partitions of one (b, h) are merged by the
//     last warp to finish one (log-sum-exp merge), tracked with an arrival counter.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"

namespace {

constexpr int kWarps = 8;
constexpr int kBlock = 16;       // tokens per KV block (TMA box height)
constexpr int kPartBlocks = 16;  // blocks per work item (256 tokens)
constexpr float kLog2e = 1.4426950408889634f;

struct DecodeArgs {
  void* out;
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
  int* header;  // [0] = work counter, [1] = status
  int* prefix;  // [batch + 1] partitions before sequence b
  int* arrive;  // [batch * num_kv_heads]
  float* part_o;   // [slot][head_dim][NT * 8]
  float2* part_ml;  // [slot][NT * 8]
};

// Workspace layout (byte offsets), shared by the size query and the launcher.
struct WsLayout {
  size_t prefix, arrive, part_o, part_ml, total;
};

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

WsLayout ws_layout(int batch, int hkv, int hd, int max_blocks, int nt) {
  WsLayout w;
  const size_t max_parts =
      size_t(batch) * size_t((max_blocks + kPartBlocks - 1) / kPartBlocks);
  const size_t slots = max_parts * size_t(hkv);
  w.prefix = 256;
  w.arrive = w.prefix + align256(sizeof(int) * (size_t(batch) + 1));
  w.part_o = w.arrive + align256(sizeof(int) * size_t(batch) * hkv);
  w.part_ml = w.part_o + align256(sizeof(float) * slots * hd * nt * 8);
  w.total = w.part_ml + align256(sizeof(float2) * slots * nt * 8);
  return w;
}

// --------------------------------------------------------------------------- prep kernel

// One CTA: per-sequence partition counts -> exclusive prefix sums, zeroed counters, and zero
// output rows for empty contexts.
template <typename T>
__global__ void __launch_bounds__(1024) decode_prep_kernel(DecodeArgs a, int row_elems) {
  __shared__ int warp_sums[32];
  const int B = a.batch;
  const int per = (B + blockDim.x - 1) / blockDim.x;
  const int b0 = threadIdx.x * per;
  int local = 0;
  for (int i = 0; i < per; ++i) {
    const int b = b0 + i;
    if (b < B) {
      int ctx = a.context_lens[b];
      ctx = ctx < 0 ? 0 : (ctx > a.max_blocks * kBlock ? a.max_blocks * kBlock : ctx);
      local += (ctx + kPartBlocks * kBlock - 1) / (kPartBlocks * kBlock);
    }
  }
  // Block-wide exclusive scan of `local`.
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = lane < (int)(blockDim.x / 32) ? warp_sums[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += v;
    }
    warp_sums[lane] = w;  // inclusive over warps
  }
  __syncthreads();
  int run = incl - local + (warp > 0 ? warp_sums[warp - 1] : 0);
  for (int i = 0; i < per; ++i) {
    const int b = b0 + i;
    if (b < B) {
      a.prefix[b] = run;
      int ctx = a.context_lens[b];
      ctx = ctx < 0 ? 0 : (ctx > a.max_blocks * kBlock ? a.max_blocks * kBlock : ctx);
      run += (ctx + kPartBlocks * kBlock - 1) / (kPartBlocks * kBlock);
      if (ctx == 0) {
        T* o = static_cast<T*>(a.out) + int64_t(b) * row_elems;
        for (int e = 0; e < row_elems; ++e) o[e] = ts::from_float<T>(0.f);
      }
    }
  }
  if (threadIdx.x == blockDim.x - 1) a.prefix[B] = run;
  for (int i = threadIdx.x; i < B * a.num_kv_heads; i += blockDim.x) a.arrive[i] = 0;
  if (threadIdx.x == 0) {
    a.header[0] = 0;
    a.header[1] = 0;
  }
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
  static constexpr int kStages = D == 128 ? 3 : 6;
  static constexpr int kRingBytes = kStages * kStageBytes;
  static constexpr int kSmemBytes = kWarps * kRingBytes + kWarps * kStages * 16 + 1024;
};

struct ItemInfo {
  int b, h, part, nparts, ctx, nblk, part_global;
};

__device__ __forceinline__ ItemInfo decode_item(const DecodeArgs& a, int item) {
  ItemInfo it;
  it.part_global = item / a.num_kv_heads;
  it.h = item - it.part_global * a.num_kv_heads;
  int lo = 0, hi = a.batch - 1;
  while (lo < hi) {  // largest b with prefix[b] <= part_global
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(a.prefix + mid) <= it.part_global) lo = mid; else hi = mid - 1;
  }
  it.b = lo;
  it.part = it.part_global - __ldg(a.prefix + lo);
  it.nparts = __ldg(a.prefix + lo + 1) - __ldg(a.prefix + lo);
  int ctx = __ldg(a.context_lens + lo);
  it.ctx = ctx > a.max_blocks * kBlock ? a.max_blocks * kBlock : ctx;
  const int total_blk = (it.ctx + kBlock - 1) / kBlock;
  const int rem = total_blk - it.part * kPartBlocks;
  it.nblk = rem < kPartBlocks ? rem : kPartBlocks;
  return it;
}

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
  uint8_t* ring = smem + warp * G::kRingBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kWarps * G::kRingBytes) + warp * S;
  int2* meta = reinterpret_cast<int2*>(smem + kWarps * G::kRingBytes + kWarps * S * 8) + warp * S;

  if (lane == 0) {
    for (int s = 0; s < S; ++s) ts::mbar_init(&bars[s], 1);
    ts::fence_mbar_init();
  }
  __syncwarp();

  const int total_items = __ldg(a.prefix + a.batch) * a.num_kv_heads;
  int* counter = a.header;

  // ---- producer state (warp-uniform except p_table, one table entry per lane)
  int nxt = 0;
  if (lane == 0) nxt = atomicAdd(counter, 1);
  int p_item = -1, p_blk = 0, p_nblk = 0, p_h = 0, p_table = 0;
  bool p_done = false;

  auto produce = [&](int s) {
    if (!p_done && p_blk == p_nblk) {
      const int item = __shfl_sync(0xffffffffu, nxt, 0);
      if (item < total_items) {
        if (lane == 0) nxt = atomicAdd(counter, 1);
        const ItemInfo it = decode_item(a, item);
        p_item = item;
        p_h = it.h;
        p_nblk = it.nblk;
        p_blk = 0;
        p_table = lane < it.nblk
                      ? __ldg(a.block_tables + int64_t(it.b) * a.max_blocks +
                              it.part * kPartBlocks + lane)
                      : 0;
      } else {
        p_done = true;
      }
    }
    if (p_done) {
      if (lane == 0) {
        meta[s] = make_int2(-1, 0);
        ts::mbar_arrive(&bars[s]);
      }
      return;
    }
    const int phys = __shfl_sync(0xffffffffu, p_table, p_blk);
    const bool valid = phys >= 0 && int64_t(phys) < a.num_blocks;
    if (lane == 0) {
      meta[s] = make_int2(p_item, valid ? p_blk : (p_blk | 0x40000000));
      if (valid) {
        ts::mbar_arrive_expect_tx(&bars[s], G::kStageBytes);
        const int row = (phys * a.num_kv_heads + p_h) * kBlock;
        uint8_t* st = ring + s * G::kStageBytes;
#pragma unroll
        for (int hf = 0; hf < G::kHalves; ++hf) {
          ts::tma_load_2d(st + hf * 2048, &kmap, &bars[s], hf * 64, row);
          ts::tma_load_2d(st + G::kTileBytes + hf * 2048, &vmap, &bars[s], hf * 64, row);
        }
      } else {
        atomicExch(a.header + 1, 2);  // block id outside the pool: flagged, block skipped
        ts::mbar_arrive(&bars[s]);
      }
    }
    ++p_blk;
  };

#pragma unroll 1
  for (int s = 0; s < S; ++s) produce(s);

  // ---- consumer state
  int cur_item = -1;
  ItemInfo it{};
  uint32_t qf[NT][KSTEPS][2];
  float oacc[NT][MTILES][4];
  float m_run[NT][2], l_run[NT][2];

  auto start_item = [&](int item) {
    cur_item = item;
    it = decode_item(a, item);
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
      T* ob = static_cast<T*>(a.out) + (int64_t(it.b) * a.num_q_heads + it.h * a.group) * D;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const float i0 = l_run[nt][0] > 0.f ? 1.f / l_run[nt][0] : 0.f;
        const float i1 = l_run[nt][1] > 0.f ? 1.f / l_run[nt][1] : 0.f;
        const int head = nt * 8 + g;  // after the transpose a lane owns one head
#pragma unroll
        for (int mt = 0; mt < MTILES; ++mt) {
          const uint32_t lo = movmatrix_pack<Mma>(oacc[nt][mt][0] * i0, oacc[nt][mt][1] * i1);
          const uint32_t hi = movmatrix_pack<Mma>(oacc[nt][mt][2] * i0, oacc[nt][mt][3] * i1);
          if (head < a.group) {
            uint32_t* orow = reinterpret_cast<uint32_t*>(ob + int64_t(head) * D);
            orow[(mt * 16 + 2 * t) / 2] = lo;
            orow[(mt * 16 + 8 + 2 * t) / 2] = hi;
          }
        }
      }
      return;
    }
    // Partial result of one partition: unnormalised O^T, running max and sum.
    const int64_t slot = int64_t(it.part_global) * a.num_kv_heads + it.h;
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
    // Last partition of (b, h) to finish: merge all of them.
    __threadfence();
    const int hd = lane % NT8;  // fixed head per lane in the [D][NT8] layout
    const int64_t slot0 = int64_t(__ldg(a.prefix + it.b)) * a.num_kv_heads + it.h;
    float mx = -INFINITY;
    for (int p = 0; p < it.nparts; ++p)
      mx = fmaxf(mx, __ldcg(&a.part_ml[(slot0 + int64_t(p) * a.num_kv_heads) * NT8 + hd].x));
    constexpr int PER = D * NT8 / 32;
    float acc[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) acc[i] = 0.f;
    float lsum = 0.f;
    for (int p = 0; p < it.nparts; ++p) {
      const int64_t sl = slot0 + int64_t(p) * a.num_kv_heads;
      const float2 ml = __ldcg(&a.part_ml[sl * NT8 + hd]);
      const float w = ml.x == -INFINITY ? 0.f : exp2f(ml.x - mx);
      lsum += w * ml.y;
      const float* src = a.part_o + sl * D * NT8;
#pragma unroll
      for (int i = 0; i < PER; ++i) acc[i] += w * __ldcg(src + lane + 32 * i);
    }
    const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
    if (hd < a.group) {
      T* orow = static_cast<T*>(a.out) +
                (int64_t(it.b) * a.num_q_heads + it.h * a.group + hd) * D;
#pragma unroll
      for (int i = 0; i < PER; ++i) orow[(lane + 32 * i) / NT8] = ts::from_float<T>(acc[i] * inv);
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
    const int2 md = meta[s];
    if (md.x < 0) break;
    if (md.x != cur_item) {
      if (cur_item >= 0) finish_item();
      start_item(md.x);
    }
    if ((md.y & 0x40000000) == 0) {
      const uint32_t kb = ts::smem_u32(ring + s * G::kStageBytes);
      const uint32_t vb = kb + G::kTileBytes;
      const int tok0 = (it.part * kPartBlocks + md.y) * kBlock;
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
          const int chunk = (ks & 3) * 2 + (lane >> 4);
          uint32_t af[4];
          ts::ldmatrix_x4(af, kb + (ks >> 2) * 2048 + row * 128 + ((chunk ^ (row & 7)) << 4));
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
          const int cg = mt * 2 + ((lane >> 3) & 1);
          uint32_t af[4];
          ts::ldmatrix_x4_trans(
              af, vb + (cg >> 3) * 2048 + vtok * 128 + (((cg & 7) ^ (vtok & 7)) << 4));
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
    return;
  }
  if (cur_item >= 0) finish_item();
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
  const cuuint64_t dims[2] = {cuuint64_t(hd), cuuint64_t(rows)};
  const cuuint64_t strides[1] = {cuuint64_t(hd) * 2};
  const cuuint32_t box[2] = {64, kBlock};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = encode(
      map, dtype == TS_BFLOAT16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
      2, const_cast<void*>(pool), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <typename T, int D, int NT>
int launch_fast(const DecodeArgs& a, const CUtensorMap& km, const CUtensorMap& vm,
                cudaStream_t s) {
  using G = Geometry<D>;
  auto kern = paged_decode_kernel<T, D, NT>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, G::kSmemBytes);
  decode_prep_kernel<T><<<1, 1024, 0, s>>>(a, a.num_q_heads * D);
  kern<<<num_sms(), kWarps * 32, G::kSmemBytes, s>>>(km, vm, a);
  return ts::launch_status("paged_decode");
}

// Whether the tensor-core decode kernel covers these arguments.
bool fast_path(int hq, int hkv, int hd, int bs, int dtype, int64_t num_blocks, const void* kp,
               const void* vp, const void* q, int64_t q_stride, const void* out) {
  if (dtype != TS_BFLOAT16 && dtype != TS_FLOAT16) return false;
  if (bs != kBlock || (hd != 64 && hd != 128)) return false;
  if (hkv <= 0 || hq % hkv != 0 || hq / hkv > 16) return false;
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
  return ws_layout(batch, num_kv_heads, head_dim, max_blocks_per_seq, nt).total;
}

extern "C" int ts_paged_decode(void* out, const void* query, int64_t query_token_stride,
                               const void* key_pool, const void* value_pool,
                               const int32_t* block_tables, int32_t max_blocks_per_seq,
                               const int32_t* context_lens, int32_t batch, int32_t num_q_heads,
                               int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                               int64_t num_blocks, float scale, int32_t dtype, void* workspace,
                               size_t workspace_bytes, void* stream) {
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
  const int group = num_q_heads / num_kv_heads;
  const int nt = group > 8 ? 2 : 1;
  const WsLayout w = ws_layout(batch, num_kv_heads, head_dim, max_blocks_per_seq, nt);
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
  a.header = reinterpret_cast<int*>(ws);
  a.prefix = reinterpret_cast<int*>(ws + w.prefix);
  a.arrive = reinterpret_cast<int*>(ws + w.arrive);
  a.part_o = reinterpret_cast<float*>(ws + w.part_o);
  a.part_ml = reinterpret_cast<float2*>(ws + w.part_ml);
#define TS_FAST(T)                                                             \
  if (head_dim == 128)                                                         \
    return nt == 1 ? launch_fast<T, 128, 1>(a, km, vm, s)                      \
                   : launch_fast<T, 128, 2>(a, km, vm, s);                     \
  return nt == 1 ? launch_fast<T, 64, 1>(a, km, vm, s) : launch_fast<T, 64, 2>(a, km, vm, s);
  if (dtype == TS_BFLOAT16) {
    TS_FAST(__nv_bfloat16)
  }
  TS_FAST(__half)
#undef TS_FAST
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
  const int group = num_q_heads / num_kv_heads;
  const int nt = group > 8 ? 2 : 1;
  const WsLayout w = ws_layout(batch, num_kv_heads, head_dim, max_blocks_per_seq, nt);
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
  a.header = reinterpret_cast<int*>(ws);
  a.prefix = reinterpret_cast<int*>(ws + w.prefix);
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
