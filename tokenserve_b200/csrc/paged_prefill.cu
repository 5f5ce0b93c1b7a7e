// K3 — paged chunked-prefill attention (causal over cached prefix blocks + the new chunk).
//
// Semantics: transformers 5.5.0 eager_attention_forward (models/llama/modeling_llama.py:199)
// with a causal mask, as HFBackend runs it for a multi-token step
// (src/tokenserve/backends/hf.py:71), except that the prefix comes from cached blocks of the
// paged pool (src/tokenserve/kv_cache.py:159-177) instead of being recomputed. Query row j of a
// sequence whose step ends at context_lens[s] sits at position context_lens[s] - q_len + j.
//
// bf16/fp16, head_dim 128, block 16, G = Hq/Hkv in {1,2,4,8,16}: tcgen05 tensor-core kernel.
//   * CTA = (sequence, KV head, pair of query tiles). A tile's 128 rows are 128/G query tokens x
//     the G query heads of the KV head (GQA packing), so each K/V tile feeds all G heads, and
//     both tiles of the pair share every K/V tile they need.
//   * warp 8 (producer): Q tiles by one 3-D TMA box per 64-column half, then K/V tiles of 128
//     tokens (8 blocks, gathered through the block table with 2-D TMA boxes, 128-byte swizzle,
//     no multicast; lane b issues block b's boxes, its table entry read one tile ahead) into a
//     3-stage K ring and a 2-stage V ring: a K stage is released after the last QK that reads it,
//     a V stage after the last PV, so K loads run further ahead.
//   * warp 9 (one lane): tcgen05.mma S_x = Q_x K^T (M=N=K=128, both K-major) into tile x's TMEM
//     S, then O_x += P_x V with P read from TMEM (written over S as two half-precision parts,
//     P_hi + P_lo, so the product keeps ~16 bits of P) and V MN-major, in the order PV_A(j),
//     QK_A(j+1), PV_B(j), QK_B(j+1): one tile's softmax overlaps the other's MMAs.
//   * warps 0-3 / 4-7 (one warpgroup per query tile, thread = row = TMEM lane): online softmax
//     in fp32 (exp2 domain, causal mask only on diagonal tiles, stale max kept unless exceeded by
//     2^8 so O is rarely rescaled), P back to TMEM, O rescale in TMEM, and the epilogue.
// Other shapes and fp32 use the CUDA-core kernel in attention_portable.cu.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "tcgen05.cuh"

namespace ts {
int paged_attention_portable(void* out, const void* query, int64_t q_stride, const void* kp,
                             const void* vp, const int32_t* bt, int max_blocks,
                             const int32_t* qsl, const int32_t* cl, int num_seqs, int num_rows,
                             int hq, int hkv, int hd, int bs, int64_t nb, float scale, int dtype,
                             cudaStream_t s);
}

namespace {

constexpr int kRows = 128;                   // query rows per tile (M)
constexpr int kKvTile = 128;                 // KV tokens per tile (N of QK, K of PV)
constexpr int kBlock = 16;                   // tokens per KV block
constexpr int kHalfBytes = 128 * 128;        // 128 rows x 128 bytes (64 columns)
constexpr int kTileBytes = 2 * kHalfBytes;   // 128 x 128 16-bit elements
constexpr int kQTiles = 2;                   // query tiles per CTA (ping-pong)
constexpr int kKStages = 3;                  // K ring (freed after the last QK of a tile)
constexpr int kVStages = 2;                  // V ring (freed after the last PV of a tile)
constexpr int kSmemBytes = (kQTiles + kKStages + kVStages) * kTileBytes + 256 + 1024;
// Warps 0..4*kQTiles-1: softmax, one warpgroup per query tile; then the producer and the MMA
// warp. With 10 warps one SM sub-partition hosts 3 of them, so a thread may use at most
// 16384 / 96 = 170 registers: the kernel is capped at 168.
constexpr int kThreads = 32 * (4 * kQTiles + 2);
constexpr int kMaxRegs = 168;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleSlack = 8.f;  // keep a stale row max unless exceeded by 2^8
constexpr uint32_t kTmemCols = 512;  // S_A [0,128), S_B [128,256), O_A [256,384), O_B [384,512)

struct PrefillArgs {
  void* out;
  const int32_t* block_tables;
  const int32_t* qsl;
  const int32_t* context_lens;
  int max_blocks;
  int num_q_heads;
  int num_kv_heads;
  int group;
  int tq;  // query tokens per tile = 128 / group
  float scale_log2;
};

struct Bars {
  uint64_t q_full, k_full[kKStages], k_empty[kKStages], v_full[kVStages], v_empty[kVStages];
  uint64_t s_full[kQTiles], p_full[kQTiles], pv_done[kQTiles];
  uint32_t tmem;
  int abort;
};

// Bounded wait that also gives up as soon as another role has aborted.
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t phase, volatile int* abort) {
  for (long long i = 0; i < ts::kMaxSpins; ++i) {
    if (ts::mbar_try_wait(bar, phase)) return true;
    if ((i & 255) == 255 && *abort) return false;
  }
  *abort = 1;
  return false;
}

__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <bool BF16>
__global__ void __maxnreg__(kMaxRegs)
    paged_prefill_tc_kernel(const __grid_constant__ CUtensorMap qmap,
                            const __grid_constant__ CUtensorMap kmap,
                            const __grid_constant__ CUtensorMap vmap, const PrefillArgs a) {
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  using Mma = ts::MmaOp<T>;
  const int pair = blockIdx.x, h = blockIdx.y, seq = blockIdx.z;
  const int q0 = a.qsl[seq];
  const int q_len = a.qsl[seq + 1] - q0;
  const int tile0 = pair * kQTiles;  // query tiles tile0 (A) and tile0 + 1 (B)
  if (tile0 * a.tq >= q_len) return;
  int ctx = a.context_lens[seq];
  if (ctx > a.max_blocks * kBlock) ctx = a.max_blocks * kBlock;
  const int p0 = ctx - q_len;
  if (p0 < 0) return;
  // KV tiles each query tile needs (causal), 0 for an empty tile.
  int n_t[kQTiles];
  int n_kv_max = 0;
#pragma unroll
  for (int x = 0; x < kQTiles; ++x) {
    const int first = (tile0 + x) * a.tq;
    if (first >= q_len) {
      n_t[x] = 0;
    } else {
      const int n_kv = p0 + min(q_len, first + a.tq);
      n_t[x] = (n_kv + kKvTile - 1) / kKvTile;
      n_kv_max = max(n_kv_max, n_kv);
    }
  }
  const int n_max = (n_kv_max + kKvTile - 1) / kKvTile;
  const int total_blk = (n_kv_max + kBlock - 1) / kBlock;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = ts::smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023) & ~1023u) - raw);
  auto sQ = [&](int x) { return smem + x * kTileBytes; };
  auto sK = [&](int st) { return smem + (kQTiles + st) * kTileBytes; };
  auto sV = [&](int st) { return smem + (kQTiles + kKStages + st) * kTileBytes; };
  Bars* bars = reinterpret_cast<Bars*>(smem + (kQTiles + kKStages + kVStages) * kTileBytes);
  volatile int* abort = &bars->abort;

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    ts::mbar_init(&bars->q_full, 1);
    for (int i = 0; i < kKStages; ++i) {
      ts::mbar_init(&bars->k_full[i], 1);
      ts::mbar_init(&bars->k_empty[i], 1);
    }
    for (int i = 0; i < kVStages; ++i) {
      ts::mbar_init(&bars->v_full[i], 1);
      ts::mbar_init(&bars->v_empty[i], 1);
    }
    for (int x = 0; x < kQTiles; ++x) {
      ts::mbar_init(&bars->s_full[x], 1);
      ts::mbar_init(&bars->p_full[x], 128);
      ts::mbar_init(&bars->pv_done[x], 1);
    }
    bars->abort = 0;
    ts::fence_mbar_init();
  }
  if (warp == 0) {
    ts::tc::tmem_alloc(&bars->tmem, kTmemCols);
    ts::tc::tmem_relinquish();
  }
  ts::tc::fence_before_sync();
  __syncthreads();
  ts::tc::fence_after_sync();
  const uint32_t tmem = bars->tmem;
  const int G = a.group;
  const int producer_warp = 4 * kQTiles, mma_warp = 4 * kQTiles + 1;

  if (warp == producer_warp) {
    // ------------------------------------------------------------ producer (TMA)
    const int32_t* table = a.block_tables + int64_t(seq) * a.max_blocks;
    if (lane == 0) {
      ts::mbar_arrive_expect_tx(&bars->q_full, kQTiles * kTileBytes);
      for (int x = 0; x < kQTiles; ++x)
        for (int hf = 0; hf < 2; ++hf)
          ts::tc::tma_load_3d(sQ(x) + hf * kHalfBytes, &qmap, &bars->q_full, hf * 64, h * G,
                              q0 + (tile0 + x) * a.tq);
    }
    // K tile j goes out as soon as its stage is free (after the last QK of tile j - kKStages);
    // V tile j one step later (its first use, PV, comes after the softmax of tile j).
    // Lane b < 8 owns block b of a KV tile: it holds that block's pool row, read from the block
    // table one tile ahead (so the table load's latency is off the issue path), and issues the
    // block's two TMA boxes; a tile costs one warp-wide issue instead of 16 serial ones.
    constexpr int kBpt = kKvTile / kBlock;
    auto table_row = [&](int j) -> int {
      const int b = j * kBpt + lane;
      return (lane < kBpt && j < n_max && b < total_blk)
                 ? (__ldg(table + b) * a.num_kv_heads + h) * kBlock
                 : -1;
    };
    auto load = [&](bool is_k, int j, int row) -> bool {
      const int nst = is_k ? kKStages : kVStages;
      const int st = j % nst;
      uint64_t* full = is_k ? &bars->k_full[st] : &bars->v_full[st];
      uint64_t* empty = is_k ? &bars->k_empty[st] : &bars->v_empty[st];
      if (j >= nst && !wait_bar(empty, ((j - nst) / nst) & 1, abort)) return false;
      const int nb = min(kBpt, total_blk - j * kBpt);  // lanes with row >= 0
      if (lane == 0) ts::mbar_arrive_expect_tx(full, nb * 2 * 2048);
      __syncwarp();
      if (row >= 0) {
        uint8_t* dst = (is_k ? sK(st) : sV(st)) + lane * 2048;
        const void* map = is_k ? static_cast<const void*>(&kmap) : static_cast<const void*>(&vmap);
        ts::tma_load_2d(dst, map, full, 0, row);
        ts::tma_load_2d(dst + kHalfBytes, map, full, 64, row);
      }
      return true;
    };
    int issued_k = 0, issued_v = 0;
    int row_k = table_row(0), row_v = -1;
    for (int j = 0; j <= n_max; ++j) {
      const int row_next = table_row(j + 1);
      if (j < n_max) {
        if (!load(true, j, row_k)) break;
        issued_k = j + 1;
      }
      if (j >= 1) {
        if (!load(false, j - 1, row_v)) break;
        issued_v = j;
      }
      row_v = row_k;
      row_k = row_next;
    }
    if (*abort && lane == 0) {
      // Let the copies still in flight land before shared memory is released.
      for (int j = max(0, issued_k - kKStages); j < issued_k; ++j)
        ts::mbar_wait_bounded(&bars->k_full[j % kKStages], (j / kKStages) & 1);
      for (int j = max(0, issued_v - kVStages); j < issued_v; ++j)
        ts::mbar_wait_bounded(&bars->v_full[j % kVStages], (j / kVStages) & 1);
      ts::mbar_wait_bounded(&bars->q_full, 0);
    }
  } else if (warp == mma_warp) {
    // ------------------------------------------------------------ MMA issuer (one lane)
    // Order per KV tile j: PV_A(j), QK_A(j+1), PV_B(j), QK_B(j+1), so the softmax of one query
    // tile overlaps the tensor-core work of the other.
    if (lane == 0) {
      constexpr uint32_t idesc_qk = ts::tc::idesc_f16(BF16, kRows, kKvTile, false);
      constexpr uint32_t idesc_pv = ts::tc::idesc_f16(BF16, kRows, 128, true);
      int last_pv[kQTiles];
      for (int x = 0; x < kQTiles; ++x) last_pv[x] = -1;
      // The last query tile to use KV tile j releases its K (after QK) and V (after PV).
      auto last_user = [&](int j) { return j < n_t[kQTiles - 1] ? kQTiles - 1 : 0; };
      // Shared-memory descriptors are built once; a tile or K step only adds its byte offset
      // / 16 to the start-address field (every address is below 256 KB, so it never carries).
      const uint64_t dq0 = ts::tc::smem_desc_sw128(ts::smem_u32(sQ(0)), 16, 1024);
      const uint64_t dk0 = ts::tc::smem_desc_sw128(ts::smem_u32(sK(0)), 16, 1024);
      const uint64_t dv0 = ts::tc::smem_desc_sw128(ts::smem_u32(sV(0)), kHalfBytes, 1024);
      auto issue_qk = [&](int x, int j) -> bool {
        const int st = j % kKStages;
        if (!wait_bar(&bars->k_full[st], (j / kKStages) & 1, abort)) return false;
        ts::tc::fence_after_sync();
        const uint64_t dq = dq0 + uint64_t((x * kTileBytes) >> 4);
        const uint64_t dk = dk0 + uint64_t((st * kTileBytes) >> 4);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off16 = ((kk >> 2) * kHalfBytes + (kk & 3) * 32) >> 4;
          ts::tc::mma_ss(tmem + x * 128, dq + off16, dk + off16, idesc_qk, kk > 0);
        }
        ts::tc::commit(&bars->s_full[x]);
        if (x == last_user(j) && j + kKStages < n_max) ts::tc::commit(&bars->k_empty[st]);
        return true;
      };
      bool ok = wait_bar(&bars->q_full, 0, abort);
      for (int x = 0; ok && x < kQTiles; ++x)
        if (n_t[x] > 0) ok = issue_qk(x, 0);
      for (int j = 0; ok && j < n_max; ++j) {
        const int st = j % kVStages;
        for (int x = 0; ok && x < kQTiles; ++x) {
          if (j >= n_t[x]) continue;
          if (!wait_bar(&bars->p_full[x], j & 1, abort) ||
              !wait_bar(&bars->v_full[st], (j / kVStages) & 1, abort)) {
            ok = false;
            break;
          }
          ts::tc::fence_after_sync();
          const uint64_t dv = dv0 + uint64_t((st * kTileBytes) >> 4);
          // O_x += P_hi V + P_lo V (P_hi in S columns [0, 64), P_lo in [64, 128)).
#pragma unroll
          for (int part = 0; part < 2; ++part)
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
              ts::tc::mma_ts(tmem + 256 + x * 128, tmem + x * 128 + part * 64 + kk * 8,
                             dv + uint64_t((kk * 2048) >> 4), idesc_pv,
                             j > 0 || part > 0 || kk > 0);
          ts::tc::commit(&bars->pv_done[x]);
          if (x == last_user(j) && j + kVStages < n_max) ts::tc::commit(&bars->v_empty[st]);
          last_pv[x] = j;
          if (j + 1 < n_t[x] && !issue_qk(x, j + 1)) ok = false;
        }
      }
      if (*abort)
        for (int x = 0; x < kQTiles; ++x)
          if (last_pv[x] >= 0) ts::mbar_wait_bounded(&bars->pv_done[x], last_pv[x] & 1);
    }
  } else if (warp < 4 * kQTiles) {
    // ------------------------------------------------------------ softmax / epilogue
    const int x = warp / 4;                 // query tile of this warpgroup
    const int r = threadIdx.x - 128 * x;    // tile row == TMEM lane
    const int n_x = n_t[x];
    const int i = r / G, g = r - (r / G) * G;
    const int qi = (tile0 + x) * a.tq + i;
    const bool row_valid = qi < q_len;
    const int pos = p0 + (row_valid ? qi : q_len - 1);
    const uint32_t lane_base = tmem + (uint32_t((warp & 3) * 32) << 16);
    const uint32_t s_col = x * 128, o_col = 256 + x * 128;
    // The first query tile to use the CTA's last KV tile clears its rows past the last key.
    int zero_tile = -1;
    for (int y = kQTiles - 1; y >= 0; --y)
      if (n_t[y] == n_max) zero_tile = y;
    const float sl = a.scale_log2;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = n_x > 0;
    for (int j = 0; ok && j < n_x; ++j) {
      if (!wait_bar(&bars->s_full[x], j & 1, abort)) {
        ok = false;
        break;
      }
      ts::tc::fence_after_sync();
      const int limit = pos - j * kKvTile;  // columns c <= limit are visible
      const bool full_tile = limit >= kKvTile - 1;
      // One TMEM round trip for the whole row: four 32-column loads, one wait; columns past
      // the causal limit become -inf.
      uint32_t sr[128];
      auto load_s = [&]() {
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          uint32_t (&chunk)[32] = *reinterpret_cast<uint32_t(*)[32]>(sr + 32 * c4);
          ts::tc::tmem_ld32(lane_base + s_col + c4 * 32, chunk);
        }
        ts::tc::wait_ld();
        if (!full_tile) {
#pragma unroll
          for (int c = 0; c < 128; ++c)
            if (c > limit) sr[c] = __float_as_uint(-INFINITY);
        }
      };
      // P = exp2(s * scale - m_run) as two half-precision parts, P = P_hi + P_lo with
      // P_lo = round(P - P_hi): the PV product then keeps ~16 mantissa bits of P instead of 8
      // (a bf16 P alone leaves errors near 2e-3 of max|O| at 1,536-token contexts). Registers
      // sr[c..c+3] of the four scores just read take P_hi of (c, c+1), (c+2, c+3) and then
      // P_lo of the same pairs. Also the row sum and the largest exponent seen (xm), which
      // the exponentials do not wait on.
      float sum0, sum1, xm;
      auto exp_pass = [&]() {
        sum0 = 0.f;
        sum1 = 0.f;
        float xa = -INFINITY, xb = -INFINITY;
#pragma unroll
        for (int c = 0; c < 128; c += 4) {
          const float x0 = fmaf(__uint_as_float(sr[c]), sl, -m_run);
          const float x1 = fmaf(__uint_as_float(sr[c + 1]), sl, -m_run);
          const float x2 = fmaf(__uint_as_float(sr[c + 2]), sl, -m_run);
          const float x3 = fmaf(__uint_as_float(sr[c + 3]), sl, -m_run);
          xa = max3f(xa, x0, x1);
          xb = max3f(xb, x2, x3);
          const float p0 = ex2(x0), p1 = ex2(x1), p2 = ex2(x2), p3 = ex2(x3);
          sum0 += p0 + p2;
          sum1 += p1 + p3;
          const uint32_t h01 = Mma::pack(p0, p1), h23 = Mma::pack(p2, p3);
          const float2 f01 = Mma::unpack(h01), f23 = Mma::unpack(h23);
          sr[c] = h01;
          sr[c + 1] = h23;
          sr[c + 2] = Mma::pack(p0 - f01.x, p1 - f01.y);
          sr[c + 3] = Mma::pack(p2 - f23.x, p3 - f23.y);
        }
        xm = fmaxf(xa, xb);
      };
      load_s();
      float corr = 1.f;
      if (j == 0) {
        // First tile: the exact row max (column 0 is always visible, so it is finite).
        float mx = -INFINITY;
#pragma unroll
        for (int c = 0; c < 128; c += 2)
          mx = max3f(mx, __uint_as_float(sr[c]), __uint_as_float(sr[c + 1]));
        m_run = mx * sl;
      }
      exp_pass();
      // Lazy rescaling: the running max is kept while no exponent exceeds it by more than
      // kRescaleSlack (P <= 2^8). Rows past that take the new max and recompute the tile.
      if (j > 0 && __any_sync(0xffffffffu, xm > kRescaleSlack)) {
        load_s();
        if (xm > kRescaleSlack) {
          corr = ex2(-xm);
          m_run += xm;
        }
        exp_pass();
      }
      // P_hi over S columns [0, 64), P_lo over [64, 128): word w of part k (pair w of the row)
      // sits in sr[4 * (w / 2) + 2 * k + w % 2].
#pragma unroll
      for (int c2 = 0; c2 < 4; ++c2) {
        const int part = c2 / 2, w0 = (c2 % 2) * 32;
        uint32_t chunk[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) chunk[i] = sr[4 * ((w0 + i) / 2) + 2 * part + (w0 + i) % 2];
        ts::tc::tmem_st32(lane_base + s_col + c2 * 32, chunk);
      }
      ts::tc::wait_st();
      l_run = l_run * corr + (sum0 + sum1);
      if (j > 0) {
        if (!wait_bar(&bars->pv_done[x], (j - 1) & 1, abort)) {
          ok = false;
          break;
        }
        ts::tc::fence_after_sync();
        if (__any_sync(0xffffffffu, corr != 1.f)) {
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4) {
            uint32_t rr[32];
            ts::tc::tmem_ld32(lane_base + o_col + c4 * 32, rr);
            ts::tc::wait_ld();
#pragma unroll
            for (int c = 0; c < 32; ++c) rr[c] = __float_as_uint(__uint_as_float(rr[c]) * corr);
            ts::tc::tmem_st32(lane_base + o_col + c4 * 32, rr);
          }
          ts::tc::wait_st();
        }
      }
      if (x == zero_tile && j == n_max - 1 && j * kKvTile + kKvTile > n_kv_max) {
        // Rows past the last visible key hold stale or unwritten data: zero them so that
        // P = 0 times V stays 0.
        const int vst = j % kVStages;
        if (!wait_bar(&bars->v_full[vst], (j / kVStages) & 1, abort)) {
          ok = false;
          break;
        }
        if (j * kKvTile + r >= n_kv_max) {
          uint4* v0 = reinterpret_cast<uint4*>(sV(vst) + r * 128);
          uint4* v1 = reinterpret_cast<uint4*>(sV(vst) + kHalfBytes + r * 128);
#pragma unroll
          for (int c = 0; c < 8; ++c) v0[c] = v1[c] = make_uint4(0, 0, 0, 0);
        }
        ts::fence_proxy_async_smem();
      }
      ts::tc::fence_before_sync();
      ts::mbar_arrive(&bars->p_full[x]);
    }
    if (ok && wait_bar(&bars->pv_done[x], (n_x - 1) & 1, abort)) {
      ts::tc::fence_after_sync();
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      T* orow = static_cast<T*>(a.out) +
                (int64_t(q0 + qi) * a.num_q_heads + h * G + g) * 128;
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) {
        uint32_t rr[32];
        ts::tc::tmem_ld32(lane_base + o_col + c4 * 32, rr);
        ts::tc::wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int c = 0; c < 16; ++c)
          pk[c] = Mma::pack(__uint_as_float(rr[2 * c]) * inv, __uint_as_float(rr[2 * c + 1]) * inv);
        if (row_valid) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c4 * 32);
#pragma unroll
          for (int c = 0; c < 4; ++c)
            dst[c] = make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
        }
      }
    }
  }
  ts::tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    ts::tc::fence_after_sync();
    ts::tc::tmem_dealloc(tmem, kTmemCols);
  }
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

CUtensorMapDataType tma_type(int dtype) {
  return dtype == TS_BFLOAT16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
}

bool encode_pool_map(CUtensorMap* map, const void* pool, int64_t rows, int dtype) {
  const cuuint64_t dims[2] = {128, cuuint64_t(rows)};
  const cuuint64_t strides[1] = {256};
  const cuuint32_t box[2] = {64, kBlock};
  const cuuint32_t estr[2] = {1, 1};
  return get_encode()(map, tma_type(dtype), 2, const_cast<void*>(pool), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Query rows [tokens][heads][128] with a token stride; box = (64 columns, G heads, 128/G tokens).
bool encode_query_map(CUtensorMap* map, const void* q, int64_t tokens, int hq, int64_t q_stride,
                      int group, int dtype) {
  const cuuint64_t dims[3] = {128, cuuint64_t(hq), cuuint64_t(tokens)};
  const cuuint64_t strides[2] = {256, cuuint64_t(q_stride) * 2};
  const cuuint32_t box[3] = {64, cuuint32_t(group), cuuint32_t(kRows / group)};
  const cuuint32_t estr[3] = {1, 1, 1};
  return get_encode()(map, tma_type(dtype), 3, const_cast<void*>(q), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool tc_path(int hq, int hkv, int hd, int bs, int dtype, int64_t num_blocks, const void* kp,
             const void* vp, const void* q, int64_t q_stride, const void* out, int num_seqs) {
  if (dtype != TS_BFLOAT16 && dtype != TS_FLOAT16) return false;
  if (hd != 128 || bs != kBlock || hkv <= 0 || hq % hkv) return false;
  const int g = hq / hkv;
  if (g != 1 && g != 2 && g != 4 && g != 8 && g != 16) return false;
  if (num_blocks * hkv * kBlock >= (int64_t(1) << 31) || num_seqs > 65535 || hkv > 65535)
    return false;
  if ((reinterpret_cast<uint64_t>(kp) | reinterpret_cast<uint64_t>(vp) |
       reinterpret_cast<uint64_t>(q) | reinterpret_cast<uint64_t>(out)) % 16)
    return false;
  if ((q_stride * 2) % 16) return false;
  return get_encode() != nullptr;
}

}  // namespace

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
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (!tc_path(num_q_heads, num_kv_heads, head_dim, block_size, dtype, num_blocks, key_pool,
               value_pool, query, query_token_stride, out, num_seqs))
    return ts::paged_attention_portable(out, query, query_token_stride, key_pool, value_pool,
                                        block_tables, max_blocks_per_seq, query_start_loc,
                                        context_lens, num_seqs, num_query_tokens, num_q_heads,
                                        num_kv_heads, head_dim, block_size, num_blocks, scale,
                                        dtype, s);
  const int group = num_q_heads / num_kv_heads;
  CUtensorMap qm, km, vm;
  const int64_t rows = num_blocks * num_kv_heads * kBlock;
  if (!encode_query_map(&qm, query, num_query_tokens, num_q_heads, query_token_stride, group,
                        dtype) ||
      !encode_pool_map(&km, key_pool, rows, dtype) || !encode_pool_map(&vm, value_pool, rows, dtype))
    return ts::set_error(TS_ERR_INVALID_ARGUMENT, "paged_prefill: cannot encode TMA maps");
  PrefillArgs a;
  a.out = out;
  a.block_tables = block_tables;
  a.qsl = query_start_loc;
  a.context_lens = context_lens;
  a.max_blocks = max_blocks_per_seq;
  a.num_q_heads = num_q_heads;
  a.num_kv_heads = num_kv_heads;
  a.group = group;
  a.tq = kRows / group;
  a.scale_log2 = scale * kLog2e;
  const int tiles = (max_query_len + a.tq - 1) / a.tq;
  if (tiles == 0) return ts::ok();
  dim3 grid((tiles + kQTiles - 1) / kQTiles, num_kv_heads, num_seqs);
  auto kern = dtype == TS_BFLOAT16 ? paged_prefill_tc_kernel<true> : paged_prefill_tc_kernel<false>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  kern<<<grid, kThreads, kSmemBytes, s>>>(qm, km, vm, a);
  return ts::launch_status("paged_prefill");
}
