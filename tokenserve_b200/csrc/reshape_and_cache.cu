// K1 — scatter the step's new K/V rows into the paged pool through the slot mapping.
//
// Semantics follow tokenserve BatchItem.slot_mapping (src/tokenserve/backends/base.py:40-45)
// and the write half of SimulatedBackend._write_and_verify
// (src/tokenserve/backends/simulated.py:156-160): token t of the step goes to physical slot
// slot_mapping[t] = block * block_size + offset, i.e. row (block, head, offset) of the pool
// [num_blocks][num_kv_heads][block_size][head_dim].
//
// HBM-bound byte copy: each thread moves one 16-byte vector (when alignment allows) of one
// (token, head) row for both K and V, so a warp reads and writes whole 512-byte spans.
#include "common.cuh"

namespace {

template <int VEC>
struct VecType;
template <>
struct VecType<16> {
  using T = uint4;
};
template <>
struct VecType<8> {
  using T = uint2;
};
template <>
struct VecType<4> {
  using T = uint32_t;
};
template <>
struct VecType<2> {
  using T = uint16_t;
};

template <int VEC>
__global__ void __launch_bounds__(256) reshape_and_cache_kernel(
    const uint8_t* __restrict__ key, const uint8_t* __restrict__ value, int64_t key_stride_b,
    int64_t value_stride_b, uint8_t* __restrict__ key_pool, uint8_t* __restrict__ value_pool,
    const int64_t* __restrict__ slot_mapping, int64_t num_tokens, int heads, int row_bytes,
    int block_size, int64_t num_slots, const int32_t* __restrict__ tags,
    int32_t* __restrict__ tag_pool, int32_t* __restrict__ error_flag) {
  // A decode's prep kernel launched programmatically after this one may start now: it waits
  // for this grid on the device before it reads anything.
  ts::allow_dependents();
  using V = typename VecType<VEC>::T;
  const int vec_per_row = row_bytes / VEC;
  const int vec_per_tok = heads * vec_per_row;
  for (int64_t t = blockIdx.x; t < num_tokens; t += gridDim.x) {
    const int64_t slot = __ldg(slot_mapping + t);
    if (slot < 0) continue;  // padding token
    if (slot >= num_slots) {
      if (error_flag != nullptr && threadIdx.x == 0) atomicExch(error_flag, 1);
      continue;
    }
    const int64_t blk = slot / block_size;
    const int64_t off = slot - blk * block_size;
    if (tag_pool != nullptr && threadIdx.x == 0) tag_pool[slot] = __ldg(tags + t);
    const uint8_t* ksrc = key + t * key_stride_b;
    const uint8_t* vsrc = value + t * value_stride_b;
    for (int j = threadIdx.x; j < vec_per_tok; j += blockDim.x) {
      const int h = j / vec_per_row;
      const int c = j - h * vec_per_row;
      const int64_t dst = ((blk * heads + h) * block_size + off) * row_bytes + int64_t(c) * VEC;
      const int64_t src = int64_t(h) * row_bytes + int64_t(c) * VEC;
      const V kv = __ldg(reinterpret_cast<const V*>(ksrc + src));
      const V vv = __ldg(reinterpret_cast<const V*>(vsrc + src));
      *reinterpret_cast<V*>(key_pool + dst) = kv;
      *reinterpret_cast<V*>(value_pool + dst) = vv;
    }
  }
}

int pick_vec(int esize, std::initializer_list<uint64_t> values) {
  for (int v : {16, 8, 4, 2}) {
    if (v < esize) break;
    bool fits = true;
    for (uint64_t x : values) fits = fits && (x % v == 0);
    if (fits) return v;
  }
  return 0;
}

}  // namespace

extern "C" int ts_reshape_and_cache(const void* key, const void* value, int64_t key_token_stride,
                                    int64_t value_token_stride, void* key_pool, void* value_pool,
                                    const int64_t* slot_mapping, int64_t num_tokens,
                                    int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                                    int64_t num_blocks, int32_t dtype, const int32_t* token_tags,
                                    int32_t* tag_pool, int32_t* error_flag, void* stream) {
  const int es = ts::dtype_size(dtype);
  if (es == 0) return ts::set_error(TS_ERR_INVALID_ARGUMENT, "reshape_and_cache: bad dtype %d", dtype);
  if (num_tokens < 0 || num_kv_heads <= 0 || head_dim <= 0 || block_size <= 0 || num_blocks <= 0)
    return ts::set_error(TS_ERR_INVALID_ARGUMENT,
                         "reshape_and_cache: bad sizes (tokens %lld, heads %d, head_dim %d, "
                         "block_size %d, blocks %lld)",
                         (long long)num_tokens, num_kv_heads, head_dim, block_size,
                         (long long)num_blocks);
  if (num_tokens == 0) return ts::ok();
  if (!key || !value || !key_pool || !value_pool || !slot_mapping)
    return ts::set_error(TS_ERR_INVALID_ARGUMENT, "reshape_and_cache: null pointer");
  if ((token_tags == nullptr) != (tag_pool == nullptr))
    return ts::set_error(TS_ERR_INVALID_ARGUMENT,
                         "reshape_and_cache: token_tags and tag_pool go together");
  if (key_token_stride < int64_t(num_kv_heads) * head_dim ||
      value_token_stride < int64_t(num_kv_heads) * head_dim)
    return ts::set_error(TS_ERR_INVALID_ARGUMENT,
                         "reshape_and_cache: token stride smaller than heads * head_dim");
  const int row_bytes = head_dim * es;
  const int vec = pick_vec(es, {reinterpret_cast<uint64_t>(key), reinterpret_cast<uint64_t>(value),
                                reinterpret_cast<uint64_t>(key_pool),
                                reinterpret_cast<uint64_t>(value_pool),
                                uint64_t(key_token_stride * es), uint64_t(value_token_stride * es),
                                uint64_t(row_bytes)});
  if (vec == 0)
    return ts::set_error(TS_ERR_MISALIGNED, "reshape_and_cache: pointers not element-aligned");
  const int vec_per_tok = num_kv_heads * (row_bytes / vec);
  const int threads = vec_per_tok >= 256 ? 256 : ((vec_per_tok + 31) / 32) * 32;
  const int64_t grid64 = num_tokens < 65535 * 8 ? num_tokens : 65535 * 8;
  const unsigned grid = static_cast<unsigned>(grid64);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t num_slots = num_blocks * block_size;
  auto k8 = static_cast<const uint8_t*>(key);
  auto v8 = static_cast<const uint8_t*>(value);
  auto kp = static_cast<uint8_t*>(key_pool);
  auto vp = static_cast<uint8_t*>(value_pool);
  const int64_t ksb = key_token_stride * es, vsb = value_token_stride * es;
#define TS_LAUNCH(V)                                                                         \
  reshape_and_cache_kernel<V><<<grid, threads, 0, s>>>(k8, v8, ksb, vsb, kp, vp, slot_mapping, \
                                                       num_tokens, num_kv_heads, row_bytes,   \
                                                       block_size, num_slots, token_tags,     \
                                                       tag_pool, error_flag)
  switch (vec) {
    case 16: TS_LAUNCH(16); break;
    case 8: TS_LAUNCH(8); break;
    case 4: TS_LAUNCH(4); break;
    default: TS_LAUNCH(2); break;
  }
#undef TS_LAUNCH
  return ts::launch_status("reshape_and_cache");
}
