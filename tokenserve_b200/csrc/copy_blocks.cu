// K4 — batched block copy across every plane ([layer][K|V]) of the paged pool.
//
// No reference counterpart: tokenserve preempts by recompute (src/tokenserve/scheduler.py:215-225)
// and only shares full blocks (src/tokenserve/kv_cache.py:179-199). Semantics: for every pair
// (src, dst) and plane p, bytes [src*block_bytes, +block_bytes) of plane p are copied to
// [dst*block_bytes, ...). HBM-bound; each CTA moves one (pair, plane) block with 16-byte
// vectors and four loads in flight per thread.
#include "common.cuh"

namespace {

template <typename V>
__global__ void __launch_bounds__(256) copy_blocks_kernel(uint8_t* __restrict__ base,
                                                          int64_t plane_stride_b,
                                                          int64_t block_bytes, int64_t num_blocks,
                                                          const int64_t* __restrict__ src_dst,
                                                          int64_t num_pairs,
                                                          int32_t* __restrict__ error_flag) {
  const int64_t nvec = block_bytes / int64_t(sizeof(V));
  for (int64_t pair = blockIdx.x; pair < num_pairs; pair += gridDim.x) {
    const int64_t src = __ldg(src_dst + 2 * pair);
    const int64_t dst = __ldg(src_dst + 2 * pair + 1);
    if (src < 0 || dst < 0 || src >= num_blocks || dst >= num_blocks) {
      if (error_flag != nullptr && threadIdx.x == 0) atomicExch(error_flag, 1);
      continue;
    }
    uint8_t* plane = base + int64_t(blockIdx.y) * plane_stride_b;
    const V* s = reinterpret_cast<const V*>(plane + src * block_bytes);
    V* d = reinterpret_cast<V*>(plane + dst * block_bytes);
    constexpr int U = 4;
    int64_t i = threadIdx.x;
    for (; i + (U - 1) * int64_t(blockDim.x) < nvec; i += U * int64_t(blockDim.x)) {
      V r[U];
#pragma unroll
      for (int u = 0; u < U; ++u) r[u] = s[i + u * int64_t(blockDim.x)];
#pragma unroll
      for (int u = 0; u < U; ++u) d[i + u * int64_t(blockDim.x)] = r[u];
    }
    for (; i < nvec; i += blockDim.x) d[i] = s[i];
  }
}

}  // namespace

extern "C" int ts_copy_blocks(void* pool_base, int64_t num_planes, int64_t plane_stride_bytes,
                              int64_t block_bytes, int64_t num_blocks, const int64_t* src_dst,
                              int64_t num_pairs, int32_t* error_flag, void* stream) {
  if (num_pairs < 0 || num_planes <= 0 || block_bytes <= 0 || num_blocks <= 0 ||
      plane_stride_bytes < block_bytes * num_blocks)
    return ts::set_error(TS_ERR_INVALID_ARGUMENT,
                         "copy_blocks: bad sizes (planes %lld, plane stride %lld, block bytes "
                         "%lld, blocks %lld, pairs %lld)",
                         (long long)num_planes, (long long)plane_stride_bytes,
                         (long long)block_bytes, (long long)num_blocks, (long long)num_pairs);
  if (num_planes > 65535)
    return ts::set_error(TS_ERR_UNSUPPORTED, "copy_blocks: more than 65535 planes");
  if (num_pairs == 0) return ts::ok();
  if (!pool_base || !src_dst) return ts::set_error(TS_ERR_INVALID_ARGUMENT, "copy_blocks: null pointer");
  const uint64_t a = reinterpret_cast<uint64_t>(pool_base) | uint64_t(plane_stride_bytes) |
                     uint64_t(block_bytes);
  const unsigned gx = static_cast<unsigned>(num_pairs < 65535 * 16 ? num_pairs : 65535 * 16);
  dim3 grid(gx, static_cast<unsigned>(num_planes));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto base = static_cast<uint8_t*>(pool_base);
  if (a % 16 == 0)
    copy_blocks_kernel<uint4><<<grid, 256, 0, s>>>(base, plane_stride_bytes, block_bytes,
                                                    num_blocks, src_dst, num_pairs, error_flag);
  else if (a % 4 == 0)
    copy_blocks_kernel<uint32_t><<<grid, 256, 0, s>>>(base, plane_stride_bytes, block_bytes,
                                                       num_blocks, src_dst, num_pairs, error_flag);
  else
    copy_blocks_kernel<uint8_t><<<grid, 256, 0, s>>>(base, plane_stride_bytes, block_bytes,
                                                      num_blocks, src_dst, num_pairs, error_flag);
  return ts::launch_status("copy_blocks");
}
