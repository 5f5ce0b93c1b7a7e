// K4 — batched block copy across every plane ([layer][K|V]) of the paged pool, and its swap
// form between the device pool and a pinned host arena of the same plane layout.
//
// No reference counterpart: tokenserve preempts by recompute (src/tokenserve/scheduler.py:215-225)
// and only shares full blocks (src/tokenserve/kv_cache.py:179-199); swap-to-host preemption is
// listed as future work (README.md "What a GPU run would add"). Semantics: for every pair
// (src, dst) and plane p, bytes [src*block_bytes, +block_bytes) of plane p of the source arena
// are copied to [dst*block_bytes, ...) of plane p of the destination arena. Each CTA moves one
// (pair, plane) block with 16-byte vectors and four loads in flight per thread: HBM-bound within
// the pool; bound by the host link when one side is pinned host memory, which the kernel reads
// or writes directly through its device-mapped address (one launch, no staging copy).
#include "common.cuh"

namespace {

struct Arena {
  uint8_t* base;
  int64_t plane_stride;
  int64_t num_blocks;
};

template <typename V>
__global__ void __launch_bounds__(256) copy_blocks_kernel(Arena dst_a, Arena src_a,
                                                          int64_t block_bytes,
                                                          const int64_t* __restrict__ src_dst,
                                                          int64_t num_pairs,
                                                          int32_t* __restrict__ error_flag) {
  const int64_t nvec = block_bytes / int64_t(sizeof(V));
  for (int64_t pair = blockIdx.x; pair < num_pairs; pair += gridDim.x) {
    const int64_t src = __ldg(src_dst + 2 * pair);
    const int64_t dst = __ldg(src_dst + 2 * pair + 1);
    if (src < 0 || dst < 0 || src >= src_a.num_blocks || dst >= dst_a.num_blocks) {
      if (error_flag != nullptr && threadIdx.x == 0) atomicExch(error_flag, 1);
      continue;
    }
    const V* s = reinterpret_cast<const V*>(src_a.base + int64_t(blockIdx.y) * src_a.plane_stride +
                                            src * block_bytes);
    V* d = reinterpret_cast<V*>(dst_a.base + int64_t(blockIdx.y) * dst_a.plane_stride +
                                dst * block_bytes);
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

int launch_copy(Arena dst, Arena src, int64_t num_planes, int64_t block_bytes,
                const int64_t* src_dst, int64_t num_pairs, int32_t* error_flag, cudaStream_t s) {
  const uint64_t a = reinterpret_cast<uint64_t>(dst.base) | reinterpret_cast<uint64_t>(src.base) |
                     uint64_t(dst.plane_stride) | uint64_t(src.plane_stride) |
                     uint64_t(block_bytes);
  const unsigned gx = static_cast<unsigned>(num_pairs < 65535 * 16 ? num_pairs : 65535 * 16);
  dim3 grid(gx, static_cast<unsigned>(num_planes));
  if (a % 16 == 0)
    copy_blocks_kernel<uint4><<<grid, 256, 0, s>>>(dst, src, block_bytes, src_dst, num_pairs,
                                                    error_flag);
  else if (a % 4 == 0)
    copy_blocks_kernel<uint32_t><<<grid, 256, 0, s>>>(dst, src, block_bytes, src_dst, num_pairs,
                                                       error_flag);
  else
    copy_blocks_kernel<uint8_t><<<grid, 256, 0, s>>>(dst, src, block_bytes, src_dst, num_pairs,
                                                      error_flag);
  return ts::launch_status("copy_blocks");
}

// The address a kernel on the current device uses for `p`, or nullptr when a kernel cannot
// reach it: pageable host memory, or another device's memory.
const void* kernel_address(const void* p) {
  cudaPointerAttributes attr{};
  if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
    (void)cudaGetLastError();
    return nullptr;
  }
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  switch (attr.type) {
    case cudaMemoryTypeHost: return attr.devicePointer;
    case cudaMemoryTypeManaged: return p;
    case cudaMemoryTypeDevice: return attr.device == dev ? p : nullptr;
    default: return nullptr;
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
  const Arena pool{static_cast<uint8_t*>(pool_base), plane_stride_bytes, num_blocks};
  return launch_copy(pool, pool, num_planes, block_bytes, src_dst, num_pairs, error_flag,
                     static_cast<cudaStream_t>(stream));
}

extern "C" int ts_swap_blocks(void* dst_base, int64_t dst_plane_stride_bytes,
                              int64_t dst_num_blocks, const void* src_base,
                              int64_t src_plane_stride_bytes, int64_t src_num_blocks,
                              int64_t num_planes, int64_t block_bytes, const int64_t* src_dst,
                              int64_t num_pairs, int32_t* error_flag, void* stream) {
  if (num_pairs < 0 || num_planes <= 0 || block_bytes <= 0 || dst_num_blocks <= 0 ||
      src_num_blocks <= 0 || dst_plane_stride_bytes < block_bytes * dst_num_blocks ||
      src_plane_stride_bytes < block_bytes * src_num_blocks)
    return ts::set_error(TS_ERR_INVALID_ARGUMENT,
                         "swap_blocks: bad sizes (planes %lld, block bytes %lld, blocks %lld -> "
                         "%lld, pairs %lld)",
                         (long long)num_planes, (long long)block_bytes, (long long)src_num_blocks,
                         (long long)dst_num_blocks, (long long)num_pairs);
  if (num_planes > 65535)
    return ts::set_error(TS_ERR_UNSUPPORTED, "swap_blocks: more than 65535 planes");
  if (num_pairs == 0) return ts::ok();
  if (!dst_base || !src_base || !src_dst)
    return ts::set_error(TS_ERR_INVALID_ARGUMENT, "swap_blocks: null pointer");
  // Every pointer the kernel dereferences must be reachable from this device: pinned host or
  // this device's memory. Pageable host memory is refused here instead of faulting the kernel.
  const void* d = kernel_address(dst_base);
  const void* s = kernel_address(src_base);
  const void* p = kernel_address(src_dst);
  const void* f = error_flag != nullptr ? kernel_address(error_flag) : nullptr;
  if (!d || !s || !p || (error_flag != nullptr && !f))
    return ts::set_error(TS_ERR_INVALID_ARGUMENT,
                         "swap_blocks: a buffer is neither pinned host memory nor memory of the "
                         "current device");
  const Arena dst{static_cast<uint8_t*>(const_cast<void*>(d)), dst_plane_stride_bytes,
                  dst_num_blocks};
  const Arena src{static_cast<uint8_t*>(const_cast<void*>(s)), src_plane_stride_bytes,
                  src_num_blocks};
  return launch_copy(dst, src, num_planes, block_bytes, static_cast<const int64_t*>(p), num_pairs,
                     static_cast<int32_t*>(const_cast<void*>(f)), static_cast<cudaStream_t>(stream));
}
