// CUDA-core paged attention for the shapes the tensor-core kernels do not cover: float32 KV
// (the tiny Llama, where greedy parity needs float32 products, so no TF32), block sizes other
// than 16 and head_dims outside {64, 128}. Decode (one query per sequence) and causal prefill.
//
// Semantics are transformers 5.5.0 eager_attention_forward (models/llama/modeling_llama.py:199)
// with repeat_kv (:187): query head q reads KV head q / (Hq / Hkv); scores are scaled by
// `scale`, causally masked for prefill and normalised with a float32 softmax.
//
// One CTA per (query row, query head); its four warps stride over the context tokens with an
// online softmax each and merge their (m, l, o) states through shared memory at the end.
#include "common.cuh"

namespace {

constexpr int kWarps = 4;

template <typename T, int NDL>  // NDL = head_dim / 32 dims per lane
__global__ void __launch_bounds__(kWarps * 32) paged_attention_portable_kernel(
    T* __restrict__ out, const T* __restrict__ query, int64_t q_stride,
    const T* __restrict__ key_pool, const T* __restrict__ value_pool,
    const int32_t* __restrict__ block_tables, int max_blocks, const int32_t* __restrict__ qsl,
    const int32_t* __restrict__ context_lens, int num_seqs, int num_q_heads, int num_kv_heads,
    int block_size, int64_t num_blocks, float scale) {
  constexpr int D = NDL * 32;
  const int row = blockIdx.x;
  const int qh = blockIdx.y;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int kvh = qh / (num_q_heads / num_kv_heads);

  // Which sequence owns this query row, and the last position it may attend to.
  int seq, n_attend;
  if (qsl == nullptr) {
    seq = row;
    n_attend = context_lens[row];
  } else {
    int lo = 0, hi = num_seqs - 1;
    while (lo < hi) {  // largest s with qsl[s] <= row
      const int mid = (lo + hi + 1) / 2;
      if (__ldg(qsl + mid) <= row) lo = mid; else hi = mid - 1;
    }
    seq = lo;
    const int q_len = qsl[seq + 1] - qsl[seq];
    n_attend = context_lens[seq] - q_len + (row - qsl[seq]) + 1;
  }
  const int max_tokens = max_blocks * block_size;
  if (n_attend > max_tokens) n_attend = max_tokens;

  float q[NDL];
  const T* qrow = query + int64_t(row) * q_stride + int64_t(qh) * D;
#pragma unroll
  for (int k = 0; k < NDL; ++k) q[k] = ts::to_float(qrow[lane + 32 * k]);

  float m = -INFINITY, l = 0.f, o[NDL];
#pragma unroll
  for (int k = 0; k < NDL; ++k) o[k] = 0.f;

  const int32_t* table = block_tables + int64_t(seq) * max_blocks;
  for (int j = warp; j < n_attend; j += kWarps) {
    const int64_t phys = __ldg(table + j / block_size);
    if (phys < 0 || phys >= num_blocks) continue;  // never reads outside the pool
    const int64_t r = ((phys * num_kv_heads + kvh) * block_size + j % block_size) * D;
    float dot = 0.f;
    float v[NDL];
#pragma unroll
    for (int k = 0; k < NDL; ++k) {
      dot += q[k] * ts::to_float(key_pool[r + lane + 32 * k]);
      v[k] = ts::to_float(value_pool[r + lane + 32 * k]);
    }
#pragma unroll
    for (int w = 16; w > 0; w >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, w);
    const float s = dot * scale;
    const float m_new = fmaxf(m, s);
    const float corr = expf(m - m_new);
    const float p = expf(s - m_new);
    l = l * corr + p;
#pragma unroll
    for (int k = 0; k < NDL; ++k) o[k] = o[k] * corr + p * v[k];
    m = m_new;
  }

  __shared__ float sm_m[kWarps], sm_l[kWarps];
  __shared__ float sm_o[kWarps][D];
  if (lane == 0) {
    sm_m[warp] = m;
    sm_l[warp] = l;
  }
#pragma unroll
  for (int k = 0; k < NDL; ++k) sm_o[warp][lane + 32 * k] = o[k];
  __syncthreads();
  if (warp == 0) {
    float mt = -INFINITY;
    for (int w = 0; w < kWarps; ++w) mt = fmaxf(mt, sm_m[w]);
    float lt = 0.f, acc[NDL];
#pragma unroll
    for (int k = 0; k < NDL; ++k) acc[k] = 0.f;
    for (int w = 0; w < kWarps; ++w) {
      const float f = sm_m[w] == -INFINITY ? 0.f : expf(sm_m[w] - mt);
      lt += sm_l[w] * f;
#pragma unroll
      for (int k = 0; k < NDL; ++k) acc[k] += sm_o[w][lane + 32 * k] * f;
    }
    const float inv = lt > 0.f ? 1.f / lt : 0.f;
    T* orow = out + (int64_t(row) * num_q_heads + qh) * D;
#pragma unroll
    for (int k = 0; k < NDL; ++k) orow[lane + 32 * k] = ts::from_float<T>(acc[k] * inv);
  }
}

template <typename T>
int launch_portable(void* out, const void* query, int64_t q_stride, const void* kp,
                    const void* vp, const int32_t* bt, int max_blocks, const int32_t* qsl,
                    const int32_t* cl, int num_seqs, int num_rows, int hq, int hkv, int hd,
                    int bs, int64_t nb, float scale, cudaStream_t s) {
  dim3 grid(num_rows, hq);
  auto o = static_cast<T*>(out);
  auto q = static_cast<const T*>(query);
  auto k = static_cast<const T*>(kp);
  auto v = static_cast<const T*>(vp);
#define TS_P(NDL)                                                                              \
  paged_attention_portable_kernel<T, NDL><<<grid, kWarps * 32, 0, s>>>(                        \
      o, q, q_stride, k, v, bt, max_blocks, qsl, cl, num_seqs, hq, hkv, bs, nb, scale)
  switch (hd) {
    case 32: TS_P(1); break;
    case 64: TS_P(2); break;
    case 128: TS_P(4); break;
    case 256: TS_P(8); break;
    default:
      return ts::set_error(TS_ERR_UNSUPPORTED, "paged attention: head_dim %d not supported", hd);
  }
#undef TS_P
  return ts::launch_status("paged_attention_portable");
}

}  // namespace

namespace ts {

// Launches the CUDA-core kernel; `qsl == nullptr` means one query row per sequence (decode).
int paged_attention_portable(void* out, const void* query, int64_t q_stride, const void* kp,
                             const void* vp, const int32_t* bt, int max_blocks,
                             const int32_t* qsl, const int32_t* cl, int num_seqs, int num_rows,
                             int hq, int hkv, int hd, int bs, int64_t nb, float scale, int dtype,
                             cudaStream_t s) {
  if (num_rows == 0) return ok();
  if (num_rows > 2147483647 || hq > 65535)
    return set_error(TS_ERR_UNSUPPORTED, "paged attention: grid too large");
  switch (dtype) {
    case TS_FLOAT32:
      return launch_portable<float>(out, query, q_stride, kp, vp, bt, max_blocks, qsl, cl,
                                    num_seqs, num_rows, hq, hkv, hd, bs, nb, scale, s);
    case TS_FLOAT16:
      return launch_portable<__half>(out, query, q_stride, kp, vp, bt, max_blocks, qsl, cl,
                                     num_seqs, num_rows, hq, hkv, hd, bs, nb, scale, s);
    case TS_BFLOAT16:
      return launch_portable<__nv_bfloat16>(out, query, q_stride, kp, vp, bt, max_blocks, qsl,
                                            cl, num_seqs, num_rows, hq, hkv, hd, bs, nb, scale, s);
    default:
      return set_error(TS_ERR_INVALID_ARGUMENT, "paged attention: bad dtype %d", dtype);
  }
}

}  // namespace ts
