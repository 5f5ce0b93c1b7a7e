// Fused element-wise parts of a Llama decoder layer, used by the paged model runner so a layer
// is ~10 kernels instead of ~35. Each reproduces the rounding points of the transformers 5.5.0
// module it replaces (models/llama/modeling_llama.py), so a float32 model computes the same
// values and a bf16/fp16 model rounds where the module rounds:
//   * ts_add_rmsnorm   — `residual + x` in the model dtype, then LlamaRMSNorm (:53-70): statistics
//                        in fp32, x * rsqrt(mean(x^2) + eps) cast to the dtype, times the weight.
//   * ts_rope_and_cache — apply_rotary_pos_emb (:146-168) on q and k (cos/sin of
//                        position * inv_freq in fp32, cast to the dtype; q*cos + rotate_half(q)*sin
//                        with each product and the sum rounded to the dtype), then K1: the rotated
//                        K and V rows scattered into the paged pool through the slot mapping.
//   * ts_silu_mul      — LlamaMLP's act_fn(gate) * up (:184) on a fused [gate | up] projection.
#include "common.cuh"

namespace {

template <typename T>
__device__ __forceinline__ T rnd(float x) {
  return ts::from_float<T>(x);
}

// ------------------------------------------------------------------------- add + RMSNorm

template <typename T, int THREADS>
__global__ void __launch_bounds__(THREADS) add_rmsnorm_kernel(T* __restrict__ out,
                                                              T* __restrict__ residual,
                                                              const T* __restrict__ x,
                                                              const T* __restrict__ weight,
                                                              int hidden, float eps) {
  const int64_t row = blockIdx.x;
  T* res = residual + row * hidden;
  const T* xr = x == nullptr ? nullptr : x + row * hidden;
  float ss = 0.f;
  for (int i = threadIdx.x; i < hidden; i += THREADS) {
    float v = ts::to_float(res[i]);
    if (xr != nullptr) {
      const T s = rnd<T>(v + ts::to_float(xr[i]));  // residual + hidden_states, in the dtype
      res[i] = s;
      v = ts::to_float(s);
    }
    ss += v * v;
  }
  __shared__ float red[THREADS / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < THREADS / 32 ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / float(hidden) + eps);
  T* o = out + row * hidden;
  for (int i = threadIdx.x; i < hidden; i += THREADS) {
    const T normed = rnd<T>(ts::to_float(res[i]) * inv);  // .to(input_dtype)
    o[i] = rnd<T>(ts::to_float(weight[i]) * ts::to_float(normed));
  }
}

// 16-byte vector of T: one LDG.128 / STG.128.
template <typename T>
struct alignas(16) Vec {
  static constexpr int E = 16 / sizeof(T);
  T v[E];
};

// Same arithmetic as add_rmsnorm_kernel, with 16-byte accesses and the row held in registers
// between the statistics pass and the output pass (one read of the residual instead of two).
// Requires hidden % E == 0, hidden <= THREADS * NV * E and 16-byte aligned rows.
template <typename T, int THREADS, int NV>
__global__ void __launch_bounds__(THREADS) add_rmsnorm_vec_kernel(T* __restrict__ out,
                                                                  T* __restrict__ residual,
                                                                  const T* __restrict__ x,
                                                                  const T* __restrict__ weight,
                                                                  int hidden, float eps) {
  constexpr int E = Vec<T>::E;
  const int nvec = hidden / E;
  const int64_t row = blockIdx.x;
  Vec<T>* res = reinterpret_cast<Vec<T>*>(residual + row * hidden);
  const Vec<T>* xr = x == nullptr ? nullptr : reinterpret_cast<const Vec<T>*>(x + row * hidden);
  float v[NV][E];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int idx = threadIdx.x + k * THREADS;
    if (idx < nvec) {
      Vec<T> r = res[idx];
      if (xr != nullptr) {
        const Vec<T> a = xr[idx];
#pragma unroll
        for (int e = 0; e < E; ++e) r.v[e] = rnd<T>(ts::to_float(r.v[e]) + ts::to_float(a.v[e]));
        res[idx] = r;
      }
#pragma unroll
      for (int e = 0; e < E; ++e) {
        v[k][e] = ts::to_float(r.v[e]);
        ss += v[k][e] * v[k][e];
      }
    }
  }
  __shared__ float red[THREADS / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < THREADS / 32; ++w) tot += red[w];
  const float inv = rsqrtf(tot / float(hidden) + eps);
  const Vec<T>* wv = reinterpret_cast<const Vec<T>*>(weight);
  Vec<T>* o = reinterpret_cast<Vec<T>*>(out + row * hidden);
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int idx = threadIdx.x + k * THREADS;
    if (idx < nvec) {
      const Vec<T> w = wv[idx];
      Vec<T> y;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const T normed = rnd<T>(v[k][e] * inv);  // .to(input_dtype)
        y.v[e] = rnd<T>(ts::to_float(w.v[e]) * ts::to_float(normed));
      }
      o[idx] = y;
    }
  }
}

__host__ __forceinline__ bool aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

// ------------------------------------------------------------------------- RoPE + K1

constexpr int kMaxHalf = 256;  // head_dim <= 512

// One CTA per token; one thread per (head, dim pair i in [0, D/2)).
template <typename T>
__global__ void rope_and_cache_kernel(const T* __restrict__ qkv, int64_t qkv_stride,
                                      T* __restrict__ q_out, T* __restrict__ key_pool,
                                      T* __restrict__ value_pool,
                                      const int64_t* __restrict__ slots,
                                      const int64_t* __restrict__ positions,
                                      const float* __restrict__ inv_freq, int hq, int hkv, int d,
                                      int block_size, int64_t num_slots,
                                      int32_t* __restrict__ error_flag) {
  ts::allow_dependents();  // the attention kernels after it wait for this grid on the device
  const int64_t t = blockIdx.x;
  const T* row = qkv + t * qkv_stride;
  const float pos = float(__ldg(positions + t));
  const int half = d / 2;
  __shared__ float cs[2][kMaxHalf];  // cos / sin per angle, rounded to the dtype
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    const float ang = pos * __ldg(inv_freq + i);
    cs[0][i] = ts::to_float(rnd<T>(cosf(ang)));
    cs[1][i] = ts::to_float(rnd<T>(sinf(ang)));
  }
  __syncthreads();
  const int64_t slot = __ldg(slots + t);
  const bool write_kv = slot >= 0 && slot < num_slots;
  if (slot >= num_slots && error_flag != nullptr && threadIdx.x == 0) atomicExch(error_flag, 1);
  const int64_t blk = write_kv ? slot / block_size : 0;
  const int64_t off = write_kv ? slot - blk * block_size : 0;
  for (int j = threadIdx.x; j < (hq + 2 * hkv) * half; j += blockDim.x) {
    const int h = j / half, i = j - (j / half) * half;
    if (h < hq + hkv) {
      // cos/sin of emb = cat(freqs, freqs): dims i and i + D/2 share the angle.
      const float x1 = ts::to_float(row[h * d + i]), x2 = ts::to_float(row[h * d + i + half]);
      const float cf = cs[0][i], sf = cs[1][i];
      // rotate_half(x) = cat(-x2, x1)
      const T y1 = rnd<T>(ts::to_float(rnd<T>(__fmul_rn(x1, cf))) +
                          ts::to_float(rnd<T>(__fmul_rn(-x2, sf))));
      const T y2 = rnd<T>(ts::to_float(rnd<T>(__fmul_rn(x2, cf))) +
                          ts::to_float(rnd<T>(__fmul_rn(x1, sf))));
      if (h < hq) {
        T* qo = q_out + (t * hq + h) * d;
        qo[i] = y1;
        qo[i + half] = y2;
      } else if (write_kv) {
        T* kd = key_pool + ((blk * hkv + (h - hq)) * block_size + off) * d;
        kd[i] = y1;
        kd[i + half] = y2;
      }
    } else if (write_kv) {
      const int hv = h - hq - hkv;
      T* vd = value_pool + ((blk * hkv + hv) * block_size + off) * d;
      vd[i] = row[h * d + i];
      vd[i + half] = row[h * d + i + half];
    }
  }
}

// rope_and_cache_kernel with each thread on E consecutive dimension pairs (16-byte accesses).
// Requires (head_dim / 2) % E == 0 and 16-byte aligned rows.
template <typename T>
__global__ void rope_and_cache_vec_kernel(const T* __restrict__ qkv, int64_t qkv_stride,
                                          T* __restrict__ q_out, T* __restrict__ key_pool,
                                          T* __restrict__ value_pool,
                                          const int64_t* __restrict__ slots,
                                          const int64_t* __restrict__ positions,
                                          const float* __restrict__ inv_freq, int hq, int hkv,
                                          int d, int block_size, int64_t num_slots,
                                          int32_t* __restrict__ error_flag) {
  ts::allow_dependents();  // the attention kernels after it wait for this grid on the device
  constexpr int E = Vec<T>::E;
  const int64_t t = blockIdx.x;
  const T* row = qkv + t * qkv_stride;
  const float pos = float(__ldg(positions + t));
  const int half = d / 2, cpr = half / E;
  // cos / sin of this token's angles, rounded to the dtype, computed once for every head.
  __shared__ float cs[2][kMaxHalf];
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    const float ang = pos * __ldg(inv_freq + i);
    cs[0][i] = ts::to_float(rnd<T>(cosf(ang)));
    cs[1][i] = ts::to_float(rnd<T>(sinf(ang)));
  }
  __syncthreads();
  const int64_t slot = __ldg(slots + t);
  const bool write_kv = slot >= 0 && slot < num_slots;
  if (slot >= num_slots && error_flag != nullptr && threadIdx.x == 0) atomicExch(error_flag, 1);
  const int64_t blk = write_kv ? slot / block_size : 0;
  const int64_t off = write_kv ? slot - blk * block_size : 0;
  for (int j = threadIdx.x; j < (hq + 2 * hkv) * cpr; j += blockDim.x) {
    const int h = j / cpr, i0 = (j - h * cpr) * E;
    const Vec<T> a = *reinterpret_cast<const Vec<T>*>(row + h * d + i0);
    const Vec<T> b = *reinterpret_cast<const Vec<T>*>(row + h * d + i0 + half);
    T* dst;
    Vec<T> y1 = a, y2 = b;
    if (h < hq + hkv) {
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const float cf = cs[0][i0 + e], sf = cs[1][i0 + e];
        const float x1 = ts::to_float(a.v[e]), x2 = ts::to_float(b.v[e]);
        y1.v[e] = rnd<T>(ts::to_float(rnd<T>(__fmul_rn(x1, cf))) +
                         ts::to_float(rnd<T>(__fmul_rn(-x2, sf))));
        y2.v[e] = rnd<T>(ts::to_float(rnd<T>(__fmul_rn(x2, cf))) +
                         ts::to_float(rnd<T>(__fmul_rn(x1, sf))));
      }
      if (h < hq) {
        dst = q_out + (t * hq + h) * d;
      } else {
        if (!write_kv) continue;
        dst = key_pool + ((blk * hkv + (h - hq)) * block_size + off) * d;
      }
    } else {
      if (!write_kv) continue;
      dst = value_pool + ((blk * hkv + (h - hq - hkv)) * block_size + off) * d;
    }
    *reinterpret_cast<Vec<T>*>(dst + i0) = y1;
    *reinterpret_cast<Vec<T>*>(dst + i0 + half) = y2;
  }
}

// ------------------------------------------------------------------------- SiLU * up

template <typename T>
__global__ void silu_mul_kernel(T* __restrict__ out, const T* __restrict__ gate_up, int64_t rows,
                                int inter) {
  const int64_t n = rows * inter;
  for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < n;
       e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = e / inter;
    const int c = int(e - r * inter);
    const float g = ts::to_float(gate_up[r * 2 * inter + c]);
    const float u = ts::to_float(gate_up[r * 2 * inter + inter + c]);
    const T a = rnd<T>(g / (1.f + expf(-g)));  // silu in fp32, result in the dtype
    out[e] = rnd<T>(ts::to_float(a) * u);
  }
}

// silu_mul_kernel on E consecutive columns per thread (16-byte accesses).
// Requires intermediate % E == 0 and 16-byte aligned rows.
template <typename T>
__global__ void silu_mul_vec_kernel(T* __restrict__ out, const T* __restrict__ gate_up,
                                    int64_t rows, int inter) {
  constexpr int E = Vec<T>::E;
  const int cpr = inter / E;
  const int64_t n = rows * cpr;
  for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < n;
       e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = e / cpr;
    const int c = int(e - r * cpr) * E;
    const Vec<T> g = *reinterpret_cast<const Vec<T>*>(gate_up + r * 2 * inter + c);
    const Vec<T> u = *reinterpret_cast<const Vec<T>*>(gate_up + r * 2 * inter + inter + c);
    Vec<T> y;
#pragma unroll
    for (int k = 0; k < E; ++k) {
      const float gf = ts::to_float(g.v[k]);
      const T a = rnd<T>(gf / (1.f + expf(-gf)));
      y.v[k] = rnd<T>(ts::to_float(a) * ts::to_float(u.v[k]));
    }
    *reinterpret_cast<Vec<T>*>(out + r * inter + c) = y;
  }
}

template <typename T>
int launch_add_rmsnorm(void* out, void* res, const void* x, const void* w, int64_t rows,
                       int hidden, float eps, cudaStream_t s) {
  constexpr int E = Vec<T>::E;
  const bool vec = hidden % E == 0 && aligned16(out) && aligned16(res) && aligned16(w) &&
                   (x == nullptr || aligned16(x));
  T* o = static_cast<T*>(out);
  T* r = static_cast<T*>(res);
  const T* xp = static_cast<const T*>(x);
  const T* wp = static_cast<const T*>(w);
  if (vec && hidden <= 256 * E)
    add_rmsnorm_vec_kernel<T, 256, 1><<<unsigned(rows), 256, 0, s>>>(o, r, xp, wp, hidden, eps);
  else if (vec && hidden <= 256 * 2 * E)
    add_rmsnorm_vec_kernel<T, 256, 2><<<unsigned(rows), 256, 0, s>>>(o, r, xp, wp, hidden, eps);
  else if (vec && hidden <= 256 * 4 * E)
    add_rmsnorm_vec_kernel<T, 256, 4><<<unsigned(rows), 256, 0, s>>>(o, r, xp, wp, hidden, eps);
  else
    add_rmsnorm_kernel<T, 256><<<unsigned(rows), 256, 0, s>>>(o, r, xp, wp, hidden, eps);
  return ts::launch_status("add_rmsnorm");
}

}  // namespace

extern "C" int ts_add_rmsnorm(void* out, void* residual, const void* x, const void* weight,
                              int64_t num_rows, int32_t hidden, float eps, int32_t dtype,
                              void* stream) {
  if (num_rows < 0 || hidden <= 0 || ts::dtype_size(dtype) == 0)
    return ts::set_error(TS_ERR_INVALID_ARGUMENT, "add_rmsnorm: bad sizes or dtype");
  if (num_rows == 0) return ts::ok();
  if (num_rows > 2147483647) return ts::set_error(TS_ERR_UNSUPPORTED, "add_rmsnorm: too many rows");
  if (!out || !residual || !weight)
    return ts::set_error(TS_ERR_INVALID_ARGUMENT, "add_rmsnorm: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case TS_FLOAT32: return launch_add_rmsnorm<float>(out, residual, x, weight, num_rows, hidden, eps, s);
    case TS_FLOAT16: return launch_add_rmsnorm<__half>(out, residual, x, weight, num_rows, hidden, eps, s);
    default: return launch_add_rmsnorm<__nv_bfloat16>(out, residual, x, weight, num_rows, hidden, eps, s);
  }
}

extern "C" int ts_rope_and_cache(const void* qkv, int64_t qkv_token_stride, void* q_out,
                                 void* key_pool, void* value_pool, const int64_t* slot_mapping,
                                 const int64_t* positions, const float* inv_freq,
                                 int64_t num_tokens, int32_t num_q_heads, int32_t num_kv_heads,
                                 int32_t head_dim, int32_t block_size, int64_t num_blocks,
                                 int32_t dtype, int32_t* error_flag, void* stream) {
  if (num_tokens < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0 ||
      head_dim % 2 || block_size <= 0 || num_blocks <= 0 || ts::dtype_size(dtype) == 0)
    return ts::set_error(TS_ERR_INVALID_ARGUMENT, "rope_and_cache: bad sizes or dtype");
  if (head_dim > 2 * kMaxHalf)
    return ts::set_error(TS_ERR_UNSUPPORTED, "rope_and_cache: head_dim above %d", 2 * kMaxHalf);
  if (qkv_token_stride < int64_t(num_q_heads + 2 * num_kv_heads) * head_dim)
    return ts::set_error(TS_ERR_INVALID_ARGUMENT, "rope_and_cache: qkv stride too small");
  if (num_tokens == 0) return ts::ok();
  if (num_tokens > 2147483647) return ts::set_error(TS_ERR_UNSUPPORTED, "rope_and_cache: too many tokens");
  if (!qkv || !q_out || !key_pool || !value_pool || !slot_mapping || !positions || !inv_freq)
    return ts::set_error(TS_ERR_INVALID_ARGUMENT, "rope_and_cache: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int work = (num_q_heads + 2 * num_kv_heads) * head_dim / 2;
  const int threads = work >= 512 ? 512 : ((work + 31) / 32) * 32;
  const int64_t ns = num_blocks * block_size;
  const int esz = ts::dtype_size(dtype), ev = 16 / esz;
  const bool vec = (head_dim / 2) % ev == 0 && (qkv_token_stride * esz) % 16 == 0 &&
                   aligned16(qkv) && aligned16(q_out) && aligned16(key_pool) &&
                   aligned16(value_pool);
  const int vwork = work / ev;
  const int vthreads = vwork >= 256 ? 256 : ((vwork + 31) / 32) * 32;
#define TS_R(T)                                                                                 \
  if (vec)                                                                                      \
    rope_and_cache_vec_kernel<T><<<unsigned(num_tokens), vthreads, 0, s>>>(                    \
        static_cast<const T*>(qkv), qkv_token_stride, static_cast<T*>(q_out),                  \
        static_cast<T*>(key_pool), static_cast<T*>(value_pool), slot_mapping, positions,       \
        inv_freq, num_q_heads, num_kv_heads, head_dim, block_size, ns, error_flag);            \
  else                                                                                          \
    rope_and_cache_kernel<T><<<unsigned(num_tokens), threads, 0, s>>>(                         \
        static_cast<const T*>(qkv), qkv_token_stride, static_cast<T*>(q_out),                  \
        static_cast<T*>(key_pool), static_cast<T*>(value_pool), slot_mapping, positions,       \
        inv_freq, num_q_heads, num_kv_heads, head_dim, block_size, ns, error_flag)
  switch (dtype) {
    case TS_FLOAT32: TS_R(float); break;
    case TS_FLOAT16: TS_R(__half); break;
    default: TS_R(__nv_bfloat16); break;
  }
#undef TS_R
  return ts::launch_status("rope_and_cache");
}

extern "C" int ts_silu_mul(void* out, const void* gate_up, int64_t num_rows,
                           int32_t intermediate, int32_t dtype, void* stream) {
  if (num_rows < 0 || intermediate <= 0 || ts::dtype_size(dtype) == 0)
    return ts::set_error(TS_ERR_INVALID_ARGUMENT, "silu_mul: bad sizes or dtype");
  if (num_rows == 0) return ts::ok();
  if (!out || !gate_up) return ts::set_error(TS_ERR_INVALID_ARGUMENT, "silu_mul: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t n = num_rows * intermediate;
  const unsigned grid = unsigned(n / 256 + 1 < 148 * 16 ? n / 256 + 1 : 148 * 16);
  const int ev = 16 / ts::dtype_size(dtype);
  if (intermediate % ev == 0 && aligned16(out) && aligned16(gate_up)) {
    const int64_t nv = n / ev;
    const unsigned vgrid = unsigned(nv / 256 + 1 < 148 * 16 ? nv / 256 + 1 : 148 * 16);
    switch (dtype) {
      case TS_FLOAT32:
        silu_mul_vec_kernel<float><<<vgrid, 256, 0, s>>>(
            static_cast<float*>(out), static_cast<const float*>(gate_up), num_rows, intermediate);
        break;
      case TS_FLOAT16:
        silu_mul_vec_kernel<__half><<<vgrid, 256, 0, s>>>(
            static_cast<__half*>(out), static_cast<const __half*>(gate_up), num_rows, intermediate);
        break;
      default:
        silu_mul_vec_kernel<__nv_bfloat16><<<vgrid, 256, 0, s>>>(
            static_cast<__nv_bfloat16*>(out), static_cast<const __nv_bfloat16*>(gate_up), num_rows,
            intermediate);
        break;
    }
    return ts::launch_status("silu_mul");
  }
  switch (dtype) {
    case TS_FLOAT32:
      silu_mul_kernel<float><<<grid, 256, 0, s>>>(static_cast<float*>(out),
                                                  static_cast<const float*>(gate_up), num_rows,
                                                  intermediate);
      break;
    case TS_FLOAT16:
      silu_mul_kernel<__half><<<grid, 256, 0, s>>>(static_cast<__half*>(out),
                                                   static_cast<const __half*>(gate_up), num_rows,
                                                   intermediate);
      break;
    default:
      silu_mul_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
          static_cast<__nv_bfloat16*>(out), static_cast<const __nv_bfloat16*>(gate_up), num_rows,
          intermediate);
      break;
  }
  return ts::launch_status("silu_mul");
}
