// (a) Per-block key centroids: build after prefill, refresh after append.
//
// centroid[b, h, j, :] = (sum over the real tokens t of block j of K[b, h, t, :]) / count,
// accumulated in float32 in token order and divided once (IEEE division).  This is
// bit-identical to the reference oracle's `keys[:, s:e].mean(axis=1)`
// (adakv/estimator.py:43-48), whose NumPy reduction over a non-contiguous axis
// adds rows sequentially in float32.  The reference's torch path builds the
// table in the cache dtype (adakv/attention.py:124-130); float32 is kept here
// because block selection must match the oracle exactly.
//
// Append (adakv/runtime.py:43-60) writes the new tokens into the preallocated
// cache in place and recomputes every touched block from its <= block_size
// tokens, so the table never drifts (the reference's running mean does, by up
// to 1e-4, tests/test_runtime_cpu.py:34-44).
//
// Layout: one warp (D = 128) or half warp (D = 64) per block, 4 dims per thread;
// a CTA of 256 threads covers 8 (or 16) consecutive blocks of one (b, kv head).
// Loads of a token row are coalesced (a warp reads D contiguous elements).
#include "kernels.h"

namespace adakv {

template <typename T>
__device__ __forceinline__ float4 load4(const T* p);
template <>
__device__ __forceinline__ float4 load4<float>(const float* p) {
  return *reinterpret_cast<const float4*>(p);
}
template <>
__device__ __forceinline__ float4 load4<__nv_bfloat16>(const __nv_bfloat16* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u),
                     __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xFFFF0000u));
}
template <>
__device__ __forceinline__ float4 load4<__half>(const __half* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}

template <typename T>
__device__ __forceinline__ void copy4(T* dst, const T* src) {
  if constexpr (sizeof(T) == 4) {
    *reinterpret_cast<float4*>(dst) = *reinterpret_cast<const float4*>(src);
  } else {
    *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(src);
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(256) centroid_kernel(CentroidParams p) {
  constexpr int TPR = D / 4;            // threads per block row
  constexpr int BPC = 256 / TPR;        // blocks per CTA
  pdl_wait();
  const int b = blockIdx.z, h = blockIdx.y;
  const int S = seq_len_of(p.seq_lens, b, p.max_seq_len);
  if (S <= 0 || S > p.max_seq_len || S < p.n_new) {
    if (threadIdx.x == 0 && blockIdx.x == 0 && h == 0) report(p.status, ADAKV_ST_BAD_SEQ_LEN);
    return;
  }
  const int S_old = S - p.n_new;
  const int nb = ceil_div(S, p.bs);
  const int first = p.n_new > 0 ? S_old / p.bs : 0;
  const int j = first + blockIdx.x * BPC + threadIdx.x / TPR;
  if (j >= nb) return;
  const int d = (threadIdx.x % TPR) * 4;
  const int t0 = j * p.bs;
  const int t1 = imin(t0 + p.bs, S);

  const T* kc = static_cast<const T*>(p.k.data) + b * p.k.sb + h * p.k.sh + d;
  T* kw = const_cast<T*>(kc);
  // new tokens come from k_new/v_new when given (append); otherwise they are
  // already in the cache and only the touched blocks are recomputed (refresh)
  const bool from_input = p.n_new > 0 && p.k_new.data != nullptr;
  T* vw = from_input ? static_cast<T*>(const_cast<void*>(p.v.data)) + b * p.v.sb + h * p.v.sh + d
                     : nullptr;
  const T* kn = from_input ? static_cast<const T*>(p.k_new.data) + b * p.k_new.sb + h * p.k_new.sh + d
                           : nullptr;
  const T* vn = from_input ? static_cast<const T*>(p.v_new.data) + b * p.v_new.sb + h * p.v_new.sh + d
                           : nullptr;

  // issue the token loads of up to 16 tokens together (independent loads in
  // flight at once), then add them in token order
  constexpr int kGroup = 16;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int base = t0; base < t1; base += kGroup) {
    float4 x[kGroup];
#pragma unroll
    for (int u = 0; u < kGroup; ++u) {
      const int t = base + u;
      if (t < t1) {
        if (from_input && t >= S_old) {  // a new token: read it from the input, store it in the cache
          const T* src = kn + (int64_t)(t - S_old) * p.k_new.ss;
          x[u] = load4<T>(src);
          copy4<T>(kw + (int64_t)t * p.k.ss, src);
          copy4<T>(vw + (int64_t)t * p.v.ss, vn + (int64_t)(t - S_old) * p.v_new.ss);
        } else {
          x[u] = load4<T>(kc + (int64_t)t * p.k.ss);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kGroup; ++u) {
      const int t = base + u;
      if (t < t1) {
        if (t == t0) {
          acc = x[u];
        } else {
          acc.x = __fadd_rn(acc.x, x[u].x);
          acc.y = __fadd_rn(acc.y, x[u].y);
          acc.z = __fadd_rn(acc.z, x[u].z);
          acc.w = __fadd_rn(acc.w, x[u].w);
        }
      }
    }
  }
  const float n = (float)(t1 - t0);
  float4 c = make_float4(__fdiv_rn(acc.x, n), __fdiv_rn(acc.y, n), __fdiv_rn(acc.z, n),
                         __fdiv_rn(acc.w, n));
  *reinterpret_cast<float4*>(p.cent + ((int64_t)(b * p.Hkv + h) * p.nb_cap + j) * D + d) = c;
}

template <typename T, int D>
static cudaError_t launch_centroid_t(const CentroidParams& p, int blocks_per_seq,
                                     cudaStream_t stream) {
  constexpr int TPR = D / 4;
  constexpr int BPC = 256 / TPR;
  dim3 grid(ceil_div(imax(blocks_per_seq, 1), BPC), p.Hkv, p.B);
  centroid_kernel<T, D><<<grid, 256, 0, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_centroid(const CentroidParams& p, int dtype, int D, int blocks_per_seq,
                            cudaStream_t stream) {
#define ADAKV_CENT_CASE(TT, DD) \
  if (D == DD) return launch_centroid_t<TT, DD>(p, blocks_per_seq, stream);
  if (dtype == ADAKV_DTYPE_F32) {
    ADAKV_CENT_CASE(float, 64) ADAKV_CENT_CASE(float, 128)
  } else if (dtype == ADAKV_DTYPE_F16) {
    ADAKV_CENT_CASE(__half, 64) ADAKV_CENT_CASE(__half, 128)
  } else if (dtype == ADAKV_DTYPE_BF16) {
    ADAKV_CENT_CASE(__nv_bfloat16, 64) ADAKV_CENT_CASE(__nv_bfloat16, 128)
  }
#undef ADAKV_CENT_CASE
  return cudaErrorInvalidValue;
}

}  // namespace adakv
