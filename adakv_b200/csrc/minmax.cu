// (b') The "minmax" (Quest) block estimator: per-block per-dimension key
// minima and maxima (adakv/estimator.py:50-57, adakv/attention.py:134-138)
// and the upper-bound score sum_d max(q_d, 0) kmax_d + min(q_d, 0) kmin_d
// (adakv/estimator.py:76-79, adakv/attention.py:190-198).
//
// Tables: kmin / kmax [B, Hkv, nb_cap, D] float32, exact (min / max of the
// cache's values converted to float32).  Scores: one warp per (block,
// sequence, KV head) scores the g query heads of the group; a lane holds D/32
// dimensions, products are fused multiply-adds in float32 and the warp sums
// them with xor shuffles (float rounding differs from NumPy's pairwise sum by
// a few ulps, like the centroid estimator).
#include "kernels.h"

namespace adakv {

constexpr int kMinmaxWarps = 8;  // blocks per CTA (one per warp)

// build (n_new == 0: every block) or refresh (the blocks touched by the last
// n_new tokens of each sequence)
template <typename T, int D>
__global__ void __launch_bounds__(kMinmaxWarps * 32) minmax_build_kernel(MinmaxParams p) {
  constexpr int E = D / 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kvh = blockIdx.y, b = blockIdx.z;
  int S = seq_len_of(p.seq_lens, b, p.max_seq_len);
  if (S < 0 || S > p.max_seq_len) return;
  const int nb = ceil_div(S, p.bs);
  const int first = p.n_new > 0 ? imax(0, (S - p.n_new) / p.bs) : 0;
  const int blk = first + blockIdx.x * kMinmaxWarps + warp;
  if (blk >= nb) return;
  const int t0 = blk * p.bs, t1 = imin(t0 + p.bs, S);
  const T* kb = static_cast<const T*>(p.k.data) + b * p.k.sb + kvh * p.k.sh + lane * E;
  float mn[E], mx[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    mn[e] = INFINITY;
    mx[e] = -INFINITY;
  }
  for (int t = t0; t < t1; ++t) {
    float x[E];
#pragma unroll
    for (int e = 0; e < E; ++e) x[e] = to_f32(kb[(int64_t)t * p.k.ss + e]);
#pragma unroll
    for (int e = 0; e < E; ++e) {
      mn[e] = fminf(mn[e], x[e]);
      mx[e] = fmaxf(mx[e], x[e]);
    }
  }
  const int64_t row = ((int64_t)(b * p.Hkv + kvh) * p.nb_cap + blk) * D + lane * E;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    p.kmin[row + e] = mn[e];
    p.kmax[row + e] = mx[e];
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(kMinmaxWarps * 32) minmax_score_kernel(MinmaxParams p) {
  constexpr int E = D / 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kvh = blockIdx.y, b = blockIdx.z;
  int S = seq_len_of(p.seq_lens, b, p.max_seq_len);
  if (S < 0 || S > p.max_seq_len) S = 0;
  const int nb = ceil_div(S, p.bs);
  const int blk = blockIdx.x * kMinmaxWarps + warp;
  if (blk >= nb) return;
  const int64_t row = ((int64_t)(b * p.Hkv + kvh) * p.nb_cap + blk) * D + lane * E;
  float mn[E], mx[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    mn[e] = p.kmin[row + e];
    mx[e] = p.kmax[row + e];
  }
  const T* qb = static_cast<const T*>(p.q.data) + b * p.q.sb + (int64_t)kvh * p.g * p.q.sh + lane * E;
  for (int j = 0; j < p.g; ++j) {
    float acc = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float qv = to_f32(qb[(int64_t)j * p.q.sh + e]);
      acc = fmaf(fmaxf(qv, 0.f), mx[e], acc);
      acc = fmaf(fminf(qv, 0.f), mn[e], acc);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) p.scores[(int64_t)(b * p.Hq + kvh * p.g + j) * p.score_stride + blk] = acc;
  }
}

template <typename F>
static cudaError_t for_each_minmax(int dtype, int D, F&& f) {
#define ADAKV_MM(TT)                                                  \
  if (D == 64) return f(minmax_build_kernel<TT, 64>, minmax_score_kernel<TT, 64>); \
  if (D == 128) return f(minmax_build_kernel<TT, 128>, minmax_score_kernel<TT, 128>);
  if (dtype == ADAKV_DTYPE_F32) {
    ADAKV_MM(float)
  } else if (dtype == ADAKV_DTYPE_F16) {
    ADAKV_MM(__half)
  } else if (dtype == ADAKV_DTYPE_BF16) {
    ADAKV_MM(__nv_bfloat16)
  }
#undef ADAKV_MM
  return cudaErrorInvalidValue;
}

cudaError_t launch_minmax_build(const MinmaxParams& p, int dtype, int D, int blocks_per_seq,
                                cudaStream_t st) {
  const dim3 grid(imax(1, ceil_div(blocks_per_seq, kMinmaxWarps)), p.Hkv, p.B);
  return for_each_minmax(dtype, D, [&](auto build, auto) {
    build<<<grid, kMinmaxWarps * 32, 0, st>>>(p);
    return cudaGetLastError();
  });
}

cudaError_t launch_minmax_score(const MinmaxParams& p, int dtype, int D, int nb_max, cudaStream_t st) {
  const dim3 grid(imax(1, ceil_div(nb_max, kMinmaxWarps)), p.Hkv, p.B);
  return for_each_minmax(dtype, D, [&](auto, auto score) {
    score<<<grid, kMinmaxWarps * 32, 0, st>>>(p);
    return cudaGetLastError();
  });
}

}  // namespace adakv
