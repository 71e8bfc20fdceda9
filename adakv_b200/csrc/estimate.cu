// (b) Centroid block estimator: scores[b, h, j] = q[b, h] . centroid[b, h / g, j]
// (unscaled, float32), the reference's einsum("hd,hbd->hb") over GQA-expanded
// centroids (adakv/estimator.py:73-74, adakv/attention.py:187-189) with the
// expansion folded away: each centroid row is read from HBM once and scored
// against all g query heads of its KV head.
//
// One CTA streams kEstRows contiguous centroid rows of one (b, kv head) into
// shared memory with a single bulk copy (the TMA engine, completion on an
// mbarrier), then 8 warps score 8 rows each.  Lane l owns dims
// [l*D/32, (l+1)*D/32) of every row and keeps the g queries' matching slices in
// registers; 32 (row, head) partial dot products are finished with one
// 31-shuffle butterfly reduce-scatter, after which lane l holds the full score of
// slot l.  The CTA also emits the per-(b, h) maximum over its rows, which the
// budget kernel combines into the softmax maximum.
//
// HBM traffic per step = the float32 centroid table (B * Hkv * nb * D * 4 bytes)
// plus q; scores (B * Hq * nb * 4 bytes) stay in L2 for the next kernels.
#include "kernels.h"

namespace adakv {

template <int E>
__device__ __forceinline__ void lds_row(const float* p, float (&c)[E]) {
  if constexpr (E == 4) {
    const float4 v = *reinterpret_cast<const float4*>(p);
    c[0] = v.x; c[1] = v.y; c[2] = v.z; c[3] = v.w;
  } else if constexpr (E == 2) {
    const float2 v = *reinterpret_cast<const float2*>(p);
    c[0] = v.x; c[1] = v.y;
  } else {
#pragma unroll
    for (int e = 0; e < E; ++e) c[e] = p[e];
  }
}

template <typename T, int D, int GP>
__global__ void __launch_bounds__(kEstThreads) estimate_kernel(EstParams p) {
  constexpr int E = D / 32;                  // floats per lane per row
  constexpr int R = 32 / GP;                 // rows per reduce-scatter group
  constexpr int RPW = kEstRows / (kEstThreads / 32);  // rows per warp (8)
  constexpr int NG = RPW / R;                // groups per warp
  static_assert(RPW % R == 0, "rows per warp must be a multiple of the group rows");
  extern __shared__ __align__(128) float tile[];     // [kEstRows][D]
  __shared__ __align__(8) uint64_t bar;
  __shared__ float wmax[kEstThreads / 32][GP];

  const int chunk = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  pdl_wait();
  const int S = seq_len_of(p.seq_lens, b, p.max_seq_len);
  if (S <= 0 || S > p.max_seq_len) {
    if (tid == 0 && chunk == 0 && kvh == 0) report(p.status, ADAKV_ST_BAD_SEQ_LEN);
    return;
  }
  const int nb = ceil_div(S, p.bs);
  const int row0 = chunk * kEstRows;
  if (row0 >= nb) return;
  const int nrows = imin(kEstRows, nb - row0);

  if (tid == 0) mbar_init(&bar, 1);
  __syncthreads();
  if (tid == 0) {
    const uint32_t bytes = (uint32_t)nrows * D * 4u;
    mbar_arrive_expect_tx(&bar, bytes);
    bulk_g2s(tile, p.cent + ((int64_t)(b * p.Hkv + kvh) * p.nb_cap + row0) * D, bytes, &bar);
  }

  // this lane's slice of the g queries of the group, in fp32
  float qr[GP][E];
  const T* qbase = static_cast<const T*>(p.q.data) + b * p.q.sb + lane * E;
#pragma unroll
  for (int j = 0; j < GP; ++j) {
#pragma unroll
    for (int e = 0; e < E; ++e)
      qr[j][e] = (j < p.g) ? to_f32(qbase[(int64_t)(kvh * p.g + j) * p.q.sh + e]) : 0.f;
  }

  if (!mbar_wait_bounded(&bar, 0)) {
    if (lane == 0) report(p.status, ADAKV_ST_WAIT_TIMEOUT);
    mbar_wait_bounded(&bar, 0);  // give an in-flight copy one more bounded chance to land
    return;
  }

  float gmax = -INFINITY;
#pragma unroll
  for (int grp = 0; grp < NG; ++grp) {
    const int rbase = warp * RPW + grp * R;
    float v[32];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float c[E];
      lds_row<E>(tile + (rbase + r) * D + lane * E, c);
#pragma unroll
      for (int j = 0; j < GP; ++j) {
        float acc = 0.f;
#pragma unroll
        for (int e = 0; e < E; ++e) acc = fmaf(qr[j][e], c[e], acc);
        v[r * GP + j] = acc;
      }
    }
    const float s = warp_reduce_scatter32(v, lane);
    const int row = rbase + lane / GP, j = lane % GP;
    if (j < p.g && row < nrows) {
      p.scores[(int64_t)(b * p.Hq + kvh * p.g + j) * p.score_stride + row0 + row] = s;
      gmax = fmaxf(gmax, s);
    }
  }
#pragma unroll
  for (int off = GP; off < 32; off <<= 1) gmax = fmaxf(gmax, __shfl_xor_sync(0xffffffffu, gmax, off));
  if (lane < GP) wmax[warp][lane] = gmax;
  __syncthreads();
  if (tid < p.g) {
    float m = wmax[0][tid];
#pragma unroll
    for (int w = 1; w < kEstThreads / 32; ++w) m = fmaxf(m, wmax[w][tid]);
    p.chunkmax[(int64_t)(b * p.Hq + kvh * p.g + tid) * p.chunks_cap + chunk] = m;
  }
  pdl_launch_dependents();
}

template <typename T, int D, int GP>
static cudaError_t launch_est_t(const EstParams& p, int nb_max, cudaStream_t stream) {
  const size_t smem = (size_t)kEstRows * D * sizeof(float);  // <= 32 KB: no opt-in needed
  dim3 grid(ceil_div(imax(nb_max, 1), kEstRows), p.Hkv, p.B);
  estimate_kernel<T, D, GP><<<grid, kEstThreads, smem, stream>>>(p);
  return cudaGetLastError();
}

template <typename T, int D>
static cudaError_t launch_est_d(const EstParams& p, int nb_max, cudaStream_t stream) {
  if (p.g <= 4) return launch_est_t<T, D, 4>(p, nb_max, stream);
  if (p.g <= 8) return launch_est_t<T, D, 8>(p, nb_max, stream);
  if (p.g <= 16) return launch_est_t<T, D, 16>(p, nb_max, stream);
  return cudaErrorInvalidValue;
}

cudaError_t launch_estimate(const EstParams& p, int dtype, int D, int nb_max, cudaStream_t stream) {
#define ADAKV_EST_CASE(TT)                                              \
  if (D == 64) return launch_est_d<TT, 64>(p, nb_max, stream);         \
  if (D == 128) return launch_est_d<TT, 128>(p, nb_max, stream);
  if (dtype == ADAKV_DTYPE_F32) {
    ADAKV_EST_CASE(float)
  } else if (dtype == ADAKV_DTYPE_F16) {
    ADAKV_EST_CASE(__half)
  } else if (dtype == ADAKV_DTYPE_BF16) {
    ADAKV_EST_CASE(__nv_bfloat16)
  }
#undef ADAKV_EST_CASE
  return cudaErrorInvalidValue;
}

}  // namespace adakv
