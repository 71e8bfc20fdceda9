// (f4) Per-key attention importance of the H2O / SnapKV eviction baselines.
//
// For query rows i in [q0, S) of each query head h (q0 = 0 for H2O, S - w for
// SnapKV's observation window) attending causally to keys j <= i:
//
//   imp[h, j] = sum_{i >= max(j, q0)} exp(s_ij - m_i) / l_i,  s_ij = scale * q_i . k_j,
//   m_i = max_{j <= i} s_ij,  l_i = sum_{j <= i} exp(s_ij - m_i)
//
// (adakv/baselines.py:69-83 and 101-117; the reference's torch runtime,
// adakv/baselines_rt.py:43-81, computes the same quantity in query chunks).
// Keys are read per KV head (h / g), never expanded to the query heads.
//
// Two passes, both over 64 x 64 (query x key) tiles staged in shared memory as
// float32 and transposed (d-major) so each thread's 4 x 4 micro-tile reads
// float4s:
//   rowstat_kernel  grid (query tiles, Hq, B): online (m_i, l_i) over the key
//                   tiles up to the causal limit -> m, l in the workspace;
//   colsum_kernel   grid (key tiles, Hq, B): for its 64 keys, the query tiles
//                   at or after them, probabilities summed over the rows in a
//                   fixed order (per-thread partials, one shared-memory fold at
//                   the end): deterministic, no atomics.
// The O(S^2 D) work runs on the CUDA cores in float32, like the reference's
// float32 einsum; logits and exponentials are float32 (the NumPy oracle uses
// float64; the difference is ~1e-6 relative).
#include "kernels.h"

namespace adakv {
namespace {

constexpr int kTile = 64;
constexpr int kLd = kTile + 4;    // padded d-major row: 4-way (not 32-way) conflicts on staging
constexpr int kImpThreads = 256;  // 16 x 16 threads, 4 x 4 outputs each

template <typename T>
__device__ __forceinline__ float to_f(T x);
template <>
__device__ __forceinline__ float to_f<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <>
__device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }

// rows [r0, r0 + 64) of a [rows, D] head slice -> dst[d * kLd + r] (float32,
// transposed); rows outside [0, nrows) read as zero
template <typename T, int D>
__device__ __forceinline__ void stage_tile(float* dst, const T* base, int64_t row_stride, int r0,
                                           int nrows) {
  for (int e = threadIdx.x; e < kTile * D; e += kImpThreads) {
    const int r = e / D, d = e - r * D;
    const int row = r0 + r;
    dst[d * kLd + r] = (row >= 0 && row < nrows) ? to_f<T>(base[(int64_t)row * row_stride + d]) : 0.f;
  }
}

// acc[a][b] = sum_d Qt[d][ty*4 + a] * Kt[d][tx*4 + b]
template <int D>
__device__ __forceinline__ void tile_dot(const float* Qt, const float* Kt, int ty, int tx,
                                         float (&acc)[4][4]) {
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b) acc[a][b] = 0.f;
#pragma unroll 8
  for (int d = 0; d < D; ++d) {
    const float4 q = *reinterpret_cast<const float4*>(Qt + d * kLd + ty * 4);
    const float4 k = *reinterpret_cast<const float4*>(Kt + d * kLd + tx * 4);
    const float qa[4] = {q.x, q.y, q.z, q.w}, kb[4] = {k.x, k.y, k.z, k.w};
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int b = 0; b < 4; ++b) acc[a][b] = fmaf(qa[a], kb[b], acc[a][b]);
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(kImpThreads) rowstat_kernel(ImportanceParams p) {
  extern __shared__ __align__(16) float smem[];
  float* Qt = smem;
  float* Kt = smem + D * kLd;
  const int b = blockIdx.z, h = blockIdx.y, g = p.Hq / p.Hkv;
  const int S = p.S, q0 = S - p.n_query;
  const int i0 = q0 + blockIdx.x * kTile;  // absolute position of the tile's first query
  const int tid = threadIdx.x, ty = tid / 16, tx = tid % 16;
  const T* qb = static_cast<const T*>(p.q.data) + b * p.q.sb + (int64_t)h * p.q.sh;
  const T* kb = static_cast<const T*>(p.k.data) + b * p.k.sb + (int64_t)(h / g) * p.k.sh;
  stage_tile<T, D>(Qt, qb, p.q.ss, i0, S);
  float m[4], l[4];
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    m[a] = -INFINITY;
    l[a] = 0.f;
  }
  const int last = imin(i0 + kTile, S) - 1;  // the tile's last query sees keys <= last
  for (int j0 = 0; j0 <= last; j0 += kTile) {
    __syncthreads();  // the previous key tile is consumed
    stage_tile<T, D>(Kt, kb, p.k.ss, j0, S);
    __syncthreads();
    float s[4][4];
    tile_dot<D>(Qt, Kt, ty, tx, s);
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      const int i = i0 + ty * 4 + a;
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int j = j0 + tx * 4 + c;
        s[a][c] = (j <= i && i < S) ? s[a][c] * p.scale : -INFINITY;
        mx = fmaxf(mx, s[a][c]);
      }
#pragma unroll
      for (int o = 1; o < 16; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float mn = fmaxf(m[a], mx);
      float sum = 0.f;
      if (mn > -INFINITY) {
#pragma unroll
        for (int c = 0; c < 4; ++c) sum += s[a][c] > -INFINITY ? expf(s[a][c] - mn) : 0.f;
      }
#pragma unroll
      for (int o = 1; o < 16; o <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      if (mn > -INFINITY) {
        l[a] = (m[a] > -INFINITY ? l[a] * expf(m[a] - mn) : 0.f) + sum;
        m[a] = mn;
      }
    }
  }
  if (tx == 0) {
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      const int r = blockIdx.x * kTile + ty * 4 + a;  // row within the query window
      if (q0 + r < S) {
        const int64_t o = ((int64_t)b * p.Hq + h) * p.n_query + r;
        p.row_m[o] = m[a];
        p.row_l[o] = l[a];
      }
    }
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(kImpThreads) colsum_kernel(ImportanceParams p) {
  extern __shared__ __align__(16) float smem[];
  float* Qt = smem;
  float* Kt = smem + D * kLd;
  float* red = smem + 2 * D * kLd;  // [16][64] column partials
  const int b = blockIdx.z, h = blockIdx.y, g = p.Hq / p.Hkv;
  const int S = p.S, q0 = S - p.n_query;
  const int j0 = blockIdx.x * kTile;
  const int tid = threadIdx.x, ty = tid / 16, tx = tid % 16;
  const T* qb = static_cast<const T*>(p.q.data) + b * p.q.sb + (int64_t)h * p.q.sh;
  const T* kb = static_cast<const T*>(p.k.data) + b * p.k.sb + (int64_t)(h / g) * p.k.sh;
  const float* rm = p.row_m + ((int64_t)b * p.Hq + h) * p.n_query;
  const float* rl = p.row_l + ((int64_t)b * p.Hq + h) * p.n_query;
  stage_tile<T, D>(Kt, kb, p.k.ss, j0, S);
  float col[4] = {0.f, 0.f, 0.f, 0.f};
  // query tiles (of the window's tiling) whose rows reach these keys
  const int first = imax(0, (j0 - q0) / kTile);
  const int ntiles = ceil_div(p.n_query, kTile);
  for (int t = first; t < ntiles; ++t) {
    const int i0 = q0 + t * kTile;
    __syncthreads();
    stage_tile<T, D>(Qt, qb, p.q.ss, i0, S);
    __syncthreads();
    float s[4][4];
    tile_dot<D>(Qt, Kt, ty, tx, s);
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      const int r = t * kTile + ty * 4 + a, i = q0 + r;
      if (i >= S) continue;
      const float mi = rm[r], inv = 1.f / rl[r];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int j = j0 + tx * 4 + c;
        if (j <= i) col[c] += expf(s[a][c] * p.scale - mi) * inv;
      }
    }
  }
  // fold the 16 row groups in a fixed order
#pragma unroll
  for (int c = 0; c < 4; ++c) red[ty * kTile + tx * 4 + c] = col[c];
  __syncthreads();
  if (tid < kTile) {
    float v = 0.f;
    for (int y = 0; y < 16; ++y) v += red[y * kTile + tid];
    const int j = j0 + tid;
    if (j < S) p.imp[((int64_t)b * p.Hq + h) * p.imp_stride + j] = v;
  }
}

template <typename T, int D>
cudaError_t launch_importance_t(const ImportanceParams& p, cudaStream_t st) {
  const size_t sm_row = sizeof(float) * 2 * D * kLd;
  const size_t sm_col = sm_row + sizeof(float) * 16 * kTile;
  cudaError_t e = cudaFuncSetAttribute(rowstat_kernel<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)sm_row);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(colsum_kernel<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm_col);
  if (e != cudaSuccess) return e;
  rowstat_kernel<T, D><<<dim3(ceil_div(p.n_query, kTile), p.Hq, p.B), kImpThreads, sm_row, st>>>(p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  colsum_kernel<T, D><<<dim3(ceil_div(p.S, kTile), p.Hq, p.B), kImpThreads, sm_col, st>>>(p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_importance(const ImportanceParams& p, int dtype, int D, cudaStream_t st) {
#define ADAKV_IMP_CASE(TT, DD) \
  if (D == DD) return launch_importance_t<TT, DD>(p, st);
  if (dtype == ADAKV_DTYPE_F32) {
    ADAKV_IMP_CASE(float, 64) ADAKV_IMP_CASE(float, 128)
  } else if (dtype == ADAKV_DTYPE_BF16) {
    ADAKV_IMP_CASE(__nv_bfloat16, 64) ADAKV_IMP_CASE(__nv_bfloat16, 128)
  } else if (dtype == ADAKV_DTYPE_F16) {
    ADAKV_IMP_CASE(__half, 64) ADAKV_IMP_CASE(__half, 128)
  }
#undef ADAKV_IMP_CASE
  return cudaErrorInvalidValue;
}

}  // namespace adakv
