// (d) Fused ragged block-sparse split-KV flash decode.
//
// out[b, h] = softmax_t((q[b, h] . K[b, h/g, t]) * sm_scale) . V[b, h/g, t] over the
// tokens t of the selected blocks of query head h (tokens >= seq_len masked), the
// semantics of the reference kernel (adakv/kernels/block_sparse_decode.py:51-100)
// and of the oracle (adakv/reference.py:76-80).
//
// Work decomposition: head h's selected list is cut into work items of up to C
// blocks (C = item_blocks); item i carries {b, h, first item of the head, count}
// plus its C block ids, so a CTA reaches its K/V with one dependent load.  The
// grid is persistent (grid-stride over items).  Per item, 128 threads issue
// cp.async 16-byte copies of all C blocks' K and V rows into shared memory
// (zero-fill past seq_len), then each of the 4 warps runs an online softmax over
// one block at a time: a token row is spread over D*sizeof(T)/16 lanes (16 for
// bf16 D=128), dot products finish with xor shuffles, and the lane keeps its
// 16-byte slice of the output accumulator.  Warps merge in shared memory into
// the item's (m, l, o); a head with one item writes its output directly,
// otherwise the item's partial goes to the workspace and the last item of the
// head to finish (atomic ticket) merges all partials in item order and writes
// the output -- no second kernel, no spinning.
//
// HBM traffic: the selected K/V blocks (bs * D * sizeof(T) * 2 bytes each), q,
// out; partials stay in L2.
#include "kernels.h"

namespace adakv {

template <typename T, int D, int BS>
__global__ void __launch_bounds__(kAttendThreads) attend_kernel(AttendParams p) {
  constexpr int VEC = 16 / sizeof(T);       // elements per 16-byte chunk
  constexpr int LPT = D / VEC;              // lanes per token row
  constexpr int TPP = 32 / LPT;             // token rows per warp pass
  constexpr int PASSES = BS / TPP;
  constexpr int ROWC = D / VEC;             // 16-byte chunks per token row
  constexpr int NW = kAttendThreads / 32;
  static_assert(LPT <= 32 && BS % TPP == 0, "unsupported tile shape");
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* Ks = reinterpret_cast<T*>(smem_raw);
  T* Vs = Ks + (size_t)p.item_blocks * BS * D;
  __shared__ int s_blk[kMaxItemBlocks];
  __shared__ float s_m[NW], s_l[NW];
  __shared__ float s_o[NW][D];
  __shared__ int s_last;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int C = p.item_blocks;
  const int d0 = (lane % LPT) * VEC;
  const int tl = lane / LPT;
  pdl_wait();

  // heads with an empty selection produce zeros
  for (int r = blockIdx.x; r < p.B * p.Hq; r += gridDim.x) {
    if (p.sel_lens[r] <= 0 && tid < D) {
      const int b = r / p.Hq, h = r % p.Hq;
      static_cast<T*>(const_cast<void*>(p.out.data))[b * p.out.sb + h * p.out.sh + tid] = from_f32<T>(0.f);
    }
  }

  const int total = *p.total_items;
  for (int item = blockIdx.x; item < total; item += gridDim.x) {
    const int4 hdr = p.work_hdr[item];
    const int b = hdr.x, h = hdr.y, base = hdr.z, K = hdr.w;
    const int first = (item - base) * C;
    const int cnt = imin(C, K - first);
    const int kvh = h / p.g;
    int S = seq_len_of(p.seq_lens, b, p.max_seq_len);
    if (S < 0 || S > p.max_seq_len) S = 0;
    const int nb = ceil_div(S, BS);
    if (tid < cnt) {
      int blk = p.work_blk[(int64_t)item * C + tid];
      if (blk < 0 || blk >= nb) {
        report(p.status, ADAKV_ST_BAD_BLOCK_ID);
        blk = -1;
      }
      s_blk[tid] = blk;
    }
    __syncthreads();

    const T* kbase = static_cast<const T*>(p.k.data) + b * p.k.sb + kvh * p.k.sh;
    const T* vbase = static_cast<const T*>(p.v.data) + b * p.v.sb + kvh * p.v.sh;
    const int nchunks = cnt * BS * ROWC;
    for (int c = tid; c < nchunks; c += kAttendThreads) {
      const int slot = c / (BS * ROWC);
      const int rem = c - slot * (BS * ROWC);
      const int tok = rem / ROWC, col = rem - tok * ROWC;
      const int blk = s_blk[slot];
      const int pos = blk * BS + tok;
      const bool valid = blk >= 0 && pos < S;
      const int64_t srow = valid ? (int64_t)pos : 0;
      const size_t soff = ((size_t)slot * BS + tok) * D + col * VEC;
      cp_async16(Ks + soff, kbase + srow * p.k.ss + col * VEC, valid);
      cp_async16(Vs + soff, vbase + srow * p.v.ss + col * VEC, valid);
    }
    cp_async_commit();

    float qf[VEC];
    {
      const uint4 u = *reinterpret_cast<const uint4*>(static_cast<const T*>(p.q.data) + b * p.q.sb +
                                                      h * p.q.sh + d0);
      Unpack16<T>::run(u, qf);
    }
    cp_async_wait_all();
    __syncthreads();

    float m_run = -INFINITY, l_run = 0.f;
    float o[VEC];
#pragma unroll
    for (int e = 0; e < VEC; ++e) o[e] = 0.f;

    for (int slot = warp; slot < cnt; slot += NW) {
      const int blk = s_blk[slot];
      if (blk < 0) continue;
      float sc[PASSES];
#pragma unroll
      for (int pp = 0; pp < PASSES; ++pp) {
        const int tok = pp * TPP + tl;
        const uint4 u = *reinterpret_cast<const uint4*>(Ks + ((size_t)slot * BS + tok) * D + d0);
        float kf[VEC];
        Unpack16<T>::run(u, kf);
        float part = 0.f;
#pragma unroll
        for (int e = 0; e < VEC; ++e) part = fmaf(qf[e], kf[e], part);
#pragma unroll
        for (int off = LPT / 2; off >= 1; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
        sc[pp] = (blk * BS + tok < S) ? part * p.sm_scale : -INFINITY;
      }
      float mb = sc[0];
#pragma unroll
      for (int pp = 1; pp < PASSES; ++pp) mb = fmaxf(mb, sc[pp]);
#pragma unroll
      for (int off = LPT; off < 32; off <<= 1) mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, off));
      const float m_new = fmaxf(m_run, mb);
      if (m_new == -INFINITY) continue;  // every token so far is masked (warp-uniform)
      const float alpha = expf(m_run - m_new);  // m_run = -inf -> 0
      float l_part = 0.f;
#pragma unroll
      for (int e = 0; e < VEC; ++e) o[e] *= alpha;
#pragma unroll
      for (int pp = 0; pp < PASSES; ++pp) {
        const int tok = pp * TPP + tl;
        const float pt = expf(sc[pp] - m_new);
        l_part += pt;
        const uint4 u = *reinterpret_cast<const uint4*>(Vs + ((size_t)slot * BS + tok) * D + d0);
        float vf[VEC];
        Unpack16<T>::run(u, vf);
#pragma unroll
        for (int e = 0; e < VEC; ++e) o[e] = fmaf(pt, vf[e], o[e]);
      }
      l_run = l_run * alpha + l_part;
      m_run = m_new;
    }
    // merge the token groups of the warp (lanes that share dims d0..)
#pragma unroll
    for (int off = LPT; off < 32; off <<= 1) {
      l_run += __shfl_xor_sync(0xffffffffu, l_run, off);
#pragma unroll
      for (int e = 0; e < VEC; ++e) o[e] += __shfl_xor_sync(0xffffffffu, o[e], off);
    }
    if (lane < LPT) {
#pragma unroll
      for (int e = 0; e < VEC; ++e) s_o[warp][d0 + e] = o[e];
    }
    if (lane == 0) {
      s_m[warp] = m_run;
      s_l[warp] = l_run;
    }
    __syncthreads();

    float M = s_m[0];
#pragma unroll
    for (int w = 1; w < NW; ++w) M = fmaxf(M, s_m[w]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < NW; ++w) {
        const float f = (s_m[w] == -INFINITY) ? 0.f : expf(s_m[w] - M);
        L += s_l[w] * f;
        if (tid < D) O += s_o[w][tid] * f;
      }
    }
    const int n_items = ceil_div(K, C);
    T* orow = static_cast<T*>(const_cast<void*>(p.out.data)) + b * p.out.sb + h * p.out.sh;
    if (n_items == 1) {
      if (tid < D) orow[tid] = from_f32<T>(L > 0.f ? O / L : 0.f);
    } else {
      if (tid < D) p.part_o[(int64_t)item * D + tid] = O;
      if (tid == 0) p.part_ml[item] = make_float2(M, L);
      __threadfence();
      __syncthreads();
      if (tid == 0) s_last = (atomicAdd(&p.head_counter[b * p.Hq + h], 1) == n_items - 1);
      __syncthreads();
      if (s_last) {
        __threadfence();
        float M2 = -INFINITY;
        for (int it = 0; it < n_items; ++it) M2 = fmaxf(M2, __ldcg(&p.part_ml[base + it]).x);
        float L2 = 0.f, O2 = 0.f;
        if (M2 != -INFINITY) {
          for (int it = 0; it < n_items; ++it) {
            const float2 ml = __ldcg(&p.part_ml[base + it]);
            const float f = (ml.x == -INFINITY) ? 0.f : expf(ml.x - M2);
            L2 += ml.y * f;
            if (tid < D) O2 += __ldcg(&p.part_o[(int64_t)(base + it) * D + tid]) * f;
          }
        }
        if (tid < D) orow[tid] = from_f32<T>(L2 > 0.f ? O2 / L2 : 0.f);
        if (tid == 0) p.head_counter[b * p.Hq + h] = 0;
      }
    }
    __syncthreads();  // shared tiles are reused by the next item
  }
}

// Stand-alone attend: build work items from a caller-given (block_table, sel_lens).
// Pass 1 (one CTA): clamp counts, exclusive scan of per-head item counts.
__global__ void __launch_bounds__(1024) items_scan_kernel(AttendParams p) {
  __shared__ int scan_scratch[33];
  const int rows = p.B * p.Hq;
  int carry = 0;
  for (int base = 0; base < rows; base += blockDim.x) {
    const int r = base + threadIdx.x;
    int items = 0;
    if (r < rows) {
      int k = p.sel_lens[r];
      if (k > p.table_width || k < 0) {
        report(p.status, ADAKV_ST_BAD_SEL_LEN);
        k = k < 0 ? 0 : p.table_width;
      }
      items = ceil_div(k, p.item_blocks);
    }
    const int off = block_exclusive_scan(items, scan_scratch);
    if (r < rows) p.head_item_base[r] = carry + off;
    carry += scan_scratch[32];
    __syncthreads();
  }
  if (threadIdx.x == 0) *p.total_items_w = carry;
}

// Pass 2 (one CTA per head): copy the head's block ids into its items.
__global__ void __launch_bounds__(256) items_fill_kernel(AttendParams p) {
  const int h = blockIdx.x, b = blockIdx.y, r = b * p.Hq + h;
  int k = p.sel_lens[r];
  k = k < 0 ? 0 : (k > p.table_width ? p.table_width : k);
  const int C = p.item_blocks;
  const int base = p.head_item_base[r];
  const int* trow = p.block_table + (int64_t)r * p.table_width;
  for (int i = threadIdx.x; i < k; i += blockDim.x)
    p.work_blk_w[(int64_t)(base + i / C) * C + i % C] = trow[i];
  for (int j = threadIdx.x; j < ceil_div(k, C); j += blockDim.x)
    p.work_hdr_w[base + j] = make_int4(b, h, base, k);
}

template <typename T, int D, int BS>
static cudaError_t launch_attend_t(const AttendParams& p, int grid, cudaStream_t stream) {
  const size_t smem = (size_t)p.item_blocks * BS * D * sizeof(T) * 2;
  attend_kernel<T, D, BS><<<grid, kAttendThreads, smem, stream>>>(p);
  return cudaGetLastError();
}

template <typename F>
static cudaError_t for_each_attend(int dtype, int D, int bs, F&& f) {
#define ADAKV_ATT_CASE(TT, DD, BB) \
  if (D == DD && bs == BB) return f(attend_kernel<TT, DD, BB>, (int)sizeof(TT));
#define ADAKV_ATT_T(TT) \
  ADAKV_ATT_CASE(TT, 64, 16) ADAKV_ATT_CASE(TT, 64, 32) ADAKV_ATT_CASE(TT, 128, 16) ADAKV_ATT_CASE(TT, 128, 32)
  if (dtype == ADAKV_DTYPE_F32) {
    ADAKV_ATT_T(float)
  } else if (dtype == ADAKV_DTYPE_F16) {
    ADAKV_ATT_T(__half)
  } else if (dtype == ADAKV_DTYPE_BF16) {
    ADAKV_ATT_T(__nv_bfloat16)
  }
#undef ADAKV_ATT_T
#undef ADAKV_ATT_CASE
  return cudaErrorInvalidValue;
}

cudaError_t attend_kernels_init() {
  for (int dt = 0; dt < 3; ++dt)
    for (int D : {64, 128})
      for (int bs : {16, 32}) {
        cudaError_t e = for_each_attend(dt, D, bs, [](auto kern, int) {
          return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)kAttendSmemMax);
        });
        if (e != cudaSuccess) return e;
      }
  return cudaSuccess;
}

int attend_ctas_per_sm(int dtype, int D, int bs, int item_blocks) {
  int n = 0;
  for_each_attend(dtype, D, bs, [&](auto kern, int elt) {
    const size_t smem = (size_t)item_blocks * bs * D * elt * 2;
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kAttendThreads, smem);
  });
  return n > 0 ? n : 1;
}

cudaError_t launch_attend(const AttendParams& p, int dtype, int D, int bs, int grid,
                          cudaStream_t stream) {
#define ADAKV_ATT_CASE(TT, DD, BB) \
  if (D == DD && bs == BB) return launch_attend_t<TT, DD, BB>(p, grid, stream);
#define ADAKV_ATT_T(TT) \
  ADAKV_ATT_CASE(TT, 64, 16) ADAKV_ATT_CASE(TT, 64, 32) ADAKV_ATT_CASE(TT, 128, 16) ADAKV_ATT_CASE(TT, 128, 32)
  if (dtype == ADAKV_DTYPE_F32) {
    ADAKV_ATT_T(float)
  } else if (dtype == ADAKV_DTYPE_F16) {
    ADAKV_ATT_T(__half)
  } else if (dtype == ADAKV_DTYPE_BF16) {
    ADAKV_ATT_T(__nv_bfloat16)
  }
#undef ADAKV_ATT_T
#undef ADAKV_ATT_CASE
  return cudaErrorInvalidValue;
}

cudaError_t launch_items(const AttendParams& p, cudaStream_t stream) {
  items_scan_kernel<<<1, 1024, 0, stream>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  items_fill_kernel<<<dim3(p.Hq, p.B), 256, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace adakv
