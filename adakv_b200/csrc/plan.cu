// (c) Entropy-driven per-head budget and ragged per-head top-k block selection.
//
// budget_kernel, one CTA per (b, query head):
//   z = scores / max(T, 1e-6); p = softmax(z) in float32; the head's weight is
//   w = -sum(p * log(max(p, 1e-9))) / log(max(nb, 2)) + 1e-6 (float64 after the
//   division), exactly the formula of adakv/budget.py:28-37.  The softmax maximum
//   comes from the estimator's per-chunk maxima; two passes over the row (from
//   L2) give the normaliser and the entropy.  The last CTA of a sequence to
//   finish (atomic ticket, no spinning) turns the Hq weights into per-head counts
//   (budget.py:71-86 + selector.py:49-54, half-to-even rounding) and the
//   per-head attend work-item offsets; the last sequence to finish turns the
//   per-sequence item totals into global item bases.
//
// select_kernel, one CTA of 1024 threads per (b, query head):
//   keys are the order-preserving uint32 images of the float32 scores, with
//   sink [0, sink) and local [nb-local, nb) blocks forced to 0xFFFFFFFF (the
//   reference's +inf bias, selector.py:44-48).  A 4-pass 8-bit MSB radix select
//   (shared-memory histograms, one warp suffix-scan per pass) finds the k-th
//   largest key T; blocks with key > T, plus the lowest-indexed blocks with
//   key == T, are written in ascending block order with two block-wide scans.
//   The row is staged in shared memory when it fits (nb <= 50K blocks), else
//   every pass re-reads it from L2.  The same CTA writes the attend work items
//   (header + up to item_blocks block ids) of its head.
#include "kernels.h"

namespace adakv {

__device__ __forceinline__ float block_max256(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_max(v);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = red[0];
#pragma unroll
  for (int w = 1; w < kBudgetThreads / 32; ++w) r = fmaxf(r, red[w]);
  __syncthreads();
  return r;
}

__device__ __forceinline__ double block_sum256(double v, double* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  double r = 0.0;
#pragma unroll
  for (int w = 0; w < kBudgetThreads / 32; ++w) r += red[w];
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(kBudgetThreads) budget_kernel(BudgetParams p) {
  __shared__ float fred[kBudgetThreads / 32];
  __shared__ double dred[kBudgetThreads / 32];
  __shared__ int s_flag;
  __shared__ double s_sumw;
  __shared__ int scan_scratch[33];
  const int h = blockIdx.x, b = blockIdx.y, row = b * p.Hq + h, tid = threadIdx.x;
  pdl_wait();
  int S = seq_len_of(p.seq_lens, b, p.max_seq_len);
  if (S < 0 || S > p.max_seq_len) S = 0;  // reported by the estimator
  const int nb = ceil_div(S, p.bs);

  double w = 0.0;
  if (nb >= 2 && p.cfg.policy == ADAKV_POLICY_ADAPTIVE) {
    const int nchunks = ceil_div(nb, kEstRows);
    float m = -INFINITY;
    for (int c = tid; c < nchunks; c += kBudgetThreads)
      m = fmaxf(m, p.chunkmax[(int64_t)row * p.chunks_cap + c]);
    m = block_max256(m, fred);
    const float Tf = (float)(p.cfg.temperature > 1e-6 ? p.cfg.temperature : 1e-6);
    const float zmax = __fdiv_rn(m, Tf);  // max(s / T) == max(s) / T (rounding is monotone)
    const float* s = p.scores + (int64_t)row * p.score_stride;
    double zacc = 0.0;
#pragma unroll 4
    for (int i = tid; i < nb; i += kBudgetThreads) zacc += (double)expf(__fdiv_rn(s[i], Tf) - zmax);
    const float Z = (float)block_sum256(zacc, dred);
    double hacc = 0.0;
#pragma unroll 4
    for (int i = tid; i < nb; i += kBudgetThreads) {
      const float e = expf(__fdiv_rn(s[i], Tf) - zmax);
      const float pi = __fdiv_rn(e, Z);
      hacc += (double)__fmul_rn(pi, logf(fmaxf(pi, 1e-9f)));
    }
    const float hsum = (float)block_sum256(hacc, dred);
    w = (double)(-hsum) / log((double)imax(nb, 2)) + 1e-6;
  }
  if (tid == 0) p.weights[row] = w;

  // ---- last CTA of this sequence: per-head counts and item offsets ----
  __threadfence();
  __syncthreads();
  if (tid == 0) s_flag = (atomicAdd(&p.seq_counter[b], 1) == p.Hq - 1);
  __syncthreads();
  if (!s_flag) return;
  __threadfence();
  if (tid == 0) {
    p.seq_counter[b] = 0;
    double sw = 0.0;
    for (int hh = 0; hh < p.Hq; ++hh) sw += __ldcg(&p.weights[b * p.Hq + hh]);
    s_sumw = sw;
  }
  __syncthreads();
  const SeqBudget sb = seq_budget(nb, p.cfg);
  int carry = 0;
  for (int base = 0; base < p.Hq; base += kBudgetThreads) {
    const int hh = base + tid;
    int items = 0;
    if (hh < p.Hq) {
      const int k = head_count(sb, p.cfg, __ldcg(&p.weights[b * p.Hq + hh]), s_sumw, p.Hq);
      p.sel_lens[b * p.Hq + hh] = k;
      items = ceil_div(k, p.item_blocks);
    }
    const int off = block_exclusive_scan(items, scan_scratch);
    if (hh < p.Hq) p.head_item_off[b * p.Hq + hh] = carry + off;
    carry += scan_scratch[32];
    __syncthreads();
  }
  if (tid == 0) p.seq_items[b] = carry;

  // ---- last sequence overall: global item bases ----
  __threadfence();
  __syncthreads();
  if (tid == 0) s_flag = (atomicAdd(p.glob_counter, 1) == p.B - 1);
  __syncthreads();
  if (!s_flag) return;
  __threadfence();
  if (tid == 0) *p.glob_counter = 0;
  carry = 0;
  for (int base = 0; base < p.B; base += kBudgetThreads) {
    const int bb = base + tid;
    const int t = bb < p.B ? __ldcg(&p.seq_items[bb]) : 0;
    const int off = block_exclusive_scan(t, scan_scratch);
    if (bb < p.B) p.seq_items[bb] = carry + off;  // now the sequence's base
    carry += scan_scratch[32];
    __syncthreads();
  }
  if (tid == 0) {
    p.seq_items[p.B] = carry;
    *p.total_items = carry;
  }
  __syncthreads();
  for (int r = tid; r < p.B * p.Hq; r += kBudgetThreads)
    p.head_item_base[r] = __ldcg(&p.seq_items[r / p.Hq]) + __ldcg(&p.head_item_off[r]);
  pdl_launch_dependents();
}

// order-preserving float -> uint32 map; NaN sorts below everything
__device__ __forceinline__ uint32_t score_key(float f) {
  const uint32_t u = __float_as_uint(f);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return 0u;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

template <bool SMEM>
__global__ void __launch_bounds__(kSelectThreads) select_kernel(SelectParams p) {
  extern __shared__ uint32_t skeys[];
  __shared__ uint32_t hist[256];
  __shared__ int s_digit, s_above;
  __shared__ int scan_scratch[33];
  const int h = blockIdx.x, b = blockIdx.y, row = b * p.Hq + h;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  pdl_wait();
  int S = seq_len_of(p.seq_lens, b, p.max_seq_len);
  if (S < 0 || S > p.max_seq_len) S = 0;
  const int nb = ceil_div(S, p.bs);
  int K = p.sel_lens[row];
  if (K > p.table_width) {
    if (tid == 0) report(p.status, ADAKV_ST_BAD_SEL_LEN);
    K = p.table_width;
  }
  if (K <= 0 || nb <= 0) return;
  const int sink = imin(p.n_sink, nb), local = imin(p.n_local, nb);
  const float* srow = p.scores + (int64_t)row * p.score_stride;
  auto make_key = [&](int i) -> uint32_t {
    return (i < sink || i >= nb - local) ? 0xFFFFFFFFu : score_key(srow[i]);
  };
  if (SMEM) {
    for (int i = tid; i < nb; i += kSelectThreads) skeys[i] = make_key(i);
    __syncthreads();
  }
  auto key = [&](int i) -> uint32_t { return SMEM ? skeys[i] : make_key(i); };

  uint32_t T = 0;
  int need = 0x7FFFFFFF;  // K >= nb: everything is selected
  if (K < nb) {
    uint32_t prefix = 0, pmask = 0;
    int rem = K;
#pragma unroll 1
    for (int pass = 0; pass < 4; ++pass) {
      const int shift = 24 - 8 * pass;
      if (tid < 256) hist[tid] = 0;
      __syncthreads();
      for (int i = tid; i < nb; i += kSelectThreads) {
        const uint32_t k = key(i);
        if ((k & pmask) == prefix) atomicAdd(&hist[(k >> shift) & 0xFFu], 1u);
      }
      __syncthreads();
      if (warp == 0) {
        // lane l owns bins 255-8l .. 248-8l (descending)
        uint32_t c[8], tot = 0;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          c[e] = hist[255 - 8 * lane - e];
          tot += c[e];
        }
        uint32_t incl = tot;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += y;
        }
        const uint32_t excl = incl - tot;
        if (excl < (uint32_t)rem && (uint32_t)rem <= incl) {
          uint32_t acc = excl;
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            if (acc + c[e] >= (uint32_t)rem) {
              s_digit = 255 - 8 * lane - e;
              s_above = (int)acc;
              break;
            }
            acc += c[e];
          }
        }
      }
      __syncthreads();
      rem -= s_above;
      prefix |= (uint32_t)s_digit << shift;
      pmask |= 0xFFu << shift;
      __syncthreads();
    }
    T = prefix;
    need = rem;  // keys equal to T taken, lowest block index first
  }

  // ---- compaction in ascending block order ----
  const int E = ceil_div(nb, kSelectThreads);
  const int beg = imin(tid * E, nb), end = imin(beg + E, nb);
  int n_gt = 0, n_eq = 0;
  for (int i = beg; i < end; ++i) {
    const uint32_t k = key(i);
    n_gt += (k > T);
    n_eq += (k == T);
  }
  const int eq_before = block_exclusive_scan(n_eq, scan_scratch);
  const int eq_take = imax(0, imin(n_eq, need - eq_before));
  const int pos0 = block_exclusive_scan(n_gt + eq_take, scan_scratch);
  const int C = p.item_blocks;
  const int item0 = p.head_item_base[row];
  int* trow = p.block_table + (int64_t)row * p.table_width;
  int pos = pos0, r = eq_before;
  for (int i = beg; i < end; ++i) {
    const uint32_t k = key(i);
    bool sel = k > T;
    if (k == T) {
      sel = r < need;
      ++r;
    }
    if (sel) {
      if (pos < K) {
        trow[pos] = i;
        p.work_blk[(int64_t)(item0 + pos / C) * C + pos % C] = i;
      }
      ++pos;
    }
  }
  const int n_items = ceil_div(K, C);
  for (int j = tid; j < n_items; j += kSelectThreads)
    p.work_hdr[item0 + j] = make_int4(b, h, item0, K);
  pdl_launch_dependents();
}

cudaError_t launch_budget(const BudgetParams& p, cudaStream_t stream) {
  dim3 grid(p.Hq, p.B);
  budget_kernel<<<grid, kBudgetThreads, 0, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t select_kernels_init() {
  return cudaFuncSetAttribute(select_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              kSelectSmemMaxKeys * (int)sizeof(uint32_t));
}

cudaError_t launch_select(const SelectParams& p, int nb_max, cudaStream_t stream) {
  dim3 grid(p.Hq, p.B);
  if (nb_max <= kSelectSmemMaxKeys) {
    select_kernel<true><<<grid, kSelectThreads, (size_t)imax(nb_max, 1) * sizeof(uint32_t), stream>>>(p);
  } else {
    select_kernel<false><<<grid, kSelectThreads, 0, stream>>>(p);
  }
  return cudaGetLastError();
}

}  // namespace adakv
