// Sequence-sharded budget + top-k without exchanging score rows.
//
// One long sequence's blocks are split over ranks, rank r holding the global
// blocks [lo_r, lo_r + n_r).  The single-device plan kernel needs two things
// of each query head's whole score row: its softmax statistics, for the
// entropy budget (adakv/budget.py:28-86), and its top content blocks
// (adakv/selector.py:18-60).  Both decompose over shards:
//
// * max, content statistics, Z = sum e^(z - M) and A = sum e^(z - M)(z - M)
//   merge across shards the way the plan kernel merges its per-CTA partials
//   (rescaled to the largest max, summed in double);
// * the clamp term of the entropy (blocks whose probability is below 1e-9)
//   depends on the merged max and Z, so each shard evaluates its own share
//   once the statistics are known everywhere (a second, Hq-double exchange);
// * a head picks Kc <= Kc_max content blocks of the whole row, and they are
//   among the union of every shard's own top Kc_max content blocks.  Each
//   shard contributes its top Kc_max as a list sorted by (score desc, block
//   asc); a candidate's position in the merged order is its index in its own
//   list plus the number of larger keys in each other list (one binary search
//   per list), so a rank finds which of its candidates are in the head's top
//   Kc without a further exchange.
//
// Every rank runs the same arithmetic on the same gathered records and so
// derives the same budgets; the union of the ranks' tables is the head's
// selection.  Three kernels, one CTA per query head each; the collectives
// between them are the caller's:
//   stage 0  shard_prep_kernel    statistics + sorted candidate list
//   stage 1  shard_clamp_kernel   this shard's clamp term, from all statistics
//   stage 2  shard_finish_kernel  every head's weight, this head's count and
//                                 this shard's part of the block table
#include "kernels.h"

namespace adakv {

namespace {

// candidate key: descending order = score descending, then block ascending
__device__ __forceinline__ unsigned long long cand_key(float s, int gidx) {
  return (static_cast<unsigned long long>(order_key(s)) << 32) |
         static_cast<unsigned long long>(~static_cast<uint32_t>(gidx));
}
__device__ __forceinline__ int key_block(unsigned long long k) {
  return static_cast<int>(~static_cast<uint32_t>(k));
}

__device__ __forceinline__ float zof(float v, float Tf, bool unit_t) {
  return unit_t ? v : __fdiv_rn(v, Tf);
}

// block-wide int sum, every thread gets it (`red`: 32 ints of shared memory)
__device__ __forceinline__ int block_sum_int(int v, int* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = __reduce_add_sync(0xffffffffu, v);
  __syncthreads();  // red may still be read by the previous call
  if (lane == 0) red[warp] = v;
  __syncthreads();
  return __reduce_add_sync(0xffffffffu, lane < nw ? red[lane] : 0);
}

__device__ __forceinline__ const double* stats_of(const ShardSelParams& p, int r, int h) {
  return reinterpret_cast<const double*>(p.xall + (size_t)r * p.xstride) + (size_t)h * kShardStatD;
}
__device__ __forceinline__ const unsigned long long* cands_of(const ShardSelParams& p, int r, int h) {
  return reinterpret_cast<const unsigned long long*>(p.xall + (size_t)r * p.xstride +
                                                     (size_t)p.Hq * kShardStatD * sizeof(double)) +
         (size_t)h * p.cap_pad;
}

// Merged max score, max z, Z and A of head hh over every rank's record, in
// rank order: the same inputs give the same result wherever it runs, so
// every rank agrees.
__device__ __forceinline__ void merge_head(const ShardSelParams& p, int hh, float& mx, float& M,
                                           double& Z, double& A) {
  mx = -INFINITY;
  M = -INFINITY;
#pragma unroll 8
  for (int r = 0; r < p.world; ++r) {
    const double* st = stats_of(p, r, hh);
    mx = fmaxf(mx, (float)st[0]);
    M = fmaxf(M, (float)st[4]);
  }
  Z = 0.0;
  A = 0.0;
#pragma unroll 8
  for (int r = 0; r < p.world; ++r) {
    const double* st = stats_of(p, r, hh);
    const float Mr = (float)st[4];
    if (Mr > -INFINITY) {
      const double sc = exp((double)Mr - (double)M);
      Z += st[5] * sc;
      A += sc * (st[6] + st[5] * ((double)Mr - (double)M));
    }
  }
}

constexpr int kSweepU = 8;  // row loads in flight per thread in a sweep

// ---- stage 0: statistics and the shard's top content candidates ----------
// UNIT_T: temperature 1 (z = s exactly, no division)
template <bool UNIT_T>
__global__ void __launch_bounds__(kShardThreads, 1) shard_prep_kernel(ShardSelParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  unsigned long long* list = reinterpret_cast<unsigned long long*>(smem);  // [kShardListCap] gathered
  unsigned long long* sorted = list + kShardListCap;                     // [kShardListCap] by bucket
  int* bpos = reinterpret_cast<int*>(sorted + kShardListCap);            // [kShardSortBuckets]
  int* bfill = bpos + kShardSortBuckets;                                 // [kShardSortBuckets]
  float* srow = reinterpret_cast<float*>(bfill + kShardSortBuckets);     // staged row
  __shared__ float wf[32][3];
  __shared__ double wd[32][4];
  __shared__ int red[33];
  __shared__ int s_n;
  __shared__ float s_mx, s_cmx, s_cmn, s_M;
  __shared__ double s_csum, s_csq, s_Z, s_A;

  const int h = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n = p.n_local, lo = p.block_lo, nb = p.nb;
  const int sink = imin(p.cfg.n_sink, nb), local = imin(p.cfg.n_local, nb);
  // content (neither sink nor local-window) blocks of the shard: [c0, c1)
  const int c0 = imin(n, imax(0, sink - lo)), c1 = imax(c0, imin(n, nb - local - lo));
  const int ncont = c1 - c0;
  const bool staged = n <= kShardStageCap;
  const float* row = p.scores + (int64_t)h * p.score_stride;
  const bool soft = nb >= 2 && p.cfg.policy == ADAKV_POLICY_ADAPTIVE;
  const float Tf = (float)(p.cfg.temperature > 1e-6 ? p.cfg.temperature : 1e-6);
  auto zof = [&](float v) -> float { return UNIT_T ? v : __fdiv_rn(v, Tf); };
  auto val = [&](int li) -> float { return staged ? srow[li] : row[li]; };
  pdl_wait();  // the scores come from the estimator

  // ---- 1. stage the row (kSweepU loads in flight per thread) and fold the
  //      max score and the content max / min / sum / sum of squares ----
  float mx = -INFINITY, cmx = -INFINITY, cmn = INFINITY, csum = 0.f, csq = 0.f;
  for (int base = 0; base < n; base += kShardThreads * kSweepU) {
    float v[kSweepU];
#pragma unroll
    for (int u = 0; u < kSweepU; ++u) {
      const int li = base + u * kShardThreads + tid;
      v[u] = li < n ? row[li] : -INFINITY;
    }
#pragma unroll
    for (int u = 0; u < kSweepU; ++u) {
      const int li = base + u * kShardThreads + tid;
      if (li < n) {
        if (staged) srow[li] = v[u];
        mx = fmaxf(mx, v[u]);
        if (li >= c0 && li < c1) {
          cmx = fmaxf(cmx, v[u]);
          cmn = fminf(cmn, v[u]);
          csum += v[u];
          csq = fmaf(v[u], v[u], csq);
        }
      }
    }
  }
  {
    const float wmx = warp_max(mx), wcmx = warp_max(cmx), wcmn = -warp_max(-cmn);
    const double ws = warp_sum((double)csum), wq = warp_sum((double)csq);
    if (lane == 0) {
      wf[warp][0] = wcmn;
      wf[warp][1] = wmx;
      wf[warp][2] = wcmx;
      wd[warp][2] = ws;
      wd[warp][3] = wq;
    }
  }
  __syncthreads();  // also publishes the staged row
  if (warp == 0) {
    const float m1 = warp_max(wf[lane][1]), m2 = warp_max(wf[lane][2]);
    const float m0 = -warp_max(-wf[lane][0]);
    const double cs = warp_sum(wd[lane][2]), cq = warp_sum(wd[lane][3]);
    if (lane == 0) {
      s_mx = m1;
      s_cmx = m2;
      s_cmn = m0;
      s_M = zof(m1);  // max z (division by T > 0 is monotone)
      s_csum = cs;
      s_csq = cq;
      s_Z = 0.0;
      s_A = 0.0;
    }
  }
  __syncthreads();

  // ---- 2. Z and A relative to the shard's max z ----
  if (soft && s_M > -INFINITY) {
    const float M = s_M;
    float z_t = 0.f, a_t = 0.f;
    for (int base = 0; base < n; base += kShardThreads * kSweepU) {
      float v[kSweepU];
#pragma unroll
      for (int u = 0; u < kSweepU; ++u) {
        const int li = base + u * kShardThreads + tid;
        v[u] = li < n ? val(li) : -INFINITY;
      }
#pragma unroll
      for (int u = 0; u < kSweepU; ++u) {
        const float d = zof(v[u]) - M;
        const float e = expf(d);
        z_t += e;
        a_t = e > 0.f ? fmaf(e, d, a_t) : a_t;
      }
    }
    const double zw = warp_sum((double)z_t), aw = warp_sum((double)a_t);
    if (lane == 0) {
      wd[warp][0] = zw;
      wd[warp][1] = aw;
    }
    __syncthreads();
    if (warp == 0) {
      const double z = warp_sum(wd[lane][0]), a = warp_sum(wd[lane][1]);
      if (lane == 0) {
        s_Z = z;
        s_A = a;
      }
    }
    __syncthreads();
  }
  const int kc = imin(p.cap, ncont);
  double* st = reinterpret_cast<double*>(p.xmine) + (size_t)h * kShardStatD;
  unsigned long long* out = reinterpret_cast<unsigned long long*>(
                                p.xmine + (size_t)p.Hq * kShardStatD * sizeof(double)) +
                            (size_t)h * p.cap_pad;
  if (tid == 0) {
    st[0] = (double)s_mx;
    st[1] = (double)s_cmx;
    st[2] = s_csum;
    st[3] = s_csq;
    st[4] = (double)s_M;
    st[5] = s_Z;
    st[6] = s_A;
    st[7] = (double)kc;
  }
  if (kc == 0) return;  // uniform over the CTA

  // content keys >= T (> T when strict) into the list in any order, at most
  // kShardListCap of them; returns how many there are
  auto gather = [&](uint32_t T, bool strict) -> int {
    __syncthreads();  // the list and s_n may still be in use
    if (tid == 0) s_n = 0;
    __syncthreads();
    for (int base = c0; base < c1; base += kShardThreads * kSweepU) {
      float v[kSweepU];
#pragma unroll
      for (int u = 0; u < kSweepU; ++u) {
        const int li = base + u * kShardThreads + tid;
        v[u] = li < c1 ? val(li) : -INFINITY;
      }
#pragma unroll
      for (int u = 0; u < kSweepU; ++u) {
        const int li = base + u * kShardThreads + tid;
        const uint32_t k = order_key(v[u]);
        const bool take = li < c1 && (strict ? k > T : k >= T);
        const unsigned b = __ballot_sync(0xffffffffu, take);
        if (b) {
          int at = 0;
          if (lane == 0) at = atomicAdd(&s_n, __popc(b));
          at = __shfl_sync(0xffffffffu, at, 0) + __popc(b & ((1u << lane) - 1u));
          if (take && at < kShardListCap) list[at] = cand_key(v[u], lo + li);
        }
      }
    }
    __syncthreads();
    return s_n;
  };
  auto count_ge = [&](uint32_t T) -> int {
    int c = 0;
    for (int base = c0; base < c1; base += kShardThreads * kSweepU) {
#pragma unroll
      for (int u = 0; u < kSweepU; ++u) {
        const int li = base + u * kShardThreads + tid;
        c += (li < c1 && order_key(val(li)) >= T) ? 1 : 0;
      }
    }
    return block_sum_int(c, red);
  };

  // ---- 3. threshold key T and the gathered keys: every content key when
  //      the shard has at most kc; else the keys >= a normal-fit guess, when
  //      there are between kc and kShardListCap of them; else bisection over
  //      the keys until such a T is found, or T is the largest key with at
  //      least kc keys >= it (exact: the keys above it, then its ties) ----
  uint32_t T = order_key(s_cmn);
  bool exact = false;
  int m;
  if (kc == ncont) {
    m = gather(T, false);
  } else {
    const double mean = s_csum / ncont, var = s_csq / ncont - mean * mean;
    const double sd = var > 0.0 ? sqrt(var) : 0.0;
    const double want = fmin((double)ncont, 1.25 * kc + 64.0);
    uint32_t lo_k = 0u, hi_k = order_key(s_cmx);  // count(>= lo_k) >= kc; count(> hi_k) < kc
    uint32_t cur = 0u;
    if (want < 0.9 * ncont) {
      cur = order_key((float)(mean + (double)normcdfinvf((float)(1.0 - want / ncont)) * sd));
      cur = cur > hi_k ? hi_k : cur;
    }
    int c = gather(cur, false);
    bool done = c >= kc && c <= kShardListCap;
    T = cur;
    for (int it = 0; it < 40 && !done; ++it) {
      if (c < kc) hi_k = cur - 1u;  // cur > lo_k here: count(>= lo_k) >= kc
      else lo_k = cur;
      if (lo_k >= hi_k) {
        T = lo_k;
        exact = true;
        break;
      }
      cur = lo_k + (uint32_t)(((uint64_t)hi_k - lo_k + 1u) >> 1);
      c = count_ge(cur);
      if (c >= kc && c <= kShardListCap) {
        T = cur;
        done = true;
        c = gather(T, false);
      }
    }
    if (!done && !exact) {
      T = lo_k;
      exact = true;
    }
    m = c;
    if (exact) {
      m = gather(T, true);  // fewer than kc keys above T
      // then keys equal to T in ascending block order (each thread owns a
      // contiguous range), up to kc in all: the reference's lowest-index ties
      const int R = ceil_div(ncont, kShardThreads);
      const int a0 = imin(c1, c0 + tid * R), a1 = imin(c1, a0 + R);
      int cnt = 0;
      for (int li = a0; li < a1; ++li) cnt += order_key(val(li)) == T ? 1 : 0;
      int off = block_exclusive_scan(cnt, red);
      const int need = kc - m;
      for (int li = a0; li < a1 && off < need; ++li) {
        const float v = val(li);
        if (order_key(v) == T) list[m + off++] = cand_key(v, lo + li);
      }
      m = kc;
      __syncthreads();
    }
  }

  // ---- 4. counting sort of the m keys, descending: buckets of the score key
  //      below the content max, each key's place = its bucket's start + the
  //      larger keys of its bucket; the first kc places are the output ----
  const uint32_t ktop = order_key(s_cmx);
  const uint32_t span = ktop - T;  // every gathered key lies in [T, ktop]
  int shift = 0;
  while ((span >> shift) >= (uint32_t)kShardSortBuckets) ++shift;  // ends by shift 21
  auto bucket_of_key = [&](unsigned long long k) -> int {
    return (int)((ktop - (uint32_t)(k >> 32)) >> shift);
  };
  for (int b = tid; b < kShardSortBuckets; b += kShardThreads) bfill[b] = 0;
  __syncthreads();
  for (int j = tid; j < m; j += kShardThreads) atomicAdd(&bfill[bucket_of_key(list[j])], 1);
  __syncthreads();
  {
    constexpr int BPT = kShardSortBuckets / kShardThreads;
    int c[BPT], tot = 0;
#pragma unroll
    for (int e = 0; e < BPT; ++e) {
      c[e] = bfill[tid * BPT + e];
      tot += c[e];
    }
    int off = block_exclusive_scan(tot, red);
#pragma unroll
    for (int e = 0; e < BPT; ++e) {
      bpos[tid * BPT + e] = off;
      bfill[tid * BPT + e] = 0;
      off += c[e];
    }
  }
  __syncthreads();
  for (int j = tid; j < m; j += kShardThreads) {
    const unsigned long long k = list[j];
    const int b = bucket_of_key(k);
    sorted[bpos[b] + atomicAdd(&bfill[b], 1)] = k;
  }
  __syncthreads();
  for (int j = tid; j < m; j += kShardThreads) {
    const unsigned long long k = sorted[j];
    const int b = bucket_of_key(k);
    const int b0 = bpos[b], b1 = b + 1 < kShardSortBuckets ? bpos[b + 1] : m;
    int place = b0;
    for (int i = b0; i < b1; ++i) place += sorted[i] > k ? 1 : 0;
    if (place < kc) out[place] = k;
  }
  pdl_launch_dependents();
}

// ---- stage 1: this shard's clamp term of the entropy ----------------------
// With zmax = max z over the whole row and Z = sum e^(z - zmax), the
// reference's H = -sum p log(max(p, 1e-9)) is log Z - A / Z - Cc / Z, Cc
// summing e (log(1e-9) - (z - zmax) + log Z) over blocks with p < 1e-9; the
// terms are evaluated as the plan kernel does (float exp, exact
// division-free test of fl(e / Z) < 1e-9f).
__global__ void __launch_bounds__(kShardThreads, 1) shard_clamp_kernel(ShardSelParams p) {
  __shared__ double red[32];
  __shared__ float s_mx;
  __shared__ double s_Z;
  const int h = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float Tf = (float)(p.cfg.temperature > 1e-6 ? p.cfg.temperature : 1e-6);
  const bool unit_t = (Tf == 1.0f);
  pdl_wait();  // every rank's records have been gathered
  if (tid == 0) {
    float mxg, M;
    double Z, A;
    merge_head(p, h, mxg, M, Z, A);
    s_mx = mxg;
    s_Z = Z;
  }
  __syncthreads();
  const double Z = s_Z;
  float cp = 0.f;
  if (p.nb >= 2 && p.cfg.policy == ADAKV_POLICY_ADAPTIVE && Z > 0.0) {
    const float zmax = zof(s_mx, Tf, unit_t);
    const double logZd = log(Z);
    const float Zf = (float)Z, logZ = (float)logZd;
    const float ln_floor = logf(1e-9f);
    const float pre = 2e-9f * Zf;  // p < 1e-9 implies e < 2e-9 Z
    const float d_hi = logf(pre), d_lo = d_hi - 25.f;
    const double clamp_mz = 0.5 * ((double)nextafterf(1e-9f, 0.f) + (double)1e-9f) * (double)Zf;
    const float* row = p.scores + (int64_t)h * p.score_stride;
    const int n = p.n_local;
    for (int base = 0; base < n; base += kShardThreads * kSweepU) {
      float v[kSweepU];
#pragma unroll
      for (int u = 0; u < kSweepU; ++u) {
        const int li = base + u * kShardThreads + tid;
        v[u] = li < n ? row[li] : INFINITY;
      }
#pragma unroll
      for (int u = 0; u < kSweepU; ++u) {
        const float d = __fsub_rn(zof(v[u], Tf, unit_t), zmax);
        if (d < d_hi && d >= d_lo) {
          const float e = expf(d);
          if (e > 0.f && e < pre && (double)e <= clamp_mz) cp = fmaf(e, ln_floor - d + logZ, cp);
        }
      }
    }
  }
  double c = warp_sum((double)cp);
  if (lane == 0) red[warp] = c;
  __syncthreads();
  if (warp == 0) {
    c = warp_sum(red[lane]);
    if (lane == 0) p.cc_mine[h] = c;
  }
  pdl_launch_dependents();
}

// ---- stage 2: budgets and this shard's part of the selection --------------
__global__ void __launch_bounds__(kShardFinishThreads, 1) shard_finish_kernel(ShardSelParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  double* s_w = reinterpret_cast<double*>(smem);  // [Hq]
  unsigned long long* lists =
      reinterpret_cast<unsigned long long*>(smem + ((size_t)p.Hq * sizeof(double) + 15) / 16 * 16);
  __shared__ int red[33];
  __shared__ int s_nc[kShardMaxWorld];
  __shared__ double s_sumw;
  const int h = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nb = p.nb;
  const bool adaptive = nb >= 2 && p.cfg.policy == ADAKV_POLICY_ADAPTIVE;
  const double lognb = log((double)imax(nb, 2));
  pdl_wait();

  // ---- 1. every head's weight (adakv/budget.py:36-37, float64 after the
  //      division), one thread per head; summed in a fixed order: every
  //      rank gets the same weights and sum ----
  if (adaptive) {
    for (int hh = tid; hh < p.Hq; hh += kShardFinishThreads) {
      float mxg, M;
      double Z, A, cc = 0.0;
      merge_head(p, hh, mxg, M, Z, A);
      if (p.cc_all) {
#pragma unroll 8
        for (int r = 0; r < p.world; ++r) cc += p.cc_all[(size_t)r * p.Hq + hh];
      }
      const double e = Z > 0.0 ? log(Z) - A / Z - cc / Z : 0.0;
      s_w[hh] = (double)(float)e / lognb + 1e-6;
    }
  }
  if (tid < p.world) s_nc[tid] = (int)stats_of(p, tid, h)[7];
  __syncthreads();
  if (warp == 0) {
    double s = 0.0;
    if (adaptive)
      for (int hh = lane; hh < p.Hq; hh += 32) s += s_w[hh];
    s = warp_sum(s);
    if (lane == 0) s_sumw = s;
  }
  __syncthreads();  // s_sumw

  const SeqBudget sb = seq_budget(nb, p.cfg);
  const double w = adaptive ? s_w[h] : 0.0;
  const int K = imin(head_count(sb, p.cfg, w, s_sumw, p.Hq), p.table_width);
  const int n_forced = (sb.sink + sb.local >= nb) ? nb : sb.sink + sb.local;
  const int Kc = imax(K - n_forced, 0);

  // The head's candidate lists, staged when they fit (loads in flight
  // together).  Only each list's first Kc keys matter: a candidate with Kc
  // larger keys in one list is out whatever the rest holds.
  const int kl = imin(Kc, p.cap_pad);
  const bool staged = (size_t)p.world * p.cap_pad * sizeof(unsigned long long) <=
                      (size_t)kShardFinishStage;
  if (staged && kl > 0) {
    const int tot = p.world * kl;
    for (int base = 0; base < tot; base += kShardFinishThreads * kSweepU) {
      unsigned long long v[kSweepU];
#pragma unroll
      for (int u = 0; u < kSweepU; ++u) {
        const int i = base + u * kShardFinishThreads + tid;
        const int r = i / kl, j = i - r * kl;
        v[u] = (i < tot && j < s_nc[r]) ? cands_of(p, r, h)[j] : 0ull;
      }
#pragma unroll
      for (int u = 0; u < kSweepU; ++u) {
        const int i = base + u * kShardFinishThreads + tid;
        const int r = i / kl, j = i - r * kl;
        if (i < tot) lists[(size_t)r * p.cap_pad + j] = v[u];
      }
    }
  }
  __syncthreads();
  auto list_of = [&](int r) -> const unsigned long long* {
    return staged ? lists + (size_t)r * p.cap_pad : cands_of(p, r, h);
  };

  // ---- 2. own candidates whose merged position is below Kc (a prefix; an
  //      own candidate at index j >= Kc is never in) ----
  const int me = p.rank, nme = imin(s_nc[me], Kc);
  int sel = 0;
  for (int j = tid; j < nme; j += kShardFinishThreads) {
    const unsigned long long key = list_of(me)[j];
    int rk = j;
    for (int r = 0; r < p.world && rk < Kc; ++r) {
      if (r == me) continue;
      const unsigned long long* L = list_of(r);
      int a = 0, b = imin(s_nc[r], Kc);  // entries of list r larger than key (up to Kc)
      while (a < b) {
        const int mid = (a + b) >> 1;
        if (L[mid] > key) a = mid + 1;
        else b = mid;
      }
      rk += a;
    }
    sel += rk < Kc ? 1 : 0;
  }
  const int t_me = block_sum_int(sel, red);
  int total = 0;
  for (int r = 0; r < p.world; ++r) total += s_nc[r];
  if (tid == 0 && total < Kc) report(p.status, ADAKV_ST_BAD_SEL_LEN);  // inconsistent records

  // ---- 3. this rank's table row: its forced blocks, then its picks ----
  const int lo = p.block_lo, hi = lo + p.n_local;
  const int e1 = imax(lo, imin(hi, sb.sink));           // [lo, e1): sink blocks held here
  const int s2 = imax(e1, imax(lo, nb - sb.local));     // [s2, hi): local-window blocks held here
  const int f1 = e1 - lo, f2 = imax(0, hi - s2);
  const int cnt = imin(f1 + f2 + t_me, p.out_width);
  int* trow = p.block_table + (int64_t)h * p.out_width;
  for (int i = tid; i < f1; i += kShardFinishThreads) trow[i] = lo + i;
  for (int i = tid; i < f2 && f1 + i < cnt; i += kShardFinishThreads) trow[f1 + i] = s2 + i;
  for (int j = tid; j < t_me && f1 + f2 + j < cnt; j += kShardFinishThreads)
    trow[f1 + f2 + j] = key_block(list_of(me)[j]);
  if (tid == 0) p.sel_lens[h] = cnt;
  pdl_launch_dependents();
}

size_t prep_smem(int n_local) {
  return 2 * kShardListCap * sizeof(unsigned long long) + 2 * kShardSortBuckets * sizeof(int) +
         (n_local <= kShardStageCap ? (size_t)n_local * sizeof(float) : 0);
}

}  // namespace

size_t shard_finish_smem(int Hq, int world, int cap_pad) {
  const size_t base = align_up((size_t)Hq * sizeof(double), 16);
  const size_t lists = (size_t)world * cap_pad * sizeof(unsigned long long);
  return base + (lists <= (size_t)kShardFinishStage ? lists : 0);
}

cudaError_t shard_kernels_init() {
  for (auto k : {shard_prep_kernel<true>, shard_prep_kernel<false>}) {
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)prep_smem(kShardStageCap));
    if (e != cudaSuccess) return e;
  }
  return cudaFuncSetAttribute(shard_finish_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)kShardFinishSmemMax);
}

cudaError_t launch_shard_select(int stage, const ShardSelParams& p, cudaStream_t st,
                                const LaunchOpts& o) {
  if (stage == 0) {
    const bool unit_t = (float)(p.cfg.temperature > 1e-6 ? p.cfg.temperature : 1e-6) == 1.0f;
    return launch_ex(unit_t ? shard_prep_kernel<true> : shard_prep_kernel<false>, dim3(p.Hq),
                     dim3(kShardThreads), prep_smem(p.n_local), st, o, p);
  }
  if (stage == 1)
    return launch_ex(shard_clamp_kernel, dim3(p.Hq), dim3(kShardThreads), 0, st, o, p);
  return launch_ex(shard_finish_kernel, dim3(p.Hq), dim3(kShardFinishThreads),
                   shard_finish_smem(p.Hq, p.world, p.cap_pad), st, o, p);
}

}  // namespace adakv
