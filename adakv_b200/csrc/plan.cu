// (c) Entropy-driven per-head budget and ragged per-head top-k block selection.
//
// One thread-block cluster of C CTAs (C = 1..8, chosen on the host) per
// (sequence, query head); CTA r of the cluster owns the blocks
// [r * L, (r + 1) * L) of the head's score row, L = ceil(nb / C) rounded up to
// 32 so every CTA owns whole bitmap words.  Row-wide quantities are merged
// through distributed shared memory: each CTA publishes its partials in a
// shared struct, `cluster.sync()`, and every CTA folds the C partials in rank
// order, so all CTAs (and all heads) compute bit-identical row values.
//
// 1. Load + statistics: the slice is staged in shared memory; max, content
//    max, content sum and sum of squares (sink/local blocks excluded).
// 2. Entropy, the formula of adakv/budget.py:28-37 with z = s / max(T, 1e-6),
//    e = exp(z - max z) in float32 per block, Z = sum e, p = e / Z:
//        H = -sum p log(max(p, 1e-9)) = log Z - A / Z - Cc / Z,
//    A = sum e (z - zmax) (one pass, no per-block division or logarithm) and
//    Cc = sum over blocks with p < 1e-9 of e (log(1e-9) - (z - zmax) + log Z),
//    the reference's clamp; sums are float per thread, double across threads.
//    Nucleus policy (budget.py:38-41) instead: the weight is 1 + the number of
//    blocks, in descending probability order, whose cumulative softmax mass
//    stays below nucleus_p, found by an MSB radix select over the score keys
//    whose histograms hold probability mass (float32 p, summed in double).
// 3. The Hq clusters of a sequence exchange entropies through per-head 64-bit
//    slots (call tag << 32 | float32 entropy; tags cleared by the estimator):
//    rank 0 publishes with one release store; warp 0 of every CTA polls the
//    sequence's slots (bounded by a 200 ms wall-clock limit, after which the
//    status word records a timeout) while the other warps merge the cluster's
//    top-k histograms.  Every CTA derives the Hq weights with the same
//    arithmetic (adakv/budget.py:36-37, float64 after the division), sums them
//    in a fixed order and computes its count (budget.py:71-86,
//    selector.py:49-54; half-to-even rounding).
// 4. Top-k over the content blocks (sink [0, sink) and local [nb-local, nb)
//    are always taken, the reference's +inf bias, selector.py:44-48): a
//    2048-bucket histogram over [cmax - range, cmax] (range = cmax - mean +
//    sd) finds the bucket holding the k-th score; that bucket's members across
//    the cluster are ranked exactly by (score desc, index asc).  A 4-pass MSB
//    radix select over order-preserving uint32 keys, merged across the
//    cluster, is the fallback; its ties at the threshold go to the lowest
//    indices.
// 5. Output: warp ballots build the slice's bitmap words; the table is written
//    in ascending block order at the cluster-wide exclusive prefix of the
//    per-CTA counts.
//
// All CTAs of one sequence must be resident together (they wait on each
// other's slots): the host sizes the grid from the cluster occupancy.
#include <algorithm>
#include <type_traits>

#include <cooperative_groups.h>

#include "kernels.h"

namespace cg = cooperative_groups;

namespace adakv {

// Slot words are single-copy atomic 64-bit values that carry their own tag
// and payload, so relaxed (uncached, gpu-scope) accesses suffice; relaxed
// loads of different slots are independent and overlap in flight.
__device__ __forceinline__ uint64_t ld_relaxed_u64(const unsigned long long* p) {
  uint64_t v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_relaxed_u64(unsigned long long* p, uint64_t v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// split cluster barrier: arrive after this CTA's writes, wait before reading
// the other CTAs' shared memory
__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// order-preserving float -> uint32 map; NaN sorts below everything
__device__ __forceinline__ uint32_t score_key(float f) {
  const uint32_t u = __float_as_uint(f);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return 0u;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

constexpr int kPW = kPlanThreads / 32;  // warps per CTA
constexpr int kPlanILP = 4;             // row elements per thread per tile (independent chains)
constexpr int kBuckets = 2048;          // bucket-select histogram bins
constexpr int kCandCap = 1024;          // members of the boundary bucket ranked exactly
constexpr int kFloorKeys = 8192;        // slice length from which the bucket floor and lists pay
constexpr int kListCap = 24;            // bucket-range blocks a thread lists
constexpr int kWinCap = 16;             // clamp-window blocks a thread defers
constexpr int kPassRun = 8;             // keys per thread and tile of the pass (2 runs of 4)

// floor(w) for 0 <= w < 2^23 (0 for w <= 0) without a float -> int conversion:
// adding 2^23 rounding toward zero leaves floor(w) in the low mantissa bits
__device__ __forceinline__ int bucket_floor(float w) {
  return __float_as_int(__fadd_rz(fmaxf(w, 0.f), 8388608.f)) - 0x4B000000;
}

// bucket of a content score: floor((cmx - s) * scale), clamped to the last
// bucket (which also takes NaN and -inf); non-decreasing as s decreases
__device__ __forceinline__ int bucket_of(float s, float cmx, float scale) {
  const float u = __fmul_rn(__fsub_rn(cmx, s), scale);
  if (!(u < (float)(kBuckets - 1))) return kBuckets - 1;
  return u <= 0.f ? 0 : (int)u;
}

// per-CTA partials read by the other CTAs of the cluster
struct PlanPart {
  float mx, cmx;       // slice max, slice content max
  double csum, csq;    // content sum / sum of squares
  float M;             // max z of the slice (softmax partials are relative to it)
  double Z, A;         // sum e^(z - M), sum e^(z - M) (z - M) over the slice
  int ncand;           // boundary-bucket candidates gathered by this CTA
  int nfix;            // blocks this CTA selected before the candidates
  int n_eq;            // radix path: keys equal to the threshold
  int n_sel;           // radix path: selected blocks of the slice
};

// Slot words carry this tag in their high half; the estimator clears every
// slot to 0 before the plan kernel starts, so a tagged word is this call's.
constexpr uint32_t kSlotTag = 0xADA0B200u;

// block-wide sum of two doubles; every thread gets the result
__device__ __forceinline__ void block_sum2(double& a, double& b, double* ra, double* rb) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  a = warp_sum(a);
  b = warp_sum(b);
  __syncthreads();  // ra / rb may still be read by a previous reduction
  if (lane == 0) {
    ra[warp] = a;
    rb[warp] = b;
  }
  __syncthreads();
  a = warp_sum(lane < kPW ? ra[lane] : 0.0);
  b = warp_sum(lane < kPW ? rb[lane] : 0.0);
}

// exclusive prefix over cluster ranks of an int field, read with one remote
// load per lane (lane r reads rank r); every lane gets its own prefix and the
// total in `tot`
__device__ __forceinline__ int rank_prefix(int v, int& tot) {
  const int lane = threadIdx.x & 31;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  tot = __shfl_sync(0xffffffffu, x, 31);
  return x - v;
}

// SMEM: the slice is staged in shared memory; LONG: the layout has room for
// the per-thread lists of the long-slice pass; NUC: the nucleus policy's
// mass-weighted select is compiled in.  Instantiations leave out the code they
// never run, which keeps the instruction footprint of the common ones small.
template <bool SMEM, bool LONG, bool NUC>
__global__ void __launch_bounds__(kPlanThreads, 1) plan_kernel(PlanParams p) {
  extern __shared__ __align__(16) uint32_t sm[];
  __shared__ __align__(16) uint32_t hist[kBuckets];   // this CTA's histogram (read by the cluster)
  __shared__ __align__(16) uint32_t ghist[kBuckets];  // the cluster's histogram
  __shared__ int cand_idx[kCandCap];      // this CTA's boundary candidates (read by the cluster)
  __shared__ uint32_t cand_key[kCandCap];
  __shared__ int all_idx[kCandCap];       // every candidate of the cluster, rank-major
  __shared__ uint32_t all_key[kCandCap];
  __shared__ PlanPart part;
  __shared__ int s_digit, s_above, s_ncand, s_nfix;
  __shared__ int s_off[kPlanMaxCluster + 1], s_fix[kPlanMaxCluster], s_taken[kPlanMaxCluster];
  __shared__ int scan_scratch[33];
  __shared__ float2 wpart[kPW];
  __shared__ float wm_s[kPW];
  __shared__ double wd[kPW][4];
  __shared__ int s_cl_over;                        // a thread's list overflowed
  __shared__ double dred[kPW], dred2[kPW];
  __shared__ double s_sumw, s_w;
  __shared__ double nmass[256];          // nucleus: probability mass per key digit
  __shared__ uint32_t ncnt[256];
  __shared__ int s_ndigit, s_ncnt_above, s_ncnt_digit;
  __shared__ double s_nmass_above;

  cg::cluster_group cl = cg::this_cluster();
  const int C = p.csize;
  const int rank = (int)cl.block_rank();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int slice_cap = p.slice_cap;
  const int nwl_alloc = (slice_cap / 32 + kPW - 1) / kPW * kPW;  // ballot words, whole passes
  uint32_t* keys = sm;                                                     // [slice_cap] (SMEM)
  uint32_t* wsel = sm + (SMEM ? slice_cap : 0);
  uint32_t* weq = wsel + nwl_alloc;
  // per-thread lists of slice indices, column `tid` (16-bit when the slice is
  // staged, so at most kPlanSmemMaxKeys long)
  using LIdx = typename std::conditional<SMEM, uint16_t, uint32_t>::type;
  LIdx* clist = reinterpret_cast<LIdx*>(weq + nwl_alloc);  // [kListCap][threads] bucket range
  LIdx* wlist = clist + kListCap * kPlanThreads;           // [kWinCap][threads] clamp window
  const PlanPart* lane_part = cl.map_shared_rank(&part, lane < C ? lane : 0);  // rank `lane`

  const int group = blockIdx.x / C;
  const int h = group % p.Hq;
  const int slot_seq = group / p.Hq;
  // sequence lengths are inputs of the whole step (the estimator never writes
  // them): read before waiting for it
  const int S_first = slot_seq < p.B ? seq_len_of(p.seq_lens, slot_seq, p.max_seq_len) : 0;
  // log(nb) of the entropy weight, off the exchange's critical path
  const double lognb_first =
      log((double)imax(ceil_div((S_first < 0 || S_first > p.max_seq_len) ? 0 : S_first, p.bs), 2));
  pdl_wait();

  for (int b0 = 0; b0 < p.B; b0 += p.seqs_per_round) {
    const int b = b0 + slot_seq;
    if (b >= p.B) break;  // uniform over the cluster
    const int row = b * p.Hq + h;
    int S = b0 == 0 ? S_first : seq_len_of(p.seq_lens, b, p.max_seq_len);
    if (S < 0 || S > p.max_seq_len) S = 0;  // reported by the estimator
    const int nb = ceil_div(S, p.bs);
    const double lognb = b0 == 0 ? lognb_first : log((double)imax(nb, 2));
    const int L = (ceil_div(nb, C) + 31) / 32 * 32;
    const int lo = imin(nb, rank * L), hi = imin(nb, lo + L);
    const int n = hi - lo;
    const int nwl = ceil_div(n, 32);
    const float* srow = p.scores + (int64_t)row * p.score_stride;

    auto val = [&](int li) -> float { return SMEM ? __uint_as_float(keys[li]) : srow[lo + li]; };
    // stage the slice in shared memory: 16-byte cp.async (every load of the
    // slice in flight at once) when it is 16-byte aligned, else plain loads;
    // the caller waits (cp_async_wait_all) before its next barrier
    auto stage_issue = [&]() {
      const float* src = srow + lo;
      if ((reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
        for (int i = 4 * tid; i < n; i += 4 * kPlanThreads)
          cp_async16_n(keys + i, src + i, (uint32_t)imin(4, n - i) * 4u);
        cp_async_commit();
      } else {
#pragma unroll 4
        for (int li = tid; li < n; li += kPlanThreads) keys[li] = __float_as_uint(src[li]);
      }
    };
    const int sink = imin(p.cfg.n_sink, nb), local = imin(p.cfg.n_local, nb);
    auto forced = [&](int i) -> bool { return i < sink || i >= nb - local; };

    const bool adaptive = nb >= 2 && p.cfg.policy == ADAKV_POLICY_ADAPTIVE;
    const bool nucleus = NUC && nb >= 2 && p.cfg.policy == ADAKV_POLICY_NUCLEUS;
    const bool soft = adaptive || nucleus;  // the row's softmax (Z) is needed
    const float Tf = (float)(p.cfg.temperature > 1e-6 ? p.cfg.temperature : 1e-6);
    const bool unit_t = (Tf == 1.0f);  // s / 1 == s exactly: skip the division
    auto zof = [&](float v) -> float { return unit_t ? v : __fdiv_rn(v, Tf); };
    float mx, cmx, m_t = -INFINITY;
    double csum, csq, Ztot = 0.0, Atot = 0.0;
    if (p.stats) {
      // ---- 1'. stage the slice while the row statistics are merged from the
      //      estimator's (chunk, warp) softmax partials, by every CTA alike ----
      if (SMEM) stage_issue();
      const int nparts = ceil_div(nb, kEstRows) * kEstConsumerWarps;
      const float* prow = p.stats + (int64_t)row * p.stats_stride * kStatF;
      SoftPart acc = soft_empty();
      constexpr int PU = 4;  // partial loads in flight per thread
      // partials c in [0, nparts], the last being the append's slot; a
      // long-slice CTA merges only its rank's share of them and the cluster
      // folds the C results below (a short slice's CTA merges them all)
      int c_lo = 0, c_hi = nparts + 1;
      if (LONG) {
        const int share = ceil_div(nparts + 1, C);
        c_lo = imin(nparts + 1, rank * share);
        c_hi = imin(nparts + 1, c_lo + share);
      }
      for (int c0 = c_lo + tid; c0 < c_hi; c0 += kPlanThreads * PU) {
        SoftPart t[PU];
#pragma unroll
        for (int u = 0; u < PU; ++u) {
          const int c = c0 + u * kPlanThreads;
          t[u] = c < c_hi ? soft_load(prow + (int64_t)(c < nparts ? c : p.stats_stride - 1) * kStatF)
                          : soft_empty();
        }
#pragma unroll
        for (int u = 0; u < PU; ++u) soft_merge(acc, t[u]);
      }
      for (int t = tid; t < kBuckets; t += kPlanThreads) hist[t] = 0u;
      if (tid < kPlanMaxCluster) s_taken[tid] = 0;
      if (tid == 0) {
        s_ncand = 0;
        s_nfix = 0;
        s_cl_over = 0;
      }
      // warp partials rescaled to the warp max; one barrier; every warp then
      // folds the kPW warp partials in the same order (identical results)
      {
        const float wm = warp_max(acc.m), wmx = warp_max(acc.mx), wcmx = warp_max(acc.cmx);
        double z = 0.0, a = 0.0;
        if (acc.m > -INFINITY) {
          const double f = (double)expf(acc.m - wm);
          z = (double)acc.Z * f;
          a = f * ((double)acc.A + (double)acc.Z * ((double)acc.m - (double)wm));
        }
        z = warp_sum(z);
        a = warp_sum(a);
        const double cs = warp_sum((double)acc.cs), cq = warp_sum((double)acc.cq);
        if (lane == 0) {
          wpart[warp] = make_float2(wmx, wcmx);
          wm_s[warp] = wm;
          wd[warp][0] = z;
          wd[warp][1] = a;
          wd[warp][2] = cs;
          wd[warp][3] = cq;
        }
      }
      if (SMEM) cp_async_wait_all();
      __syncthreads();  // also publishes the staged slice
      {
        const bool in = lane < kPW;
        const float wm = in ? wm_s[lane] : -INFINITY;
        const float M = warp_max(wm);
        mx = warp_max(in ? wpart[lane].x : -INFINITY);
        cmx = warp_max(in ? wpart[lane].y : -INFINITY);
        double z = 0.0, a = 0.0;
        if (in && wm > -INFINITY) {
          const double f = (double)expf(wm - M);
          z = wd[lane][0] * f;
          a = f * (wd[lane][1] + wd[lane][0] * ((double)wm - (double)M));
        }
        Ztot = warp_sum(z);
        Atot = warp_sum(a);
        csum = warp_sum(in ? wd[lane][2] : 0.0);
        csq = warp_sum(in ? wd[lane][3] : 0.0);
        if (LONG && tid == 0) {
          part.mx = mx;
          part.cmx = cmx;
          part.csum = csum;
          part.csq = csq;
          part.M = M;
          part.Z = Ztot;
          part.A = Atot;
        }
      }
      if (LONG) {
        cl.sync();  // (1') every CTA's share of the partials is merged
        const bool in = lane < C;
        mx = warp_max(in ? lane_part->mx : -INFINITY);
        cmx = warp_max(in ? lane_part->cmx : -INFINITY);
        csum = warp_sum(in ? lane_part->csum : 0.0);
        csq = warp_sum(in ? lane_part->csq : 0.0);
        const float Mr = in ? lane_part->M : -INFINITY;
        const float M = warp_max(Mr);
        double z = 0.0, a = 0.0;
        if (in && Mr > -INFINITY) {
          const double zr = lane_part->Z, ar = lane_part->A;
          const double sc = exp((double)Mr - (double)M);
          z = zr * sc;
          a = sc * (ar + zr * ((double)Mr - (double)M));
        }
        Ztot = warp_sum(z);
        Atot = warp_sum(a);
      }
    } else {
      // ---- 1. load the slice: statistics and per-thread softmax partials ----
      // Each thread keeps (m_t, z_t, a_t) = (max z, sum e^(z - m_t),
      // sum e^(z - m_t) (z - m_t)) over its blocks, rescaled when m_t grows.
      mx = -INFINITY;
      cmx = -INFINITY;
      float csum_f = 0.f, csq_f = 0.f;
      float z_t = 0.f, a_t = 0.f;
      if (SMEM) {
        stage_issue();
        cp_async_wait_all();
        __syncthreads();
      }
      for (int base = 0; base < n; base += kPlanThreads * kPlanILP) {
        float v[kPlanILP];
#pragma unroll
        for (int r = 0; r < kPlanILP; ++r) {
          const int li = base + r * kPlanThreads + tid;
          v[r] = li < n ? val(li) : -INFINITY;
        }
        float tm = -INFINITY;
#pragma unroll
        for (int r = 0; r < kPlanILP; ++r) {
          const int li = base + r * kPlanThreads + tid;
          if (li < n) {
            mx = fmaxf(mx, v[r]);
            tm = fmaxf(tm, zof(v[r]));
            if (!forced(lo + li)) {
              cmx = fmaxf(cmx, v[r]);
              csum_f += v[r];
              csq_f = fmaf(v[r], v[r], csq_f);
            }
          }
        }
        if (soft && tm > m_t) {
          if (m_t > -INFINITY) {
            const float sc = expf(m_t - tm);
            a_t = sc * fmaf(z_t, m_t - tm, a_t);
            z_t *= sc;
          }
          m_t = tm;
        }
        if (soft) {
#pragma unroll
          for (int r = 0; r < kPlanILP; ++r) {
            const int li = base + r * kPlanThreads + tid;
            if (li < n) {
              const float d = zof(v[r]) - m_t;
              const float e = expf(d);
              z_t += e;
              if (e > 0.f) a_t = fmaf(e, d, a_t);
            }
          }
        }
      }
      for (int t = tid; t < kBuckets; t += kPlanThreads) hist[t] = 0u;
      if (tid < kPlanMaxCluster) s_taken[tid] = 0;
      if (tid == 0) {
        s_ncand = 0;
        s_nfix = 0;
        s_cl_over = 0;
      }
      // warp partials (softmax partials rescaled to the warp max), then one
      // fold of the warps by warp 0, then the cluster
      {
        const float wm = warp_max(m_t);
        double zw = 0.0, aw = 0.0;
        if (soft && m_t > -INFINITY) {
          const double sc = exp((double)m_t - (double)wm);
          zw = (double)z_t * sc;
          aw = sc * ((double)a_t + (double)z_t * ((double)m_t - (double)wm));
        }
        zw = warp_sum(zw);
        aw = warp_sum(aw);
        const float wmx = warp_max(mx), wcmx = warp_max(cmx);
        const double wsum = warp_sum((double)csum_f), wsq = warp_sum((double)csq_f);
        if (lane == 0) {
          wpart[warp] = make_float2(wmx, wcmx);
          wm_s[warp] = wm;
          wd[warp][0] = zw;
          wd[warp][1] = aw;
          wd[warp][2] = wsum;
          wd[warp][3] = wsq;
        }
      }
      __syncthreads();  // also publishes the staged slice
      if (warp == 0) {
        const bool in = lane < kPW;
        const float M = warp_max(in ? wm_s[lane] : -INFINITY);
        double z = 0.0, a = 0.0;
        if (in && wm_s[lane] > -INFINITY) {
          const double sc = exp((double)wm_s[lane] - (double)M);
          z = wd[lane][0] * sc;
          a = sc * (wd[lane][1] + wd[lane][0] * ((double)wm_s[lane] - (double)M));
        }
        z = warp_sum(z);
        a = warp_sum(a);
        const float m1 = warp_max(in ? wpart[lane].x : -INFINITY);
        const float m2 = warp_max(in ? wpart[lane].y : -INFINITY);
        const double cs = warp_sum(in ? wd[lane][2] : 0.0);
        const double cq = warp_sum(in ? wd[lane][3] : 0.0);
        if (lane == 0) {
          part.mx = m1;
          part.cmx = m2;
          part.csum = cs;
          part.csq = cq;
          part.M = M;
          part.Z = z;
          part.A = a;
        }
      }
      cl.sync();  // (1) slice statistics and softmax partials of every CTA
      {
        const bool in = lane < C;
        mx = warp_max(in ? lane_part->mx : -INFINITY);
        cmx = warp_max(in ? lane_part->cmx : -INFINITY);
        csum = warp_sum(in ? lane_part->csum : 0.0);
        csq = warp_sum(in ? lane_part->csq : 0.0);
        if (soft) {
          const float Mr = in ? lane_part->M : -INFINITY;
          const float M = warp_max(Mr);
          double z = 0.0, a = 0.0;
          if (in && Mr > -INFINITY) {
            const double zr = lane_part->Z, ar = lane_part->A;
            const double sc = exp((double)Mr - (double)M);
            z = zr * sc;
            a = sc * (ar + zr * ((double)Mr - (double)M));
          }
          Ztot = warp_sum(z);
          Atot = warp_sum(a);
        }
      }
    }

    // ---- top-k bucket geometry (independent of the budget) ----
    const double nc_d = (double)(nb - imin(nb, sink + local));
    const double mean_c = nc_d > 0 ? csum / nc_d : 0.0;
    const double var_c = nc_d > 0 ? csq / nc_d - mean_c * mean_c : 0.0;
    const double sd_c = var_c > 0.0 ? sqrt(var_c) : 0.0;
    // Bucket floor: the content score with about 4 x table_width content
    // blocks above it under a normal fit of the row, never below mean - sd.
    // Only blocks above it are histogrammed and listed as selection
    // candidates; a histogram holding fewer blocks than the row picks sends
    // the row to the radix select, so the floor affects speed only.
    // (long slices only: a short slice's passes are cheaper than the fit)
    const bool long_slice = LONG && L >= kFloorKeys;  // L is the same in every CTA of the row
    double floor_c = mean_c - sd_c;
    if (long_slice) {
      const double want = 4.0 * (double)p.table_width;
      if (nc_d > 0.0 && want < 0.8 * nc_d)
        floor_c = fmax(floor_c, mean_c + (double)normcdfinvf((float)(1.0 - want / nc_d)) * sd_c);
    }
    const double range = (double)cmx - floor_c;
    const bool buckets_ok = isfinite(cmx) && range > 0.0 && isfinite(range);
    const float scale = buckets_ok ? (float)((double)(kBuckets - 1) / range) : 0.f;

    // ---- 2. clamp correction of this slice, and the histogram and list of
    //      its content blocks above the bucket floor ----
    // With zmax = max z (= max(s) / T, monotone rounding), d = z - zmax and
    // e = exp(d) as the reference computes them, H = log Z - A / Z - Cc / Z
    // where Cc sums e (log(1e-9) - d + log Z) over blocks with e / Z < 1e-9.
    // On long slices both kinds of rare block are set aside per thread
    // (column `tid` of a shared table, so a warp's stores are conflict-free)
    // and finished after the pass: the per-key work is a few compares and
    // predicated stores.
    const float zmax = unit_t ? mx : __fdiv_rn(mx, Tf);
    // log Z once, for the clamp terms (float) and the entropy (double)
    const double logZd = adaptive ? log(Ztot) : 0.0;
    float cp = 0.f;
    int ncl = 0;  // blocks this thread listed
    {
      const float Zf = (float)Ztot;
      const float logZ = (float)logZd;
      const float ln_floor = logf(1e-9f);
      const float pre = 2e-9f * Zf;  // p < 1e-9 implies e < 2e-9 * Z
      // p < 1e-9 needs d < log(2e-9 Z); below d_lo the clamp's correction
      // e (log 1e-9 - log p) is under 1e-18 of H: skip the exp there
      const float d_hi = adaptive ? logf(pre) : -INFINITY;
      const float d_lo = d_hi - 25.f;
      // p = e / Z rounded to float is below 1e-9f exactly when e <= mid * Z,
      // mid = the midpoint between 1e-9f and the float below it (a tie rounds
      // down: 1e-9f has an odd significand); mid * Z is exact in double
      // (25 + 24 significant bits), so no division is needed
      const double clamp_mz = 0.5 * ((double)nextafterf(1e-9f, 0.f) + (double)1e-9f) * (double)Zf;
      auto corr = [&](float d) {
        const float e = expf(d);
        if (e > 0.f && e < pre && (double)e <= clamp_mz) cp = fmaf(e, ln_floor - d + logZ, cp);
      };
      if (!long_slice) {
        // short slice: one inline pass (the deferred lists do not pay here)
        for (int base = 0; base < n; base += kPlanThreads * kPlanILP) {
#pragma unroll
          for (int r = 0; r < kPlanILP; ++r) {
            const int li = base + r * kPlanThreads + tid;
            if (li < n) {
              const float v = val(li);
              if (adaptive) {
                const float d = __fsub_rn(zof(v), zmax);
                if (d < d_hi && d >= d_lo) corr(d);
              }
              if (buckets_ok && !forced(lo + li)) {
                const int bk = bucket_of(v, cmx, scale);
                if (bk < kBuckets - 1) atomicAdd(&hist[bk], 1u);
              }
            }
          }
        }
      } else {
        int nwin = 0;
        auto flush = [&]() {
          for (int i = 0; i < nwin; ++i) corr(__fsub_rn(zof(val((int)wlist[i * kPlanThreads + tid])), zmax));
          nwin = 0;
        };
        // 2 runs of 4 consecutive keys per thread and tile (vector shared loads
        // when the slice is staged); a window list that might not take another
        // tile is finished first, so it never overflows
        for (int base = 0; base < n; base += kPassRun * kPlanThreads) {
          float vv[kPassRun];
#pragma unroll
          for (int u = 0; u < kPassRun / 4; ++u) {
            const int li0 = base + u * 4 * kPlanThreads + 4 * tid;
            if (SMEM) {
              if (li0 < n) {
                const uint4 w4 = *reinterpret_cast<const uint4*>(keys + li0);
                vv[4 * u + 0] = __uint_as_float(w4.x);
                vv[4 * u + 1] = __uint_as_float(w4.y);
                vv[4 * u + 2] = __uint_as_float(w4.z);
                vv[4 * u + 3] = __uint_as_float(w4.w);
              }
            } else {
#pragma unroll
              for (int e = 0; e < 4; ++e) vv[4 * u + e] = li0 + e < n ? srow[lo + li0 + e] : 0.f;
            }
          }
#pragma unroll
          for (int u = 0; u < kPassRun / 4; ++u) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int li = base + u * 4 * kPlanThreads + 4 * tid + e;
              const bool valid = li < n;
              const float v = vv[4 * u + e];
              if (adaptive) {
                const float d = __fsub_rn(zof(v), zmax);
                const bool win = valid && d < d_hi && d >= d_lo;
                if (win) wlist[nwin * kPlanThreads + tid] = (LIdx)li;
                nwin += win;
              }
              // in the bucket range: bucket_of(v) < kBuckets - 1; a full list
              // keeps counting (the selection then scans the slice)
              const float w = __fmul_rn(__fsub_rn(cmx, v), scale);
              const bool in = buckets_ok && valid && w < (float)(kBuckets - 1) && !forced(lo + li);
              if (in) {
                atomicAdd(&hist[bucket_floor(w)], 1u);
                clist[imin(ncl, kListCap - 1) * kPlanThreads + tid] = (LIdx)li;
              }
              ncl += in;
            }
          }
          if (nwin > kWinCap - kPassRun) flush();
        }
        flush();
        if (ncl > kListCap) s_cl_over = 1;
      }
    }
    // ---- nucleus weight (adakv/budget.py:38-41): the blocks, in descending
    //      probability order, whose cumulative softmax mass stays below
    //      nucleus_p.  MSB radix select over the score keys with histograms of
    //      probability mass (p = e / Z in float32, summed in double) merged over
    //      the cluster; ties at the threshold key share one probability. ----
    int ncount = 0;
    if (nucleus) {
      const float Zf = (float)Ztot;
      const double P = p.cfg.nucleus_p;
      uint32_t prefix = 0, pmask = 0;
      double above = 0.0;  // mass of the blocks ranked above the current prefix
      int n_above = 0;
      bool all = false;
#pragma unroll 1
      for (int pass = 0; pass < 4; ++pass) {
        const int shift = 24 - 8 * pass;
        for (int t = tid; t < 256; t += kPlanThreads) {
          nmass[t] = 0.0;
          ncnt[t] = 0u;
        }
        __syncthreads();
        for (int li = tid; li < n; li += kPlanThreads) {
          const float v = val(li);
          const uint32_t k = score_key(v);
          if ((k & pmask) == prefix) {
            const float pr = __fdiv_rn(expf(__fsub_rn(zof(v), zmax)), Zf);
            const int dg = (k >> shift) & 0xFF;
            atomicAdd(&nmass[dg], (double)pr);
            atomicAdd(&ncnt[dg], 1u);
          }
        }
        cl.sync();  // every CTA's histograms complete
        if (warp == 0) {
          double m8[8], tot = 0.0;
          int c8[8], ctot = 0;
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            m8[e] = 0.0;
            c8[e] = 0;
          }
#pragma unroll
          for (int r = 0; r < kPlanMaxCluster; ++r) {
            if (r < C) {
              const double* mr = cl.map_shared_rank(nmass, r);
              const uint32_t* cr = cl.map_shared_rank(ncnt, r);
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                m8[e] += mr[255 - 8 * lane - e];
                c8[e] += (int)cr[255 - 8 * lane - e];
              }
            }
          }
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            tot += m8[e];
            ctot += c8[e];
          }
          double incl = tot;
          int cincl = ctot;
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            const double y = __shfl_up_sync(0xffffffffu, incl, o);
            const int cy = __shfl_up_sync(0xffffffffu, cincl, o);
            if (lane >= o) {
              incl += y;
              cincl += cy;
            }
          }
          // below the first pass the prefix's mass bounds the target (rounding)
          const double all_mass = __shfl_sync(0xffffffffu, incl, 31);
          const double Pu = pass > 0 ? fmin(P, above + all_mass) : P;
          const double excl = incl - tot;
          const int cexcl = cincl - ctot;
          if (lane == 0) s_ndigit = -1;
          __syncwarp();
          if (above + excl < Pu && Pu <= above + incl) {
            double acc = excl;
            int cacc = cexcl;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              if (above + acc + m8[e] >= Pu) {
                s_ndigit = 255 - 8 * lane - e;
                s_nmass_above = acc;
                s_ncnt_above = cacc;
                s_ncnt_digit = c8[e];
                break;
              }
              acc += m8[e];
              cacc += c8[e];
            }
          }
        }
        cl.sync();  // digit read by every CTA before the histograms are cleared again
        if (s_ndigit < 0) {  // all the mass is below nucleus_p (same in every CTA)
          all = true;
          break;
        }
        above += s_nmass_above;
        n_above += s_ncnt_above;
        prefix |= (uint32_t)s_ndigit << shift;
        pmask |= 0xFFu << shift;
      }
      if (all) {
        ncount = nb;
      } else {
        // the s_ncnt_digit blocks whose key equals the threshold share one probability
        const uint32_t T = prefix;
        const float sT = __uint_as_float((T & 0x80000000u) ? (T & 0x7FFFFFFFu) : ~T);
        const double pT = (double)__fdiv_rn(expf(__fsub_rn(zof(sT), zmax)), Zf);
        const int E = s_ncnt_digit;
        long long ties = pT > 0.0 ? (long long)ceil((P - above) / pT) - 1 : (long long)E;
        ties = ties < 0 ? 0 : (ties > E ? E : ties);
        ncount = n_above + (int)ties;
      }
    }
    double t_mine = 0.0;
    if (nucleus) t_mine = rank == 0 ? (double)(ncount + 1) : 0.0;  // weight = count + 1
    if (adaptive) {
      double c2 = cp, z2 = 0.0;
      block_sum2(c2, z2, dred, dred2);
      // this CTA's share of H: CTA 0 carries log Z - A / Z, every CTA -Cc_r / Z
      t_mine = (rank == 0 ? logZd - Atot / Ztot : 0.0) - c2 / Ztot;
    }
    __syncthreads();
    cluster_arrive_release();  // (2) this CTA's histogram is complete
    unsigned long long* slots = &p.slots[0].word;
    if (tid == 0 && !((p.debug_flags & 1) && row == 0)) {
      const float thi = (float)t_mine;
      const float tlo = (float)(t_mine - (double)thi);
      const size_t at = ((size_t)row * C + rank) * 2;
      st_relaxed_u64(slots + at, ((uint64_t)kSlotTag << 32) | (uint64_t)__float_as_uint(thi));
      st_relaxed_u64(slots + at + 1, ((uint64_t)kSlotTag << 32) | (uint64_t)__float_as_uint(tlo));
    }
    auto weight_of = [&](double e) -> double {
      // entropy: adakv/budget.py:36-37, float64 after the division; nucleus:
      // the published count + 1 (budget.py:41)
      return nucleus ? e : (double)(float)e / lognb + 1e-6;
    };

    // ---- exchange across the sequence's heads (warp 0) / merge histograms ----
    if (warp == 0) {
      const uint64_t t0 = globaltimer_ns();
      bool ok = false;
      double ents[4];  // Hq <= 128
      while (true) {
        bool mine = true;
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          const int hh = lane + q4 * 32;
          double e = 0.0;
          if (hh < p.Hq) {
            const unsigned long long* hs = slots + (size_t)(b * p.Hq + hh) * C * 2;
#pragma unroll
            for (int r = 0; r < kPlanMaxCluster; ++r) {
              if (r < C) {
                const uint64_t v0 = ld_relaxed_u64(hs + 2 * r);
                const uint64_t v1 = ld_relaxed_u64(hs + 2 * r + 1);
                mine &= ((uint32_t)(v0 >> 32) == kSlotTag) && ((uint32_t)(v1 >> 32) == kSlotTag);
                e += (double)__uint_as_float((uint32_t)v0) + (double)__uint_as_float((uint32_t)v1);
              }
            }
          }
          ents[q4] = e;
        }
        ok = __all_sync(0xffffffffu, mine);
        // lanes may read the timer at different moments: lane 0 decides for
        // the warp, so no lane leaves the loop (and its warp-wide __all_sync)
        // while another stays in it
        const bool expired = __shfl_sync(0xffffffffu, globaltimer_ns() - t0 > p.wait_ns, 0);
        if (ok || expired) break;
      }
      if (!ok && lane == 0) report(p.status, ADAKV_ST_WAIT_TIMEOUT);
      double ps = 0.0;
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        const int hh = lane + q4 * 32;
        if (hh < p.Hq && soft) {
          const double wv = weight_of(ents[q4]);
          ps += wv;
          if (hh == h) s_w = wv;
        }
      }
      ps = warp_sum(ps);  // fixed xor tree: every CTA of the sequence gets the same sum
      if (lane == 0) s_sumw = ps;
      cluster_wait_acquire();
    } else {
      cluster_wait_acquire();  // every histogram of the cluster is complete
      for (int j = tid - 32; buckets_ok && j < kBuckets / 4; j += kPlanThreads - 32) {
        uint4 acc = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
        for (int r = 0; r < kPlanMaxCluster; ++r) {
          if (r < C) {
            const uint4 x = reinterpret_cast<const uint4*>(cl.map_shared_rank(hist, r))[j];
            acc.x += x.x;
            acc.y += x.y;
            acc.z += x.z;
            acc.w += x.w;
          }
        }
        reinterpret_cast<uint4*>(ghist)[j] = acc;
      }
    }
    __syncthreads();
    pdl_launch_dependents();  // every CTA is past the exchange: the attend grid may launch
    const SeqBudget sbud = seq_budget(nb, p.cfg);
    const double w = soft ? s_w : 0.0;
    const int K = imin(head_count(sbud, p.cfg, w, s_sumw, p.Hq), p.table_width);
    const int n_forced = (sink + local >= nb) ? nb : sink + local;
    const int Kc = K - n_forced;  // content blocks to pick
    const bool all = K >= nb;

    // ---- 4. top-k ----
    bool use_radix = false;
    int jstar = kBuckets, need_b = 0;
    if (!all && Kc > 0) {
      use_radix = !buckets_ok;
      if (!use_radix) {
        // the bucket holding the Kc-th content block (buckets ascend = scores descend)
        constexpr int BPT = kBuckets / kPlanThreads;
        uint32_t cb[BPT], tot = 0;
#pragma unroll
        for (int e = 0; e < BPT; ++e) {
          cb[e] = ghist[tid * BPT + e];
          tot += cb[e];
        }
        const int before = block_exclusive_scan((int)tot, scan_scratch);
        if (tid == 0) s_digit = kBuckets - 1;
        __syncthreads();
        if (before < Kc && Kc <= before + (int)tot) {
          int acc = before;
#pragma unroll
          for (int e = 0; e < BPT; ++e) {
            if (acc + (int)cb[e] >= Kc) {
              s_digit = tid * BPT + e;
              s_above = acc;
              break;
            }
            acc += (int)cb[e];
          }
        }
        __syncthreads();
        jstar = s_digit;
        if (jstar >= kBuckets - 1 || (int)ghist[jstar] > kCandCap) use_radix = true;
        else need_b = Kc - s_above;
      }
    }
    const bool bucketed = !all && Kc > 0 && !use_radix;
    if (bucketed && long_slice && !s_cl_over) {
      // every warp's list is complete: the forced blocks, then the listed
      // blocks of buckets above jstar; the members of bucket jstar are
      // candidates, ranked across the cluster
      for (int wi = tid; wi < nwl; wi += kPlanThreads) wsel[wi] = 0u;
      __syncthreads();
      int cnt = 0;
      const int f1 = imin(sink, hi), f2 = imax(nb - local, lo);
      for (int i = lo + tid; i < f1; i += kPlanThreads, ++cnt)
        atomicOr(&wsel[(i - lo) >> 5], 1u << ((i - lo) & 31));
      for (int i = f2 + tid; i < hi; i += kPlanThreads, ++cnt)
        atomicOr(&wsel[(i - lo) >> 5], 1u << ((i - lo) & 31));
      for (int i = 0; i < ncl; ++i) {
        const int li = (int)clist[i * kPlanThreads + tid];
        const float v = val(li);
        const int bk = bucket_floor(__fmul_rn(__fsub_rn(cmx, v), scale));
        if (bk < jstar) {
          atomicOr(&wsel[li >> 5], 1u << (li & 31));
          ++cnt;
        } else if (bk == jstar) {
          const int slot = atomicAdd(&s_ncand, 1);
          cand_idx[slot] = lo + li;
          cand_key[slot] = score_key(v);
        }
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
      if (lane == 0 && cnt) atomicAdd(&s_nfix, cnt);
      __syncthreads();
      if (tid == 0) {
        part.ncand = s_ncand;
        part.nfix = s_nfix;
      }
    } else if (!use_radix) {
      // selected: forced blocks, every content block of a bucket above jstar;
      // the members of bucket jstar are candidates, ranked across the cluster
      int nfix = 0;  // lane 0: blocks this warp selected
      for (int j0 = 0; j0 * kPlanThreads < n; j0 += 4) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int j = j0 + u;
          if (j * kPlanThreads >= n) break;  // uniform over the CTA
          const int li = j * kPlanThreads + tid;
          bool sel = false;
          if (li < n) {
            if (all || forced(lo + li)) {
              sel = true;
            } else if (bucketed) {
              const float v = val(li);
              const int bk = bucket_of(v, cmx, scale);
              sel = bk < jstar;
              if (bk == jstar) {
                const int slot = atomicAdd(&s_ncand, 1);
                cand_idx[slot] = lo + li;
                cand_key[slot] = score_key(v);
              }
            }
          }
          const uint32_t bsel = __ballot_sync(0xffffffffu, sel);
          if (lane == 0) {
            wsel[j * kPW + warp] = bsel;
            weq[j * kPW + warp] = 0u;
            nfix += __popc(bsel);
          }
        }
      }
      if (lane == 0 && nfix) atomicAdd(&s_nfix, nfix);
      __syncthreads();
      if (tid == 0) {
        part.ncand = s_ncand;
        part.nfix = s_nfix;
      }
    }
    cl.sync();  // (3) candidates and counts of every CTA

    int pos = 0;  // this CTA's first table position
    if (!use_radix) {
      if (warp == 0) {
        const bool in = lane < C;
        int tot;
        const int nc = in ? lane_part->ncand : 0;
        const int off = rank_prefix(nc, tot);
        if (in) {
          s_off[lane] = off;
          s_fix[lane] = lane_part->nfix;
        }
        if (lane == 0) s_off[C] = tot;
      }
      __syncthreads();
      const int ntot = bucketed ? s_off[C] : 0;
      // copy every CTA's candidates (one remote load per entry)
      for (int u = tid; u < ntot; u += kPlanThreads) {
        int r = 0;
        while (r + 1 < C && s_off[r + 1] <= u) ++r;
        const int t = u - s_off[r];
        all_key[u] = cl.map_shared_rank(cand_key, r)[t];
        all_idx[u] = cl.map_shared_rank(cand_idx, r)[t];
      }
      __syncthreads();
      for (int u = tid; u < ntot; u += kPlanThreads) {
        const uint32_t ku = all_key[u];
        const int iu = all_idx[u];
        int rk = 0;
        for (int c = 0; c < ntot; ++c) {
          const uint32_t kc = all_key[c];
          rk += (kc > ku) || (kc == ku && all_idx[c] < iu);
        }
        if (rk < need_b) {
          int r = 0;
          while (r + 1 < C && s_off[r + 1] <= u) ++r;
          atomicAdd(&s_taken[r], 1);
          if (r == rank) atomicOr(&wsel[(iu - lo) >> 5], 1u << ((iu - lo) & 31));
        }
      }
      __syncthreads();
      for (int r = 0; r < rank; ++r) pos += s_fix[r] + s_taken[r];
    } else {
      // ---- radix select over the cluster (fallback) ----
      if (SMEM) {
        for (int li = tid; li < n; li += kPlanThreads)
          keys[li] = forced(lo + li) ? 0xFFFFFFFFu : score_key(__uint_as_float(keys[li]));
        __syncthreads();
      }
      auto key = [&](int li) -> uint32_t {
        return SMEM ? keys[li] : (forced(lo + li) ? 0xFFFFFFFFu : score_key(srow[lo + li]));
      };
      uint32_t prefix = 0, pmask = 0;
      int rem = K;
#pragma unroll 1
      for (int pass = 0; pass < 4; ++pass) {
        const int shift = 24 - 8 * pass;
        if (tid < 256) hist[tid] = 0;
        __syncthreads();
        for (int li = tid; li < n; li += kPlanThreads) {
          const uint32_t k = key(li);
          if ((k & pmask) == prefix) atomicAdd(&hist[(k >> shift) & 0xFFu], 1u);
        }
        cl.sync();  // every CTA's digit histogram complete
        if (warp == 0) {
          uint32_t c[8], tot = 0;
#pragma unroll
          for (int e = 0; e < 8; ++e) c[e] = 0;
#pragma unroll
          for (int r = 0; r < kPlanMaxCluster; ++r) {
            if (r < C) {
              const uint32_t* hr = cl.map_shared_rank(hist, r);
#pragma unroll
              for (int e = 0; e < 8; ++e) c[e] += hr[255 - 8 * lane - e];
            }
          }
#pragma unroll
          for (int e = 0; e < 8; ++e) tot += c[e];
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
        cl.sync();  // digit read by every CTA before any histogram is cleared again
        rem -= s_above;
        prefix |= (uint32_t)s_digit << shift;
        pmask |= 0xFFu << shift;
      }
      const uint32_t T = prefix;
      const int need = rem;  // ties at T resolved in index order
      for (int j = 0; j * kPlanThreads < n; ++j) {
        const int li = j * kPlanThreads + tid;
        const bool valid = li < n;
        const uint32_t k = valid ? key(li) : 0u;
        const uint32_t bgt = __ballot_sync(0xffffffffu, valid && k > T);
        const uint32_t beq = __ballot_sync(0xffffffffu, valid && k == T);
        if (lane == 0) {
          wsel[j * kPW + warp] = bgt;
          weq[j * kPW + warp] = beq;
        }
      }
      __syncthreads();
      const int wpt = ceil_div(nwl, kPlanThreads);
      const int w0 = imin(tid * wpt, nwl), w1 = imin(w0 + wpt, nwl);
      int n_eq = 0;
      for (int wi = w0; wi < w1; ++wi) n_eq += __popc(weq[wi]);
      int eq_before = block_exclusive_scan(n_eq, scan_scratch);
      if (tid == 0) part.n_eq = scan_scratch[32];
      cl.sync();
      {
        int tot;
        const int pre = rank_prefix(lane < C ? lane_part->n_eq : 0, tot);
        eq_before += __shfl_sync(0xffffffffu, pre, rank);
      }
      int n_sel = 0;
      for (int wi = w0; wi < w1; ++wi) {
        uint32_t e = weq[wi];
        const int take = imax(0, imin(__popc(e), need - eq_before));
        eq_before += __popc(e);
        uint32_t low = 0;
        for (int t = 0; t < take; ++t) {
          low |= e & (0u - e);
          e &= e - 1u;
        }
        const uint32_t sw = wsel[wi] | low;
        wsel[wi] = sw;
        n_sel += __popc(sw);
      }
      const int nb4 = block_exclusive_scan(n_sel, scan_scratch);
      (void)nb4;
      if (tid == 0) part.n_sel = scan_scratch[32];
      cl.sync();
      int tot;
      const int pre = rank_prefix(lane < C ? lane_part->n_sel : 0, tot);
      pos = __shfl_sync(0xffffffffu, pre, rank);
      __syncthreads();
    }

    // ---- 5. bitmap + ascending table ----
    const int wpt = ceil_div(nwl, kPlanThreads);  // words per thread (consecutive)
    const int w0 = imin(tid * wpt, nwl), w1 = imin(w0 + wpt, nwl);
    int n_sel = 0;
    for (int wi = w0; wi < w1; ++wi) n_sel += __popc(wsel[wi]);
    pos += block_exclusive_scan(n_sel, scan_scratch);
    int* trow = p.block_table + (int64_t)row * p.table_width;
    uint32_t* brow = p.bitmap + (int64_t)row * p.bm_words + lo / 32;
    for (int wi = w0; wi < w1; ++wi) {
      uint32_t s = wsel[wi];
      brow[wi] = s;
      while (s) {
        const int bit = __ffs(s) - 1;
        s &= s - 1u;
        if (pos < p.table_width) trow[pos] = lo + wi * 32 + bit;
        ++pos;
      }
    }
    if (rank == 0 && tid == 0) p.sel_lens[row] = nb > 0 ? K : 0;
    __syncthreads();  // shared buffers are reused by the next round
  }
  cl.sync();  // no CTA leaves while another may still read its shared memory
  pdl_launch_dependents();
}

PlanLayout plan_layout(int nb_max, int csize) {
  PlanLayout l{};
  l.csize = csize;
  l.slice_cap = (ceil_div(imax(nb_max, 1), csize) + 31) / 32 * 32;
  l.smem_keys = l.slice_cap <= kPlanSmemMaxKeys;
  const int nwl_alloc = (l.slice_cap / 32 + kPW - 1) / kPW * kPW;
  // the per-thread lists exist for slices long enough to use them
  const bool lists = l.slice_cap >= kFloorKeys;
  l.smem = (size_t)(l.smem_keys ? l.slice_cap : 0) * 4 + (size_t)2 * nwl_alloc * 4 +
           (lists ? (size_t)(kListCap + kWinCap) * kPlanThreads * (l.smem_keys ? 2 : 4) : 0);
  return l;
}

using PlanKernel = void (*)(PlanParams);

// the instantiation a layout and policy run (slices beyond the staging limit are long)
static PlanKernel plan_kernel_for(const PlanLayout& l, bool nucleus) {
  if (nucleus) {
    if (!l.smem_keys) return plan_kernel<false, true, true>;
    return l.slice_cap >= kFloorKeys ? plan_kernel<true, true, true> : plan_kernel<true, false, true>;
  }
  if (!l.smem_keys) return plan_kernel<false, true, false>;
  return l.slice_cap >= kFloorKeys ? plan_kernel<true, true, false> : plan_kernel<true, false, false>;
}

cudaError_t plan_kernels_init() {
  for (PlanKernel k : {plan_kernel<true, false, false>, plan_kernel<true, true, false>,
                       plan_kernel<false, true, false>, plan_kernel<true, false, true>,
                       plan_kernel<true, true, true>, plan_kernel<false, true, true>}) {
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPlanSmemMax);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

int plan_active_clusters(const PlanLayout& l, bool nucleus) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(l.csize, 1, 1);
  cfg.blockDim = dim3(kPlanThreads, 1, 1);
  cfg.dynamicSmemBytes = l.smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = l.csize;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  const cudaError_t e = cudaOccupancyMaxActiveClusters(&n, plan_kernel_for(l, nucleus), &cfg);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return 0;
  }
  return n;
}

cudaError_t launch_plan(const PlanParams& p, const PlanLayout& l, int grid, cudaStream_t st,
                        const LaunchOpts& o) {
  LaunchOpts oc = o;
  oc.cluster_x = (unsigned)l.csize;
  return launch_ex(plan_kernel_for(l, p.cfg.policy == ADAKV_POLICY_NUCLEUS), dim3(grid),
                   dim3(kPlanThreads), l.smem, st, oc, p);
}

}  // namespace adakv
