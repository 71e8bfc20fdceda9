// (c) Entropy-driven per-head budget and ragged per-head top-k block selection,
// one kernel, one CTA of 1024 threads per (sequence, query head).
//
// 1. The head's score row is staged in shared memory (coalesced loads) with
//    its max and content statistics in the same pass.
// 2. Weight, exactly the formula of adakv/budget.py:28-37: z = s / max(T, 1e-6),
//    p = softmax(z) in float32, w = -sum(p * log(max(p, 1e-9))) / log(max(nb, 2))
//    + 1e-6 (float64 after the division, as NumPy promotes it).
// 3. The Hq CTAs of a sequence exchange entropies through per-head 64-bit
//    slots (call tag | float32 entropy bits; tags cleared by the estimator):
//    each CTA publishes its word with one release store and warp 0 polls the
//    sequence's slots (bounded by a 200 ms wall-clock limit, after which the
//    status word records a timeout) while the other warps build the top-k
//    histogram.  Every CTA turns the Hq entropies into weights with the same
//    arithmetic and sums them in the same fixed order, so all heads see the
//    same total, and derives its count with the reference's arithmetic
//    (budget.py:71-86, selector.py:49-54; half-to-even rounding).  The grid is
//    at most one CTA per SM (so all of it is resident once the estimator
//    drains) and processes whole sequences per round.
// 4. Top-k: bucket select over the content blocks (sink [0, sink) and local
//    [nb-local, nb) are always taken, the reference's +inf bias,
//    selector.py:44-48): one histogram finds the bucket holding the k-th
//    score and its members are ranked exactly by (score, lowest index).  A
//    4-pass MSB radix select over order-preserving uint32 keys is the
//    fallback; blocks with key > T and the lowest-indexed blocks with key ==
//    T are selected.
// 5. Output: warp ballots build the selection bitmap word by word (element
//    j*1024 + t lands in word j*32 + warp), ties are resolved on the bitmap with
//    one block scan, and a second scan writes the ascending block table.
#include <algorithm>

#include "kernels.h"

namespace adakv {

__device__ __forceinline__ uint64_t ld_acquire_u64(const unsigned long long* p) {
  uint64_t v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_u64(unsigned long long* p, uint64_t v) {
  asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// single-barrier block sum: warp results in shared memory, then every warp
// folds the 32 partials itself (same order in every warp)
__device__ __forceinline__ double block_sum_1s(double v, double* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  return warp_sum(lane < (int)(blockDim.x >> 5) ? red[lane] : 0.0);
}

// order-preserving float -> uint32 map; NaN sorts below everything
__device__ __forceinline__ uint32_t score_key(float f) {
  const uint32_t u = __float_as_uint(f);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return 0u;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

constexpr int kPlanILP = 8;     // row elements per thread per tile (independent chains)
constexpr int kBuckets = 2048;  // bucket-select histogram bins (2 per thread)
constexpr int kCandCap = 1024;  // members of the boundary bucket ranked exactly

// bucket of a content score: floor((cmx - s) * scale), clamped to the last
// bucket (which also takes NaN and -inf); non-decreasing as s decreases
__device__ __forceinline__ int bucket_of(float s, float cmx, float scale) {
  const float u = __fmul_rn(__fsub_rn(cmx, s), scale);
  if (!(u < (float)(kBuckets - 1))) return kBuckets - 1;
  return u <= 0.f ? 0 : (int)u;
}

template <bool SMEM>
__global__ void __launch_bounds__(kPlanThreads, 1) plan_kernel(PlanParams p) {
  extern __shared__ __align__(16) uint32_t sm[];
  __shared__ uint32_t hist[kBuckets];
  __shared__ int s_digit, s_above, s_ncand;
  __shared__ int scan_scratch[33];
  __shared__ float fred[33], gred[33];
  __shared__ double dred[33], dred2[33];
  __shared__ double s_sumw;
  __shared__ int cand_idx[kCandCap];
  __shared__ uint32_t cand_key[kCandCap];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // ballot words are written 32 at a time: round the word count up to 32
  const int nw_alloc = (p.nw_max + 31) / 32 * 32;
  uint32_t* keys = sm;                                        // [nw_alloc * 32] (SMEM only)
  float* ecache = reinterpret_cast<float*>(sm + (SMEM ? nw_alloc * 32 : 0));  // exp(z - zmax)
  uint32_t* wsel = reinterpret_cast<uint32_t*>(ecache) + (p.ecache ? nw_alloc * 32 : 0);
  uint32_t* weq = wsel + nw_alloc;                            // [nw_alloc]

  pdl_wait();
  // per-call tag, never 0 (the estimator cleared every tag to 0)
  const uint32_t ep = (*reinterpret_cast<const volatile uint32_t*>(p.epoch) & 0x7FFFFFFFu) | 0x80000000u;
  const int h = blockIdx.x % p.Hq;
  const int slot_seq = blockIdx.x / p.Hq;

  for (int b0 = 0; b0 < p.B; b0 += p.seqs_per_round) {
    const int b = b0 + slot_seq;
    if (b >= p.B) break;
    const int row = b * p.Hq + h;
    int S = seq_len_of(p.seq_lens, b, p.max_seq_len);
    if (S < 0 || S > p.max_seq_len) S = 0;  // reported by the estimator
    const int nb = ceil_div(S, p.bs);
    const int nw = ceil_div(nb, 32);
    const float* srow = p.scores + (int64_t)row * p.score_stride;

    auto val = [&](int i) -> float { return SMEM ? __uint_as_float(keys[i]) : srow[i]; };
    const int sink = imin(p.cfg.n_sink, nb), local = imin(p.cfg.n_local, nb);
    auto forced = [&](int i) -> bool { return i < sink || i >= nb - local; };

    // ---- load the row (staged in shared memory) and its statistics in one pass:
    //      max (softmax), content max / mean / spread (top-k buckets) ----
    float mx = -INFINITY, cmx = -INFINITY, csum_f = 0.f, csq_f = 0.f;
    for (int base = 0; base < nb; base += kPlanThreads * kPlanILP) {
      float v[kPlanILP];
#pragma unroll
      for (int r = 0; r < kPlanILP; ++r) {
        const int i = base + r * kPlanThreads + tid;
        v[r] = i < nb ? srow[i] : -INFINITY;
      }
#pragma unroll
      for (int r = 0; r < kPlanILP; ++r) {
        const int i = base + r * kPlanThreads + tid;
        if (i < nb) {
          if (SMEM) keys[i] = __float_as_uint(v[r]);
          mx = fmaxf(mx, v[r]);
          if (!forced(i)) {
            cmx = fmaxf(cmx, v[r]);
            csum_f += v[r];
            csq_f = fmaf(v[r], v[r], csq_f);
          }
        }
      }
    }
    {
      mx = warp_max(mx);
      cmx = warp_max(cmx);
      double csum_w = warp_sum((double)csum_f), csq_w = warp_sum((double)csq_f);
      __syncthreads();
      if (lane == 0) {
        fred[warp] = mx;
        gred[warp] = cmx;
        dred[warp] = csum_w;
        dred2[warp] = csq_w;
      }
      __syncthreads();  // also publishes the staged row
      mx = warp_max(fred[lane]);
      cmx = warp_max(gred[lane]);
    }
    const double csum = warp_sum(dred[lane]), csq = warp_sum(dred2[lane]);

    // ---- entropy (adakv/budget.py:28-37) ----
    float ent = 0.f;
    if (nb >= 2 && p.cfg.policy == ADAKV_POLICY_ADAPTIVE) {
      const float m = mx;
      const float Tf = (float)(p.cfg.temperature > 1e-6 ? p.cfg.temperature : 1e-6);
      const bool unit_t = (Tf == 1.0f);  // s / 1 == s exactly: skip the division
      const float zmax = unit_t ? m : __fdiv_rn(m, Tf);  // max(s / T) == max(s) / T (monotone rounding)
      auto ez = [&](int i) -> float {
        const float z = unit_t ? val(i) : __fdiv_rn(val(i), Tf);
        return expf(z - zmax);
      };
      // per-thread partial sums in float (at most a few dozen terms each), the
      // cross-thread sums in double
      float zpart = 0.f;
      for (int base = 0; base < nb; base += kPlanThreads * kPlanILP) {
#pragma unroll
        for (int r = 0; r < kPlanILP; ++r) {
          const int i = base + r * kPlanThreads + tid;
          if (i < nb) {
            const float e = ez(i);
            if (p.ecache) ecache[i] = e;
            zpart += e;
          }
        }
      }
      const float Z = (float)block_sum_1s((double)zpart, dred);
      float hpart = 0.f;
      for (int base = 0; base < nb; base += kPlanThreads * kPlanILP) {
#pragma unroll
        for (int r = 0; r < kPlanILP; ++r) {
          const int i = base + r * kPlanThreads + tid;
          if (i < nb) {
            const float e = p.ecache ? ecache[i] : ez(i);
            const float pi = __fdiv_rn(e, Z);
            hpart += __fmul_rn(pi, logf(fmaxf(pi, 1e-9f)));
          }
        }
      }
      const float hsum = (float)block_sum_1s((double)hpart, dred);
      ent = -hsum;
    }
    auto weight_of = [&](float e) -> double {  // adakv/budget.py:36-37, float64 after the division
      return (double)e / log((double)imax(nb, 2)) + 1e-6;
    };
    const double w = (nb >= 2 && p.cfg.policy == ADAKV_POLICY_ADAPTIVE) ? weight_of(ent) : 0.0;

    // ---- publish (entropy, tag) in one 64-bit release store ----
    unsigned long long* myslot = &p.slots[row].word;
    if (tid == 0) st_release_u64(myslot, ((uint64_t)ep << 32) | (uint64_t)__float_as_uint(ent));

    // ---- bucket histogram (independent of the budget) while warp 0 waits ----
    const double nc_d = (double)(nb - imin(nb, sink + local));
    const double mean_c = nc_d > 0 ? csum / nc_d : 0.0;
    const double var_c = nc_d > 0 ? csq / nc_d - mean_c * mean_c : 0.0;
    const double range = (double)cmx - mean_c + (var_c > 0.0 ? sqrt(var_c) : 0.0);
    const bool buckets_ok = isfinite(cmx) && range > 0.0 && isfinite(range);
    const float scale = buckets_ok ? (float)((double)(kBuckets - 1) / range) : 0.f;
    for (int t = tid; t < kBuckets; t += kPlanThreads) hist[t] = 0u;
    __syncthreads();
    if (warp == 0) {
      const uint64_t t0 = globaltimer_ns();
      bool ok = false;
      float ents[4];  // Hq <= 128
      while (true) {
        bool mine = true;
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          const int hh = lane + q4 * 32;
          if (hh < p.Hq) {
            const uint64_t v = ld_acquire_u64(&p.slots[b * p.Hq + hh].word);
            mine &= ((uint32_t)(v >> 32) == ep);
            ents[q4] = __uint_as_float((uint32_t)v);
          }
        }
        ok = __all_sync(0xffffffffu, mine);
        if (ok || globaltimer_ns() - t0 > kWaitLimitNs) break;
      }
      if (!ok && lane == 0) report(p.status, ADAKV_ST_WAIT_TIMEOUT);
      double part = 0.0;
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        const int hh = lane + q4 * 32;
        if (hh < p.Hq && p.cfg.policy == ADAKV_POLICY_ADAPTIVE && nb >= 2) part += weight_of(ents[q4]);
      }
      part = warp_sum(part);  // fixed xor tree: every CTA of the sequence gets the same sum
      if (lane == 0) s_sumw = part;
    } else if (buckets_ok) {
      for (int i = tid - 32; i < nb; i += kPlanThreads - 32) {
        if (!forced(i)) {
          const int bk = bucket_of(val(i), cmx, scale);
          if (bk < kBuckets - 1) atomicAdd(&hist[bk], 1u);
        }
      }
    }
    __syncthreads();
    pdl_launch_dependents();  // every CTA is past the exchange: the attend grid may launch
    const SeqBudget sbud = seq_budget(nb, p.cfg);
    const int K = imin(head_count(sbud, p.cfg, w, s_sumw, p.Hq), p.table_width);
    const int n_forced = (sink + local >= nb) ? nb : sink + local;
    const int Kc = K - n_forced;  // content blocks to pick

    // ---- top-k ----
    // Bucket select: content block i goes to bucket floor((cmx - s_i) * scale),
    // a non-decreasing function of -s_i (correctly rounded subtraction and
    // multiplication are monotone), so every block of a lower bucket outranks
    // every block of a higher one.  Buckets span [cmx - range, cmx] with
    // range = cmx - mean + sd, fine near the k-th score; blocks past the range
    // share the last bucket.  One histogram pass finds the bucket holding the
    // Kc-th block; its few members are ranked exactly by (score, lowest index).
    // A full MSB radix select takes over when the boundary falls in the last
    // bucket or holds too many members.
    bool use_radix = false;
    int jstar = kBuckets, need_b = 0;
    if (K < nb && Kc > 0) {
      use_radix = !buckets_ok;
      if (!use_radix) {
        // find the bucket holding the Kc-th content block (buckets ascend = scores descend)
        constexpr int BPT = kBuckets / kPlanThreads;
        uint32_t cb[BPT], tot = 0;
#pragma unroll
        for (int e = 0; e < BPT; ++e) {
          cb[e] = hist[tid * BPT + e];
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
        if (jstar >= kBuckets - 1 || (int)hist[jstar] > kCandCap) {
          use_radix = true;
        } else {
          need_b = Kc - s_above;
          if (tid == 0) s_ncand = 0;
          __syncthreads();
          for (int base = 0; base < nb; base += kPlanThreads * kPlanILP) {
#pragma unroll
            for (int r = 0; r < kPlanILP; ++r) {
              const int i = base + r * kPlanThreads + tid;
              if (i < nb && !forced(i)) {
                const float v = val(i);
                if (bucket_of(v, cmx, scale) == jstar) {
                  const int slot = atomicAdd(&s_ncand, 1);
                  cand_idx[slot] = i;
                  cand_key[slot] = score_key(v);
                }
              }
            }
          }
          __syncthreads();
        }
      }
    }

    uint32_t T = 0;
    int need = 0;  // ties at T resolved in index order (radix path only)
    if (use_radix) {
      if (SMEM) {
        for (int i = tid; i < nb; i += kPlanThreads)
          keys[i] = forced(i) ? 0xFFFFFFFFu : score_key(__uint_as_float(keys[i]));
        __syncthreads();
      }
      auto key = [&](int i) -> uint32_t {
        return SMEM ? keys[i] : (forced(i) ? 0xFFFFFFFFu : score_key(srow[i]));
      };
      uint32_t prefix = 0, pmask = 0;
      int rem = K;
#pragma unroll 1
      for (int pass = 0; pass < 4; ++pass) {
        const int shift = 24 - 8 * pass;
        if (tid < 256) hist[tid] = 0;
        __syncthreads();
        for (int i = tid; i < nb; i += kPlanThreads) {
          const uint32_t k = key(i);
          if ((k & pmask) == prefix) atomicAdd(&hist[(k >> shift) & 0xFFu], 1u);
        }
        __syncthreads();
        if (warp == 0) {
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
      }
      T = prefix;
      need = rem;
      for (int j = 0; j * kPlanThreads < nb; ++j) {
        const int i = j * kPlanThreads + tid;
        const bool valid = i < nb;
        const uint32_t k = valid ? key(i) : 0u;
        const uint32_t bgt = __ballot_sync(0xffffffffu, valid && k > T);
        const uint32_t beq = __ballot_sync(0xffffffffu, valid && k == T);
        if (lane == 0) {
          wsel[j * 32 + warp] = bgt;
          weq[j * 32 + warp] = beq;
        }
      }
    } else {
      // selected: forced blocks, every content block of a bucket above jstar,
      // and the need_b best members of bucket jstar
      const bool all = K >= nb;
      for (int j = 0; j * kPlanThreads < nb; ++j) {
        const int i = j * kPlanThreads + tid;
        bool sel = false;
        if (i < nb) {
          if (all || forced(i)) sel = true;
          else if (Kc > 0 && jstar < kBuckets) sel = bucket_of(val(i), cmx, scale) < jstar;
        }
        const uint32_t bsel = __ballot_sync(0xffffffffu, sel);
        if (lane == 0) {
          wsel[j * 32 + warp] = bsel;
          weq[j * 32 + warp] = 0u;
        }
      }
      __syncthreads();
      if (!all && Kc > 0 && jstar < kBuckets) {
        const int nc = s_ncand;
        for (int t = tid; t < nc; t += kPlanThreads) {
          const uint32_t kt = cand_key[t];
          const int it = cand_idx[t];
          int rank = 0;
          for (int c = 0; c < nc; ++c) {
            const uint32_t kc = cand_key[c];
            rank += (kc > kt) || (kc == kt && cand_idx[c] < it);
          }
          if (rank < need_b) atomicOr(&wsel[it >> 5], 1u << (it & 31));
        }
      }
    }
    __syncthreads();
    const int wpt = ceil_div(nw, kPlanThreads);  // words per thread (consecutive)
    const int w0 = imin(tid * wpt, nw), w1 = imin(w0 + wpt, nw);
    int n_sel = 0;
    if (use_radix) {
      int n_eq = 0;
      for (int wi = w0; wi < w1; ++wi) n_eq += __popc(weq[wi]);
      int eq_before = block_exclusive_scan(n_eq, scan_scratch);
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
    } else {
      for (int wi = w0; wi < w1; ++wi) n_sel += __popc(wsel[wi]);
    }
    int pos = block_exclusive_scan(n_sel, scan_scratch);
    int* trow = p.block_table + (int64_t)row * p.table_width;
    uint32_t* brow = p.bitmap + (int64_t)row * p.bm_words;
    for (int wi = w0; wi < w1; ++wi) {
      uint32_t s = wsel[wi];
      brow[wi] = s;
      while (s) {
        const int bit = __ffs(s) - 1;
        s &= s - 1u;
        if (pos < p.table_width) trow[pos] = wi * 32 + bit;
        ++pos;
      }
    }
    if (tid == 0) p.sel_lens[row] = nb > 0 ? K : 0;
    __syncthreads();  // shared buffers are reused by the next round
  }
  pdl_launch_dependents();
}

bool plan_ecache(int nb_max) { return nb_max <= kPlanECacheMax; }

size_t plan_smem_bytes(int nb_max) {
  const int nw_alloc = (ceil_div(imax(nb_max, 1), 32) + 31) / 32 * 32;
  const bool smem_keys = nb_max <= kPlanSmemMaxKeys;
  return (size_t)(smem_keys ? nw_alloc * 32 : 0) * 4 +
         (size_t)(plan_ecache(nb_max) ? nw_alloc * 32 : 0) * 4 + (size_t)2 * nw_alloc * 4;
}

cudaError_t plan_kernels_init() {
  cudaError_t e = cudaFuncSetAttribute(plan_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)std::max(plan_smem_bytes(kPlanSmemMaxKeys),
                                                     plan_smem_bytes(kPlanECacheMax)));
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(plan_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)plan_smem_bytes(kPlanMaxBlocks));
}

int plan_ctas_per_sm(int nb_max) {
  int n = 0;
  const size_t smem = plan_smem_bytes(nb_max);
  if (nb_max <= kPlanSmemMaxKeys)
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, plan_kernel<true>, kPlanThreads, smem);
  else
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, plan_kernel<false>, kPlanThreads, smem);
  return n;
}

cudaError_t launch_plan(const PlanParams& p, int nb_max, int grid, cudaStream_t st,
                        const LaunchOpts& o) {
  const size_t smem = plan_smem_bytes(nb_max);
  if (nb_max <= kPlanSmemMaxKeys)
    return launch_ex(plan_kernel<true>, dim3(grid), dim3(kPlanThreads), smem, st, o, p);
  return launch_ex(plan_kernel<false>, dim3(grid), dim3(kPlanThreads), smem, st, o, p);
}

}  // namespace adakv
