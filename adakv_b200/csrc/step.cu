// (a)-(d) One AdaKV decode step in one persistent kernel.
//
// One CTA per SM (256 threads), launched as thread-block clusters of C CTAs
// (C chosen by the host).  The step's three dependent stages run as phases of
// the same grid with no kernel boundary between them:
//   A -> B: every CTA adds one to a monotonic arrival counter (release) when
//           its scores and statistics records are written; a selection CTA
//           waits for this call's GRID arrivals (acquire);
//   B -> B, B -> C, C -> C: the head entropies, the ready words of the
//           selection bitmaps and the attention partials' flags are tagged
//           64-bit words (call tag << 32 | payload): a reader re-reads, all at
//           once, the words that do not carry this call's tag yet, so it
//           proceeds one round trip after the last one lands, and nothing has
//           to be reset between calls.
// Every wait is bounded in time; on expiry the status word records
// ADAKV_ST_WAIT_TIMEOUT and the kernel runs to completion on what it has.
//
// Phase A -- append + estimator (adakv/runtime.py:43-60, adakv/estimator.py:73-74).
//   The (sequence, KV head, block) rows of every centroid table form one list,
//   split evenly over the CTAs.  A CTA streams its rows through a 6-stage ring
//   of 64-row stages with 1-D bulk copies (TMA engine, one CTA per copy); each
//   stage is refilled by the last warp to finish with it.  A warp scores 8
//   rows per stage against the g query heads of the row's KV head: LPR = 2g
//   lanes share a row (D / LPR dims each, queries in registers) and one
//   reduce-scatter over those lanes leaves every head's score in a lane.
//   Scores go out as plain floats, and each warp folds them per head into a
//   softmax record (max, content max / sum / sum of squares, m, Z, A) stored
//   once per (sequence, KV head) run of its CTA.  When the step appends
//   tokens, warp 7 of CTA (b * Hkv + kvh) first writes them into the K/V
//   cache, recomputes the touched blocks' centroids from their tokens
//   (token-order float32 sum, one IEEE division: bit-identical to a rebuild)
//   and scores those rows itself.
//
// Phase B -- entropy budget + top-k (adakv/budget.py:28-86, adakv/selector.py:18-60).
//   One cluster of C CTAs per query head; rank r owns a 32-aligned slice of
//   the score row.  Every CTA folds the head's estimator records (and the
//   rows the append scored) into the row's max, content statistics and
//   softmax sums, the same arithmetic in every rank; one pass over the slice
//   builds the 2048-bucket content histogram and the clamp correction of the
//   entropy H = log Z - A / Z - Cc / Z (Cc: the reference's max(p, 1e-9)
//   clamp); histograms and clamp terms merge through distributed shared
//   memory and rank 0 publishes H.  Warp 0 polls the H of every head of the
//   sequence; every CTA derives the same per-head counts (fixed-order sums,
//   half-to-even rounding).  A head's selection is the forced sink/local
//   blocks, every block of the buckets above the threshold bucket, and the
//   exactly ranked (score desc, index asc) top members of that bucket,
//   gathered from every rank; an exact 4-pass radix select over
//   order-preserving keys covers the rows the buckets cannot resolve.  Each
//   rank writes its bitmap words and table segment, then a ready word.
//
// Phase C -- block-sparse split-KV flash decode (adakv/kernels/block_sparse_decode.py:51-100).
//   The CTAs are split into B * Hkv contiguous groups, one per (sequence, KV
//   head).  A CTA polls the ready words of its group's g heads, ORs their
//   bitmaps into the union, takes its share of it and gathers those K/V blocks
//   (16-byte cp.async, zero-filled past seq_len, XOR-swizzled tiles) for an
//   m16n8k16 tensor-core pass over the g query rows (each head masked by its
//   own selection), then publishes its (m, l, o) partial.  Every CTA of the
//   group then merges all the group's partials, in split order, for its own
//   share of the output columns.
//
// HBM traffic: the float32 centroid tables, the union of the selected K/V
// blocks and the appended tokens; scores, records, bitmaps and partials stay
// in L2.
//
// Memory ordering across CTAs: the appended K/V tokens reach the attend phase
// through the arrival counter (release after the cache writes, acquire by the
// selection CTA) and fences around the ready words (selection CTA: fence
// before publishing; attend CTA: fence after reading them).
//
// All CTAs must be resident at once (they wait on one another): the host
// launches at most one CTA per SM, sized by the cluster occupancy, and every
// wait is bounded.
#include <cooperative_groups.h>

#include "attend_mma.cuh"
#include "kernels.h"

namespace cg = cooperative_groups;

namespace adakv {

namespace {

constexpr int kSW = kStepThreads / 32;  // warps per CTA
constexpr int kBk = 2048;               // selection buckets
constexpr int kDebugSkipPublish = 1;
constexpr int kDebugTimeline = 2;

// debug timeline: globaltimer stamp `slot` of this CTA (one thread calls it)
#define STEP_STAMP(slot) \
  do { \
    if (p.debug_flags & kDebugTimeline) p.timeline[cta * kStepTimelineSlots + (slot)] = globaltimer_ns(); \
  } while (0)

__device__ __forceinline__ float h16lo(uint32_t w, const __nv_bfloat16*) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float h16hi(uint32_t w, const __nv_bfloat16*) {
  return __uint_as_float(w & 0xFFFF0000u);
}
__device__ __forceinline__ float h16lo(uint32_t w, const __half*) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(w & 0xFFFFu)));
}
__device__ __forceinline__ float h16hi(uint32_t w, const __half*) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(w >> 16)));
}

// four consecutive 16-bit elements -> fp32
template <typename T>
__device__ __forceinline__ void load4(const T* p, float (&f)[4]) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  f[0] = h16lo(u.x, (const T*)nullptr);
  f[1] = h16hi(u.x, (const T*)nullptr);
  f[2] = h16lo(u.y, (const T*)nullptr);
  f[3] = h16hi(u.y, (const T*)nullptr);
}

// Reduce-scatter of G per-lane partial sums over groups of LPR lanes (lane
// bits below LPR): afterwards every lane holds the group-wide sum of head
// (sub >> log2(LPR / G)) (sub = lane % LPR); the last levels are plain
// all-reduces of that one value.
template <int G, int LPR>
__device__ __forceinline__ float reduce_heads(float (&v)[G], int lane) {
#pragma unroll
  for (int lvl = 0; (LPR >> (lvl + 1)) >= 1; ++lvl) {
    const int off = LPR >> (lvl + 1);
    const int nv = G >> lvl;
    if (nv > 1) {
      const int half = nv / 2;
      const bool upper = (lane & off) != 0;
#pragma unroll
      for (int i = 0; i < half; ++i) {
        const float send = upper ? v[i] : v[i + half];
        const float keep = upper ? v[i + half] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
      }
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], off);
    }
  }
  return v[0];
}

// bucket of a content score: floor((cmx - s) * scale), clamped to the last
// bucket (which also takes NaN and -inf); non-decreasing as s decreases
__device__ __forceinline__ int bucket_of(float s, float cmx, float scale) {
  const float u = __fmul_rn(__fsub_rn(cmx, s), scale);
  if (!(u < (float)(kBk - 1))) return kBk - 1;
  return u <= 0.f ? 0 : (int)u;
}

// block-wide sums of two doubles: every thread gets the same result (warp
// xor trees, then the kSW warp values folded in warp order)
__device__ __forceinline__ void block_sum2d(double& a, double& b, double (*red)[4]) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  a = warp_sum(a);
  b = warp_sum(b);
  __syncthreads();
  if (lane == 0) {
    red[warp][0] = a;
    red[warp][1] = b;
  }
  __syncthreads();
  a = 0.0;
  b = 0.0;
#pragma unroll
  for (int w = 0; w < kSW; ++w) {
    a += red[w][0];
    b += red[w][1];
  }
}

// Exact top-K of one score row by a 4-pass MSB radix select over order-preserving
// keys (forced sink / local blocks take the largest key), ties at the threshold
// to the lowest block indices; the selection is ORed into sbits (its forced
// bits may already be set).  The fallback for rows the buckets cannot resolve,
// kept out of line so that its code is not fetched on the common path.
// srow is overwritten with the keys; hist (256 words) and weq (nw words) are scratch.
__device__ __noinline__ void radix_select_top(float* srow, int nb, int sink, int local, int K,
                                              uint32_t* hist, uint32_t* weq, uint32_t* sbits,
                                              int* scan_scratch, int* s_digit, int* s_above) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nw = ceil_div(nb, 32);
  __syncthreads();
  for (int j = tid; j < nb; j += kStepThreads) {
    const bool f = j < sink || j >= nb - local;
    srow[j] = __uint_as_float(f ? 0xFFFFFFFFu : order_key(srow[j]));
  }
  uint32_t prefix = 0, pmask = 0;
  int rem = K;
#pragma unroll 1
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    __syncthreads();
    for (int t = tid; t < 256; t += kStepThreads) hist[t] = 0u;
    __syncthreads();
    for (int j = tid; j < nb; j += kStepThreads) {
      const uint32_t k = __float_as_uint(srow[j]);
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
            *s_digit = 255 - 8 * lane - e;
            *s_above = (int)acc;
            break;
          }
          acc += c[e];
        }
      }
    }
    __syncthreads();
    rem -= *s_above;
    prefix |= (uint32_t)*s_digit << shift;
    pmask |= 0xFFu << shift;
  }
  // keys above the threshold, then the first `rem` keys equal to it in index order
  for (int w = warp; w < nw; w += kSW) {
    const int j = w * 32 + lane;
    const uint32_t k = j < nb ? __float_as_uint(srow[j]) : 0u;
    const uint32_t gt = __ballot_sync(0xffffffffu, j < nb && k > prefix);
    const uint32_t eq = __ballot_sync(0xffffffffu, j < nb && k == prefix);
    if (lane == 0) {
      sbits[w] |= gt;
      weq[w] = eq;
    }
  }
  __syncthreads();
  const int wpt = ceil_div(nw, kStepThreads);
  const int w0 = imin(tid * wpt, nw), w1 = imin(w0 + wpt, nw);
  int n_eq = 0;
  for (int w = w0; w < w1; ++w) n_eq += __popc(weq[w]);
  int eq_before = block_exclusive_scan(n_eq, scan_scratch);
  for (int w = w0; w < w1; ++w) {
    uint32_t e = weq[w];
    const int take = imax(0, imin(__popc(e), rem - eq_before));
    eq_before += __popc(e);
    uint32_t low = 0;
    for (int t = 0; t < take; ++t) {
      low |= e & (0u - e);
      e &= e - 1u;
    }
    sbits[w] |= low;
  }
}

// shared-memory carve-up of one step CTA; the three phases reuse the same bytes
struct StepSmem {
  size_t ring;                                                      // phase A
  size_t srow, sbk, sbits, hist, ghist, ckey, cidx, akey, aidx, b_end;  // phase B
  size_t kv, uw, hw, list, mask, wpart, c_end;                      // phase C
  size_t total;
};

__host__ __device__ inline StepSmem step_smem_layout(int D, int g, int nb_max, int nbt, int slice_cap,
                                                     int csize) {
  auto al = [](size_t x) { return (x + 127) / 128 * 128; };
  const int nw = (nb_max + 31) / 32;
  const int ls = ((nb_max + csize - 1) / csize + 31) / 32 * 32;  // slice of one cluster rank
  StepSmem s;
  s.ring = al((size_t)kStepStages * (kStepRows * D * 4 + g * D * 2));
  s.srow = 0;  // the slice; the whole row on the exact (radix) path
  s.sbk = s.srow + al((size_t)nb_max * 4);
  s.sbits = s.sbk + al((size_t)ls * 2);
  s.hist = s.sbits + al((size_t)nw * 4);
  s.ghist = s.hist + al((size_t)kBk * 4);
  s.ckey = s.ghist + al((size_t)(kBk > nw ? kBk : nw) * 4);
  s.cidx = s.ckey + al((size_t)kStepCandCap * 4);
  s.akey = s.cidx + al((size_t)kStepCandCap * 4);
  s.aidx = s.akey + al((size_t)kStepCandCap * 4);
  s.b_end = s.aidx + al((size_t)kStepCandCap * 4);
  s.kv = 0;
  s.uw = s.kv + al((size_t)2 * 2 * nbt * 16 * D * 2);
  s.hw = s.uw + al((size_t)nw * 4);
  s.list = s.hw + al((size_t)g * nw * 4);
  s.mask = s.list + al((size_t)slice_cap * 4);
  s.wpart = s.mask + al((size_t)slice_cap * 4);
  s.c_end = s.wpart + al((size_t)kSW * g * (D + 2) * 4);
  size_t t = s.ring;
  t = t > s.b_end ? t : s.b_end;
  t = t > s.c_end ? t : s.c_end;
  s.total = t;
  return s;
}

// One cluster rank's share of a head's selection, read by the other ranks
// through distributed shared memory.
struct RankPart {
  double Cc;               // clamp correction of the slice
  int ncand, nsel;         // threshold-bucket candidates; selected blocks of the slice
};

// A head's row statistics: max score, content max / sum / sum of squares, and
// Z = sum e^(z - m), A = sum e^(z - m) (z - m) of z = s / T relative to m = max z.
struct RowStats {
  float mx, cmx, m;
  double cs, cq, Z, A;
};

// floor(a b / c) in 32-bit unsigned arithmetic: every use has a b < 2^31
// (rows <= kStepMaxHeads * kStepMaxBlocks = 2^22, grid <= 256)
__device__ __forceinline__ int muldiv(int a, int b, int c) {
  return (int)(((unsigned)a * (unsigned)b) / (unsigned)c);
}
// The CTA whose estimator rows [floor(R c / grid), floor(R (c + 1) / grid)) hold row r.
__device__ __forceinline__ int cta_of_row(int r, int R, int grid) {
  return (int)(((unsigned)(r + 1) * (unsigned)grid - 1u) / (unsigned)R);
}
__device__ __forceinline__ int first_row_of(int c, int R, int grid) { return muldiv(R, c, grid); }

// a sequence takes part when 1 <= S <= max_seq_len and it holds the appended tokens
__device__ __forceinline__ int valid_len(const StepParams& p, int b) {
  const int S = seq_len_of(p.seq_lens, b, p.max_seq_len);
  const bool ok = S > 0 && S <= p.max_seq_len && (p.n_new <= 0 || S >= p.n_new);
  return ok ? S : 0;
}

}  // namespace

template <typename T, int D, int G>
__global__ void __launch_bounds__(kStepThreads, 1) step_kernel(StepParams p) {
  constexpr int BS = 16;
  constexpr int LPR = 2 * G;             // lanes per centroid row
  constexpr int RPP = 32 / LPR;          // rows per warp pass
  constexpr int RPW = kStepRows / kSW;   // rows per warp and stage
  constexpr int PASSES = RPW / RPP;
  constexpr int DL = D / LPR;            // dims per lane
  constexpr int CH = DL / 4;             // float4 chunks per lane and row
  constexpr int E = D / 32;              // dims per lane in the refresh warp
  constexpr int VEC = 8;                 // 16-bit elements per 16-byte chunk
  constexpr int ROWC = D / VEC;          // 16-byte chunks per token row
  constexpr int BLK = BS * D;            // elements of one K (or V) block
  static_assert(CH >= 1 && RPW % RPP == 0 && E == 4, "unsupported step shape");

  extern __shared__ __align__(128) unsigned char sm[];
  __shared__ __align__(8) uint64_t full_bar[kStepStages];
  __shared__ int rel_cnt[kStepStages];
  __shared__ int4 sdesc[kStepMaxDesc];
  __shared__ int s_nstage;
  __shared__ int s_S[kStepMaxBatch];
  __shared__ int s_rb[kStepMaxBatch + 1];
  __shared__ uint32_t s_tag;
  __shared__ double redd[kSW][4];
  __shared__ float redm[kSW][3];
  __shared__ int scan_scratch[33];
  __shared__ double s_w, s_sumw;
  __shared__ int s_jstar, s_digit, s_above, s_ncand;
  __shared__ RankPart s_part;
  __shared__ RowStats s_row;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int GRID = gridDim.x, cta = blockIdx.x;
  const bool appending = p.n_new > 0 && p.k_new.data != nullptr;

  // Nothing is read before the previous kernel on the stream has completed:
  // q, the caches, the centroid table and seq_lens may all be its outputs.
  pdl_wait();

  // ---------------------------------------------------------------- set-up
  if (tid == 0) {
    STEP_STAMP(0);
    for (int s = 0; s < kStepStages; ++s) {
      mbar_init(&full_bar[s], 1);
      rel_cnt[s] = 0;
    }
  }
  if (tid == 32) {  // the call tag, read beside the sequence lengths
    const uint32_t e = *reinterpret_cast<volatile uint32_t*>(p.epoch);
    s_tag = (e + 1u) ? e + 1u : 1u;
  }
  if (tid < p.B) {
    const int S = valid_len(p, tid);
    s_S[tid] = S;
    if (S == 0 && cta == 0) report(p.status, ADAKV_ST_BAD_SEQ_LEN);
  }
  __syncthreads();
  const uint32_t tag = s_tag;
  if (warp == 0) {  // row list prefix over the sequences (B <= 32)
    const int nbb = lane < p.B ? ceil_div(s_S[lane], BS) : 0;
    const int cnt = p.Hkv * nbb;
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane < p.B) s_rb[lane] = incl - cnt;
    if (lane == 31) s_rb[p.B] = incl;
    __syncwarp();
    if (lane == 0) {
      // this CTA's rows [r0, r1) as ring stages of <= 64 rows of one (sequence, KV head)
      const int R = s_rb[p.B];
      const int r0 = first_row_of(cta, R, GRID), r1 = first_row_of(cta + 1, R, GRID);
      int r = r0, ns = 0, b = 0;
      while (r < r1) {
        while (r >= s_rb[b + 1]) ++b;
        const int nb = ceil_div(s_S[b], BS);
        const int loc = r - s_rb[b];
        const int kvh = loc / nb, j = loc - kvh * nb;
        const int n = imin(kStepRows, imin(nb - j, r1 - r));
        const int skip = appending ? (s_S[b] - p.n_new) / BS : nb;  // first refreshed block
        if (ns == kStepMaxDesc) {  // the host sizes grids so that this cannot happen
          report(p.status, ADAKV_ST_WAIT_TIMEOUT);
          break;
        }
        sdesc[ns++] = make_int4(b * p.Hkv + kvh, j, n, imax(0, skip - j));
        r += n;
      }
      s_nstage = ns;
    }
  }
  __syncthreads();
  const int nstage = s_nstage;
  // ring stage: kStepRows centroid rows (fp32), then the G query rows of
  // the stage's KV head (T), both brought by the TMA engine
  constexpr int STAGE_F = kStepRows * D + G * D * (int)sizeof(T) / 4;  // floats per stage
  float* ring = reinterpret_cast<float*>(sm);
  auto issue = [&](int i, int slot) {
    const int4 d = sdesc[i];
    const uint32_t bytes = (uint32_t)d.z * D * 4u;
    const int b = d.x / p.Hkv, kvh = d.x - b * p.Hkv;
    float* st = ring + slot * STAGE_F;
    mbar_arrive_expect_tx(&full_bar[slot], bytes + (uint32_t)(G * D * sizeof(T)));
    bulk_g2s(st, p.cent + ((int64_t)d.x * p.nb_cap + d.y) * D, bytes, &full_bar[slot]);
    const T* qsrc = static_cast<const T*>(p.q.data) + b * p.q.sb + (int64_t)kvh * G * p.q.sh;
#pragma unroll
    for (int j = 0; j < G; ++j)
      bulk_g2s(reinterpret_cast<T*>(st + kStepRows * D) + j * D, qsrc + j * p.q.sh,
               (uint32_t)(D * sizeof(T)), &full_bar[slot]);
  };
  // the append refresh reads the touched block's older tokens: warm L2 with
  // them before this CTA's estimator burst fills the DRAM queues
  if (appending && warp == kSW - 1 && cta < p.B * p.Hkv) {
    const int b = cta / p.Hkv, kvh = cta - b * p.Hkv;
    const int S = s_S[b];
    if (S > 0) {
      const int S_old = S - p.n_new;
      const T* kc = static_cast<const T*>(p.k.data) + b * p.k.sb + kvh * p.k.sh;
      for (int t = (S_old / BS) * BS + (lane >> 1); t < S_old; t += 16) {
        const char* row = reinterpret_cast<const char*>(kc + (int64_t)t * p.k.ss);
        asm volatile("prefetch.global.L2 [%0];" ::"l"(row + (lane & 1) * 128) : "memory");
      }
    }
  }
  __syncthreads();
  if (tid == 0)
    for (int i = 0; i < imin(kStepStages, nstage); ++i) issue(i, i);

  // ---------------------------------------------------------------- phase A
  // fused append: warp 7 of CTA (b * Hkv + kvh) refreshes that table's tail
  if (appending && warp == kSW - 1 && cta < p.B * p.Hkv) {
    const int b = cta / p.Hkv, kvh = cta - b * p.Hkv;
    const int S = s_S[b];
    if (S > 0) {
      const int S_old = S - p.n_new;
      const int nb = ceil_div(S, BS);
      const int d = lane * E;
      T* kc = static_cast<T*>(const_cast<void*>(p.k.data)) + b * p.k.sb + kvh * p.k.sh + d;
      T* vc = static_cast<T*>(const_cast<void*>(p.v.data)) + b * p.v.sb + kvh * p.v.sh + d;
      const T* kn = static_cast<const T*>(p.k_new.data) + b * p.k_new.sb + kvh * p.k_new.sh + d;
      const T* vn = static_cast<const T*>(p.v_new.data) + b * p.v_new.sb + kvh * p.v_new.sh + d;
      const T* qb = static_cast<const T*>(p.q.data) + b * p.q.sb + (int64_t)kvh * G * p.q.sh + d;
      float qv[G][E];
#pragma unroll
      for (int j = 0; j < G; ++j) load4<T>(qb + j * p.q.sh, qv[j]);
      for (int blk = S_old / BS; blk < nb; ++blk) {
        const int t0 = blk * BS, t1 = imin(t0 + BS, S);
        uint2 x[BS];
#pragma unroll
        for (int u = 0; u < BS; ++u) {
          const int t = t0 + u;
          if (t < t1) {
            const T* src = (t >= S_old) ? kn + (int64_t)(t - S_old) * p.k_new.ss : kc + (int64_t)t * p.k.ss;
            x[u] = *reinterpret_cast<const uint2*>(src);
          }
        }
#pragma unroll
        for (int u = 0; u < BS; ++u) {
          const int t = t0 + u;
          if (t < t1 && t >= S_old) {
            *reinterpret_cast<uint2*>(kc + (int64_t)t * p.k.ss) = x[u];
            *reinterpret_cast<uint2*>(vc + (int64_t)t * p.v.ss) =
                *reinterpret_cast<const uint2*>(vn + (int64_t)(t - S_old) * p.v_new.ss);
          }
        }
        float acc[E];
#pragma unroll
        for (int u = 0; u < BS; ++u) {
          const int t = t0 + u;
          if (t < t1) {
            const float xf[4] = {h16lo(x[u].x, (const T*)nullptr), h16hi(x[u].x, (const T*)nullptr),
                                 h16lo(x[u].y, (const T*)nullptr), h16hi(x[u].y, (const T*)nullptr)};
#pragma unroll
            for (int e = 0; e < E; ++e) acc[e] = (t == t0) ? xf[e] : __fadd_rn(acc[e], xf[e]);
          }
        }
        const float nf = (float)(t1 - t0);
        float cen[E];
#pragma unroll
        for (int e = 0; e < E; ++e) cen[e] = __fdiv_rn(acc[e], nf);
        float* crow = p.cent + ((int64_t)(b * p.Hkv + kvh) * p.nb_cap + blk) * D + d;
        *reinterpret_cast<float4*>(crow) = make_float4(cen[0], cen[1], cen[2], cen[3]);
        float sc[G];
#pragma unroll
        for (int j = 0; j < G; ++j) {
          float part = 0.f;
#pragma unroll
          for (int e = 0; e < E; ++e) part = fmaf(qv[j][e], cen[e], part);
#pragma unroll
          for (int o = 16; o; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
          sc[j] = part;
        }
#pragma unroll
        for (int j = 0; j < G; ++j)
          if (lane == j) p.scores[(size_t)(b * p.Hq + kvh * G + j) * p.fs_stride + blk] = sc[j];
      }
    }
  }
  {
    const int sub = lane % LPR, rin = lane / LPR;
    float qf[G][DL];
    int qrun = -1;
    // Score statistics of head (sub >> 1) over this lane's rows of the current
    // piece (this CTA's rows of one (sequence, KV head)); each warp's record
    // per head, p.piece[((group + cta) * kSW + warp) * G + h], lets the
    // selection phase skip a statistics pass over the row.  (group + cta)
    // numbers the pieces in row order: both indices are non-decreasing along
    // the rows and one of them steps at every piece boundary.
    SoftPart ps = soft_empty();
    const float Tf = (float)(p.cfg.temperature > 1e-6 ? p.cfg.temperature : 1e-6);
    const bool unit_t = (Tf == 1.0f);
    for (int i = 0; i < nstage; ++i) {
      const int slot = i % kStepStages;
      const uint32_t par = (uint32_t)(i / kStepStages) & 1u;
      // a lane that gives up makes the whole warp give up: the reduce-scatter
      // below needs every lane
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&full_bar[slot], par))) {
        if (lane == 0) report(p.status, ADAKV_ST_WAIT_TIMEOUT);
        break;
      }
      if (warp == 0 && lane == 0) {
        if (i == 0) STEP_STAMP(8);
        if (i == nstage - 1) STEP_STAMP(9);
      }
      const int4 d = sdesc[i];
      const int b = d.x / p.Hkv, kvh = d.x - b * p.Hkv;
      const float* tile = ring + slot * STAGE_F;
      if (d.x != qrun) {  // queries of a new (sequence, KV head) run, from the stage
        qrun = d.x;
        const T* qs = reinterpret_cast<const T*>(tile + kStepRows * D);
#pragma unroll
        for (int h = 0; h < G; ++h)
#pragma unroll
          for (int k = 0; k < CH; ++k) {
            float f[4];
            load4<T>(qs + h * D + 4 * (sub + LPR * k), f);
#pragma unroll
            for (int e = 0; e < 4; ++e) qf[h][4 * k + e] = f[e];
          }
      }
      float* srow0 = p.scores + (size_t)(b * p.Hq + kvh * G) * p.fs_stride + d.y;
      const int nbs = ceil_div(s_S[b], BS);
      const int f_lo = imin(p.cfg.n_sink, nbs), f_hi = nbs - imin(p.cfg.n_local, nbs);
#pragma unroll
      for (int pp = 0; pp < PASSES; ++pp) {
        const int row = warp * RPW + pp * RPP + rin;
        float acc[G];
#pragma unroll
        for (int h = 0; h < G; ++h) acc[h] = 0.f;
        if (row < d.z) {
          const float* rp = tile + row * D;
#pragma unroll
          for (int k = 0; k < CH; ++k) {
            const float4 c = *reinterpret_cast<const float4*>(rp + 4 * (sub + LPR * k));
#pragma unroll
            for (int h = 0; h < G; ++h) {
              acc[h] = fmaf(qf[h][4 * k + 0], c.x, acc[h]);
              acc[h] = fmaf(qf[h][4 * k + 1], c.y, acc[h]);
              acc[h] = fmaf(qf[h][4 * k + 2], c.z, acc[h]);
              acc[h] = fmaf(qf[h][4 * k + 3], c.w, acc[h]);
            }
          }
        }
        const float s = reduce_heads<G, LPR>(acc, lane);
        if (row < d.z && row < d.w) {
          if ((sub & 1) == 0) srow0[(size_t)(sub >> 1) * p.fs_stride + row] = s;
          const int j = d.y + row;
          soft_add(ps, s, unit_t ? s : __fdiv_rn(s, Tf), j >= f_lo && j < f_hi);
        }
      }
      __syncwarp();
      if (lane == 0) {
        const int old = atomicAdd(&rel_cnt[slot], 1);
        if (old == kSW - 1) {  // last warp out refills the stage
          rel_cnt[slot] = 0;
          if (i + kStepStages < nstage) issue(i + kStepStages, slot);
        }
      }
      // a piece ends with this stage: fold the lanes of each head and store
      // the warp's record
      if (i + 1 == nstage || sdesc[i + 1].x != d.x) {
#pragma unroll 1
        for (int off = LPR; off < 32; off <<= 1) soft_merge(ps, soft_shfl_xor(ps, off));
        if (lane < LPR && (lane & 1) == 0)
          soft_store(p.piece + (((size_t)(d.x + cta) * kSW + warp) * G + (lane >> 1)) * 8, ps);
        ps = soft_empty();
      }
    }
  }
  __syncthreads();  // the ring is drained (its bytes are reused below); every score is written
  if (tid == 0) {
    fence_acq_rel_gpu();
    red_release_add_u64(p.arrive, 1ull);
    STEP_STAMP(1);
  }

  // ---------------------------------------------------------------- phase B
  // One thread-block cluster of CL CTAs per query head; rank r owns blocks
  // [r Ls, (r + 1) Ls) of the row (Ls a multiple of 32: whole bitmap words).
  const int CL = p.csize;
  const bool head_cta = cta < p.B * p.Hq * CL;
  if (head_cta) {
    cg::cluster_group cl = cg::this_cluster();
    const int hr = cta / CL, rank = cta - hr * CL;
    const int b = hr / p.Hq, h = hr - b * p.Hq;
    const int nb = ceil_div(s_S[b], BS);
    const int Ls = (ceil_div(nb, CL) + 31) / 32 * 32;
    const int lo = imin(nb, rank * Ls), hi = imin(nb, lo + Ls), n = hi - lo;
    const int nwl = ceil_div(n, 32), w_lo = lo / 32;
    const StepSmem L = step_smem_layout(D, G, p.nb_max, p.nbt, p.slice_cap, CL);
    float* srow = reinterpret_cast<float*>(sm + L.srow);        // the slice (li = j - lo)
    uint16_t* sbk = reinterpret_cast<uint16_t*>(sm + L.sbk);    // bucket of each slice block
    uint32_t* sbits = reinterpret_cast<uint32_t*>(sm + L.sbits);
    uint32_t* hist = reinterpret_cast<uint32_t*>(sm + L.hist);  // this rank's histogram
    uint32_t* ghist = reinterpret_cast<uint32_t*>(sm + L.ghist);  // the cluster's
    uint32_t* ckey = reinterpret_cast<uint32_t*>(sm + L.ckey);    // this rank's candidates
    int* cidx = reinterpret_cast<int*>(sm + L.cidx);
    uint32_t* akey = reinterpret_cast<uint32_t*>(sm + L.akey);    // every rank's candidates
    int* aidx = reinterpret_cast<int*>(sm + L.aidx);
    const SelectCfg& cf = p.cfg;
    const int sink = imin(cf.n_sink, nb), local = imin(cf.n_local, nb);
    auto forced = [&](int j) -> bool { return j < sink || j >= nb - local; };
    const bool adaptive = nb >= 2 && cf.policy == ADAKV_POLICY_ADAPTIVE;
    const float Tf = (float)(cf.temperature > 1e-6 ? cf.temperature : 1e-6);
    const bool unit_t = (Tf == 1.0f);
    auto zof = [&](float v) -> float { return unit_t ? v : __fdiv_rn(v, Tf); };

    for (int t = tid; t < kBk; t += kStepThreads) hist[t] = 0u;
    if (tid == 0) {
      s_ncand = 0;
      s_jstar = -1;
    }

    // ---- every CTA's scores are out (this call's GRID arrivals), then the
    //      slice in one batch of L2 loads ----
    if (tid == 0) {
      const unsigned long long target = (unsigned long long)tag * (unsigned long long)GRID;
      if (ld_acquire_u64(p.arrive) < target) {
        const uint64_t t0 = globaltimer_ns();
        while (ld_acquire_u64(p.arrive) < target) {
          if (globaltimer_ns() - t0 > p.wait_ns) {
            report(p.status, ADAKV_ST_WAIT_TIMEOUT);
            break;
          }
        }
      }
    }
    __syncthreads();
    if (tid == 0) STEP_STAMP(10);
    const float* grow = p.scores + (size_t)hr * p.fs_stride;  // 16-byte aligned rows
    // ---- the slice, and the row's statistics (the same arithmetic in every
    //      CTA of the cluster): each thread folds its share of the
    //      estimator's warp records of this head and of the blocks the append
    //      refresh scored, then one block-wide reduction ----
    {
      const int kvh = h / G, hh = h - kvh * G, gi = b * p.Hkv + kvh;
      const int R = s_rb[p.B], R0 = s_rb[b] + kvh * nb;
      const int skip = appending ? (s_S[b] - p.n_new) / BS : nb;  // rows the estimator scored
      int c_lo = 0, nrec = 0;
      if (skip > 0) {
        c_lo = cta_of_row(R0, R, GRID);
        nrec = (cta_of_row(R0 + nb - 1, R, GRID) - c_lo + 1) * kSW;
      }
      const bool all_rows = R >= GRID;  // every CTA scored rows
      auto record = [&](int r) -> SoftPart {
        const int c = c_lo + r / kSW;
        const bool has = all_rows || first_row_of(c, R, GRID) < first_row_of(c + 1, R, GRID);
        return has ? soft_load_cg(p.piece + (((size_t)(gi + c) * kSW + r % kSW) * G + hh) * 8)
                   : soft_empty();
      };
      // the first two records of this thread stay in flight over the slice copy
      SoftPart acc = tid < nrec ? record(tid) : soft_empty();
      const SoftPart t1 = tid + kStepThreads < nrec ? record(tid + kStepThreads) : soft_empty();
      constexpr int ST = 4 * kStepThreads;
      for (int j0 = 4 * tid; j0 < n; j0 += 4 * ST) {
        float4 x[4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (j0 + u * ST < n) x[u] = __ldcg(reinterpret_cast<const float4*>(grow + lo + j0 + u * ST));
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (j0 + u * ST < n) *reinterpret_cast<float4*>(srow + j0 + u * ST) = x[u];
      }
      soft_merge(acc, t1);
      for (int r = tid + 2 * kStepThreads; r < nrec; r += kStepThreads) soft_merge(acc, record(r));
      for (int j = skip + tid; j < nb; j += kStepThreads) {
        const float v = __ldcg(grow + j);
        soft_add(acc, v, zof(v), !forced(j));
      }
      // threads rescaled to their warp max, double sums over fixed xor trees,
      // then the kSW warp results folded the same way by every warp
      float M = warp_max(acc.m);
      float mx = warp_max(acc.mx), cmx = warp_max(acc.cmx);
      double z = 0.0, a = 0.0;
      if (acc.m > -INFINITY) {
        const double f = (double)expf(acc.m - M);
        z = (double)acc.Z * f;
        a = f * ((double)acc.A + (double)acc.Z * ((double)acc.m - (double)M));
      }
      z = warp_sum(z);
      a = warp_sum(a);
      double cs = warp_sum((double)acc.cs), cq = warp_sum((double)acc.cq);
      if (lane == 0) {
        redm[warp][0] = M;
        redm[warp][1] = mx;
        redm[warp][2] = cmx;
        redd[warp][0] = z;
        redd[warp][1] = a;
        redd[warp][2] = cs;
        redd[warp][3] = cq;
      }
      __syncthreads();
      const bool wl = lane < kSW;
      const float wm = wl ? redm[lane][0] : -INFINITY;
      M = warp_max(wm);
      mx = warp_max(wl ? redm[lane][1] : -INFINITY);
      cmx = warp_max(wl ? redm[lane][2] : -INFINITY);
      z = 0.0;
      a = 0.0;
      if (wl && wm > -INFINITY) {
        const double f = (double)expf(wm - M);
        z = redd[lane][0] * f;
        a = f * (redd[lane][1] + redd[lane][0] * ((double)wm - (double)M));
      }
      z = warp_sum(z);
      a = warp_sum(a);
      cs = warp_sum(wl ? redd[lane][2] : 0.0);
      cq = warp_sum(wl ? redd[lane][3] : 0.0);
      if (tid == 0) {
        s_row = RowStats{mx, cmx, M, cs, cq, z, a};
        STEP_STAMP(19);
      }
    }
    __syncthreads();
    if (tid == 0) STEP_STAMP(2);
    const int nch = ceil_div(n, 4);
    const float4* srow4 = reinterpret_cast<const float4*>(srow);
    const float cmx = s_row.cmx, M = s_row.m;
    const double csum = s_row.cs, csq = s_row.cq, Z = s_row.Z, A = s_row.A;
    const double nc_d = (double)(nb - imin(nb, sink + local));
    const double mean_c = nc_d > 0 ? csum / nc_d : 0.0;
    const double var_c = nc_d > 0 ? csq / nc_d - mean_c * mean_c : 0.0;
    const double sd_c = var_c > 0.0 ? sqrt(var_c) : 0.0;
    const double range = (double)cmx - (mean_c - sd_c);
    const bool buckets_ok = isfinite(cmx) && range > 0.0 && isfinite(range);
    const float scale = buckets_ok ? (float)((double)(kBk - 1) / range) : 0.f;
    const float zmax = M;  // = max over the row of s / T

    // ---- pass 2: clamp correction, content histogram, each block's bucket
    //      (8 blocks per thread and iteration) ----
    {
      float cpa = 0.f, cpb = 0.f;
      const float Zf = (float)Z;
      const float logZ = adaptive ? (float)log(Z) : 0.f;
      const float cst = logf(1e-9f) + logZ;
      const float d_hi = adaptive ? logf(2e-9f * Zf) : -INFINITY, d_lo = d_hi - 25.f;
      // a block is clamped when p = e / Z (float, rounded) < 1e-9; decided
      // from the fast product e' * (1 / Z), e' = __expf (relative error
      // < 5e-6 on this window), unless it lies within 1e-5 of the bound, where
      // the rounded quotient of expf is taken
      const float invZ = 1.f / Zf;
      const float clamp_lo = 1e-9f * (1.f - 1e-5f), clamp_hi = 1e-9f * (1.f + 1e-5f);
      // near the bound: e / Z rounded to float is below 1e-9f exactly when
      // e <= mid * Z, mid = the midpoint between 1e-9f and the float below it
      // (1e-9f has an odd significand, so a tie rounds down; the product is
      // exact in double)
      const double clamp_mz = 0.5 * ((double)nextafterf(1e-9f, 0.f) + (double)1e-9f) * (double)Zf;
#pragma unroll 1
      for (int c = tid; c < nch; c += 2 * kStepThreads) {
        const int c2 = c + kStepThreads;
        const float4 x = srow4[c];
        const float4 y = c2 < nch ? srow4[c2] : make_float4(0.f, 0.f, 0.f, 0.f);
        const float v[8] = {x.x, x.y, x.z, x.w, y.x, y.y, y.z, y.w};
        // branch-free per block; the rare near-bound clamp decisions after
        uint32_t bk8[8];
        bool band[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int li = 4 * (e < 4 ? c : c2) + (e & 3), j = lo + li;
          const bool in = li < n;
          const bool content = in && buckets_ok && !forced(j);
          const int bk = content ? bucket_of(v[e], cmx, scale) : kBk - 1;
          atomicAdd(&hist[bk], bk < kBk - 1 ? 1u : 0u);
          bk8[e] = (uint32_t)bk;
          const float dd = __fsub_rn(zof(v[e]), zmax);
          const bool win = adaptive && in && dd < d_hi && dd >= d_lo;
          const float ex = __expf(dd);
          const float pr = ex * invZ;
          band[e] = win && pr >= clamp_lo && pr <= clamp_hi;
          const float t = (win && ex > 0.f && pr < clamp_lo) ? ex * (cst - dd) : 0.f;
          if (e & 1) cpb += t; else cpa += t;
        }
        bool any_band = false;
#pragma unroll
        for (int e = 0; e < 8; ++e) any_band |= band[e];
        if (any_band) {
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            if (band[e]) {
              const float dd = __fsub_rn(zof(v[e]), zmax);
              const float ea = expf(dd);
              if (ea > 0.f && (double)ea <= clamp_mz) cpa += __expf(dd) * (cst - dd);
            }
          }
        }
        reinterpret_cast<uint2*>(sbk)[c] = make_uint2(bk8[0] | (bk8[1] << 16), bk8[2] | (bk8[3] << 16));
        if (c2 < nch)
          reinterpret_cast<uint2*>(sbk)[c2] = make_uint2(bk8[4] | (bk8[5] << 16), bk8[6] | (bk8[7] << 16));
      }
      const float cp = cpa + cpb;
      double c2 = cp, dummy = 0.0;
      block_sum2d(c2, dummy, redd);
      if (tid == 0) {
        s_part.Cc = c2;
        STEP_STAMP(16);
      }
    }
    cl.sync();  // (2) every rank's histogram and clamp correction
    if (tid == 0) STEP_STAMP(17);
    // the cluster's histogram (thread t: buckets [8t, 8t + 8)) and the entropy
    {
      static_assert(kBk == 8 * kStepThreads, "8 buckets per thread");
      uint4 s0 = make_uint4(0u, 0u, 0u, 0u), s1 = s0;
      for (int r = 0; r < CL; ++r) {
        const uint4* rh = reinterpret_cast<const uint4*>(cl.map_shared_rank(hist, r));
        const uint4 x0 = rh[2 * tid], x1 = rh[2 * tid + 1];
        s0.x += x0.x; s0.y += x0.y; s0.z += x0.z; s0.w += x0.w;
        s1.x += x1.x; s1.y += x1.y; s1.z += x1.z; s1.w += x1.w;
      }
      reinterpret_cast<uint4*>(ghist)[2 * tid] = s0;
      reinterpret_cast<uint4*>(ghist)[2 * tid + 1] = s1;
      if (adaptive && tid == 0) {
        double Cc = 0.0;
        for (int r = 0; r < CL; ++r) Cc += cl.map_shared_rank(&s_part, r)->Cc;
        // entropy, adakv/budget.py:36-37 with the max(p, 1e-9) clamp
        const double H = log(Z) - A / Z - Cc / Z;
        if (rank == 0 && !((p.debug_flags & kDebugSkipPublish) && hr == 0))
          str_u64(p.hslot + hr, tword(tag, __float_as_uint((float)H)));
        STEP_STAMP(11);
      }
    }

    // ---- the sequence's entropies -> this head's weight and the weight sum ----
    if (warp == 0 && adaptive) {
      PollBudget pb{p.wait_ns, 0, false};
      const double lognb = log((double)imax(nb, 2));
      constexpr int NQ = kStepMaxHeads / 32;
      const unsigned long long* base = p.hslot + b * p.Hq + lane;
      const int nq = lane < p.Hq ? ceil_div(p.Hq - lane, 32) : 0;
      unsigned long long w[NQ];
#pragma unroll
      for (int q4 = 0; q4 < NQ; ++q4) w[q4] = q4 < nq ? ldr_u64(base + q4 * 32) : 0ull;
      wait_tagged_n<NQ>(base, 32, w, nq, tag, pb);
      double ps = 0.0, mine = 0.0;
#pragma unroll
      for (int q4 = 0; q4 < NQ; ++q4) {
        const int hh = lane + q4 * 32;
        if (q4 < nq) {
          // entropy weight, adakv/budget.py:36-37: float32 entropy / log(nb) in float64
          const double wv = (double)__uint_as_float((uint32_t)w[q4]) / lognb + 1e-6;
          ps += wv;
          if (hh == h) mine = wv;
        }
      }
      if (__any_sync(0xffffffffu, pb.dead) && lane == 0) report(p.status, ADAKV_ST_WAIT_TIMEOUT);
      ps = warp_sum(ps);  // fixed xor tree: every CTA of the sequence gets the same sum
      mine = warp_sum(mine);
      if (lane == 0) {
        s_sumw = ps;
        s_w = mine;
      }
    }
    __syncthreads();
    if (tid == 0) STEP_STAMP(3);

    // ---- this head's count (budget.py:71-86, selector.py:49-54) ----
    const SeqBudget sbud = seq_budget(nb, cf);
    const double w_h = adaptive ? s_w : 0.0, sum_w = adaptive ? s_sumw : 0.0;
    const int K = imin(head_count(sbud, cf, w_h, sum_w, p.Hq), p.table_width);
    const int n_forced = (sink + local >= nb) ? nb : sink + local;
    const int Kc = K - n_forced;
    const bool all = K >= nb;

    // ---- threshold bucket: the one holding the Kc-th content block ----
    int js = -1, need = 0;
    if (!all && Kc > 0 && buckets_ok) {
      const uint4 h0 = reinterpret_cast<const uint4*>(ghist)[2 * tid];
      const uint4 h1 = reinterpret_cast<const uint4*>(ghist)[2 * tid + 1];
      const uint32_t c8[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
      uint32_t tot = 0;
#pragma unroll
      for (int e = 0; e < 8; ++e) tot += c8[e];
      uint32_t acc = (uint32_t)block_exclusive_scan((int)tot, scan_scratch);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        if (acc < (uint32_t)Kc && (uint32_t)Kc <= acc + c8[e]) {
          s_jstar = 8 * tid + e;
          s_digit = Kc - (int)acc;  // members of the threshold bucket to take
        }
        acc += c8[e];
      }
      __syncthreads();
      js = s_jstar;
      need = s_digit;
    }
    if (tid == 0) STEP_STAMP(20);
    // the exact fallback: no usable bucket range, or a crowded threshold bucket
    const bool exact = !all && Kc > 0 && (js < 0 || js >= kBk - 1 || (int)ghist[js] > kStepCandCap);

    if (!exact) {
      // ---- this rank's slice, 8 blocks (one uint4 of buckets) per thread and
      //      four threads per bitmap word: forced blocks, buckets above the
      //      threshold, candidates of the threshold bucket ----
      const int nq = 4 * nwl;
      for (int g0 = 0; g0 < nq; g0 += kStepThreads) {
        const int g = g0 + tid;
        uint32_t sb = 0u;
        if (g < nq) {
          const uint4 u = reinterpret_cast<const uint4*>(sbk)[g];
          const uint32_t pr[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int li = 8 * g + e, j = lo + li;
            const int bk = (int)((e & 1) ? pr[e >> 1] >> 16 : pr[e >> 1] & 0xFFFFu);
            const bool in = li < n;
            const bool sel = in && (all || forced(j) || (Kc > 0 && bk < js));
            const bool cand = in && !all && Kc > 0 && bk == js && !forced(j);
            sb |= (uint32_t)sel << (8 * (g & 3) + e);
            if (cand) {
              const int slot = atomicAdd(&s_ncand, 1);
              ckey[slot] = order_key(srow[li]);
              cidx[slot] = j;
            }
          }
        }
        sb |= __shfl_xor_sync(0xffffffffu, sb, 1);
        sb |= __shfl_xor_sync(0xffffffffu, sb, 2);
        if (g < nq && (g & 3) == 0) sbits[g >> 2] = sb;
      }
      __syncthreads();
      if (tid == 0) {
        s_part.ncand = s_ncand;
        STEP_STAMP(21);
      }
    }
    cl.sync();  // (3) every rank's candidates
    if (tid == 0) STEP_STAMP(12);
    if (exact) {
      // rank 0 ranks the whole row exactly (radix select); the other ranks publish nothing
      if (rank == 0) {
        const int nw = ceil_div(nb, 32);
        for (int j = 4 * tid; j < nb; j += 4 * kStepThreads)
          *reinterpret_cast<float4*>(srow + j) = __ldcg(reinterpret_cast<const float4*>(grow + j));
        for (int w = tid; w < nw; w += kStepThreads) sbits[w] = 0u;
        __syncthreads();
        radix_select_top(srow, nb, sink, local, K, hist, ghist, sbits, scan_scratch, &s_digit, &s_above);
        __syncthreads();
      }
    } else if (!all && Kc > 0) {
      // every rank's candidates, in rank order; each rank decides its own
      // by exact rank (score desc, index asc) among all of them
      int off = 0, tot = 0;
      for (int r = 0; r < CL; ++r) {
        const int nc = cl.map_shared_rank(&s_part, r)->ncand;
        if (r < rank) off += nc;
        tot += nc;
      }
      int base = 0;
      for (int r = 0; r < CL; ++r) {
        const int nc = cl.map_shared_rank(&s_part, r)->ncand;
        const uint32_t* rk = cl.map_shared_rank(ckey, r);
        const int* ri = cl.map_shared_rank(cidx, r);
        for (int u = tid; u < nc; u += kStepThreads) {
          akey[base + u] = rk[u];
          aidx[base + u] = ri[u];
        }
        base += nc;
      }
      __syncthreads();
      const int mine = s_ncand;
      for (int u = tid; u < mine; u += kStepThreads) {
        const uint32_t ku = akey[off + u];
        const int iu = aidx[off + u];
        int rk = 0;
        for (int c2 = 0; c2 < tot; ++c2) {
          const uint32_t kc = akey[c2];
          rk += (kc > ku) || (kc == ku && aidx[c2] < iu);
        }
        if (rk < need) atomicOr(&sbits[(iu - lo) >> 5], 1u << ((iu - lo) & 31));
      }
      __syncthreads();
    }
    if (tid == 0) STEP_STAMP(14);

    // ---- publish this rank's bitmap words and its ascending table segment ----
    const bool writes = !exact || rank == 0;
    const int wb = exact ? 0 : w_lo, wn = exact ? ceil_div(nb, 32) : nwl;
    {
      uint32_t* brow = p.bitmap + (size_t)hr * p.fb_stride + wb;
      for (int w = tid; w < wn && writes; w += kStepThreads) brow[w] = sbits[w];
      const int wpt = ceil_div(wn, kStepThreads);
      const int w0 = imin(tid * wpt, wn), w1 = imin(w0 + wpt, wn);
      int cnt = 0;
      for (int w = w0; w < w1 && writes; ++w) cnt += __popc(sbits[w]);
      int pos = block_exclusive_scan(cnt, scan_scratch);
      if (tid == 0) s_part.nsel = writes ? scan_scratch[32] : 0;
      cl.sync();  // (4) every rank's count; after this no rank reads another's shared memory
      if (tid == 0) STEP_STAMP(18);
      int before = 0, total = 0;
      for (int r = 0; r < CL; ++r) {
        const int ns = cl.map_shared_rank(&s_part, r)->nsel;
        if (r < rank) before += ns;
        total += ns;
      }
      pos += before;
      int* trow = p.block_table + (int64_t)hr * p.table_width;
      for (int w = w0; w < w1 && writes; ++w) {
        uint32_t sw = sbits[w];
        while (sw) {
          const int bit = __ffs(sw) - 1;
          sw &= sw - 1u;
          if (pos < p.table_width) trow[pos] = (wb + w) * 32 + bit;
          ++pos;
        }
      }
      if (rank == 0 && tid == 0) p.sel_lens[hr] = total;
    }
    __syncthreads();
    if (tid == 0) {
      fence_acq_rel_gpu();  // release: the bitmap words, and the appended tokens acquired above
      str_u64(p.ready + (size_t)hr * CL + rank, tword(tag, 1u));
      STEP_STAMP(4);
    }
    // (the ranks still read each other's s_part after barrier 4: keep every
    // CTA of the cluster resident until they are done; see the end of the kernel)
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  }

  // ---------------------------------------------------------------- phase C
  pdl_launch_dependents();
  {
    const int NG = p.B * p.Hkv;
    const int gi = cta_of_row(cta, GRID, NG);  // CTAs split over the NG groups like rows over CTAs
    const int c_first = muldiv(gi, GRID, NG), c_next = muldiv(gi + 1, GRID, NG);
    const int split = cta - c_first, SPLIT = c_next - c_first;
    const int b = gi / p.Hkv, kvh = gi - b * p.Hkv;
    const int S = s_S[b];
    const int nb = ceil_div(S, BS);
    const int nw = ceil_div(nb, 32);
    const int row0 = b * p.Hq + kvh * G;
    const StepSmem L = step_smem_layout(D, G, p.nb_max, p.nbt, p.slice_cap, CL);
    T* kvbuf = reinterpret_cast<T*>(sm + L.kv);
    uint32_t* uw = reinterpret_cast<uint32_t*>(sm + L.uw);
    uint32_t* hw = reinterpret_cast<uint32_t*>(sm + L.hw);
    int* list = reinterpret_cast<int*>(sm + L.list);
    uint32_t* lmask = reinterpret_cast<uint32_t*>(sm + L.mask);
    float* wpart = reinterpret_cast<float*>(sm + L.wpart);
    const T* kbase = static_cast<const T*>(p.k.data) + b * p.k.sb + kvh * p.k.sh;
    const T* vbase = static_cast<const T*>(p.v.data) + b * p.v.sb + kvh * p.v.sh;
    const T* qbase = static_cast<const T*>(p.q.data) + b * p.q.sb + (int64_t)kvh * G * p.q.sh;
    const int gid = lane >> 2, tig = lane & 3;
    MmaAcc<D> acc;
    uint32_t qa[D / 16][4];
#pragma unroll
    for (int nn = 0; nn < MmaAcc<D>::NT; ++nn)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc.o[nn][e] = 0.f;
    acc.m[0] = acc.m[1] = -INFINITY;
    acc.l[0] = acc.l[1] = 0.f;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = gid + (e & 1) * 8;
        const int col = ks * 16 + (e >> 1) * 8 + tig * 2;
        qa[ks][e] = r < G ? *reinterpret_cast<const uint32_t*>(qbase + (int64_t)r * p.q.sh + col) : 0u;
      }
    }
    const float scale_log2 = p.sm_scale * 1.4426950408889634f;

    // ---- the group's G bitmaps: warp 0 waits for the G x CL ready words ----
    if (warp == 0) {
      PollBudget pb{p.wait_ns, 0, false};
      const int nr = G * CL;  // <= 32
      unsigned long long x[1] = {lane < nr ? ldr_u64(p.ready + (size_t)row0 * CL + lane) : 0ull};
      wait_tagged_n<1>(p.ready + (size_t)row0 * CL + lane, 1, x, lane < nr ? 1 : 0, tag, pb);
      if (__any_sync(0xffffffffu, pb.dead) && lane == 0) report(p.status, ADAKV_ST_WAIT_TIMEOUT);
      fence_acq_rel_gpu();  // acquire: the bitmaps and the appended K/V tokens
    }
    __syncthreads();
    if (tid == 0) STEP_STAMP(5);
    const int wpt = ceil_div(nw, kStepThreads);
    const int w0 = imin(tid * wpt, nw), w1 = imin(w0 + wpt, nw);
    int cnt = 0;
    for (int w = w0; w < w1; ++w) {
      uint32_t u = 0;
#pragma unroll
      for (int hh = 0; hh < G; ++hh) {
        const uint32_t v = __ldcg(p.bitmap + (size_t)(row0 + hh) * p.fb_stride + w);
        hw[hh * nw + w] = v;
        u |= v;
      }
      uw[w] = u;
      cnt += __popc(u);
    }
    const int before = block_exclusive_scan(cnt, scan_scratch);
    const int U = scan_scratch[32];
    const int lo = muldiv(U, split, SPLIT), hi = muldiv(U, split + 1, SPLIT);
    if (before < hi && before + cnt > lo) {
      int rk = before;
      for (int w = w0; w < w1 && rk < hi; ++w) {
        uint32_t u = uw[w];
        const int pc = __popc(u);
        if (rk + pc <= lo) {
          rk += pc;
          continue;
        }
        while (u && rk < hi) {
          const int bit = __ffs(u) - 1;
          u &= u - 1u;
          if (rk >= lo && rk - lo < p.slice_cap) list[rk - lo] = w * 32 + bit;
          ++rk;
        }
      }
    }
    __syncthreads();
    if (tid == 0) STEP_STAMP(22);
    const int n = imin(hi - lo, p.slice_cap);
    for (int i = tid; i < n; i += kStepThreads) {
      const int id = list[i], w = id >> 5, bit = id & 31;
      uint32_t m = 0;
#pragma unroll
      for (int hh = 0; hh < G; ++hh) m |= ((hw[hh * nw + w] >> bit) & 1u) << hh;
      lmask[i] = m;
    }
    __syncthreads();

    // ---- two-stage gather ring + tensor-core attention, NSLOT blocks per stage ----
    const int NSLOT = p.nbt;
    auto issue_kv = [&](int first, int stage) {
      const int cntb = imin(NSLOT, n - first);
      T* kb = kvbuf + (size_t)stage * 2 * NSLOT * BLK;
      T* vb = kb + (size_t)NSLOT * BLK;
      const int chunks = cntb * BS * ROWC;
      for (int c = tid; c < chunks; c += kStepThreads) {
        const int slot = c / (BS * ROWC);
        const int rem = c - slot * (BS * ROWC);
        const int tok = rem / ROWC, col = rem - tok * ROWC;
        const int pos = list[first + slot] * BS + tok;
        const bool valid = pos < S;
        const int64_t srow_ = valid ? (int64_t)pos : 0;
        const size_t off = (size_t)slot * BLK + tok * D + (col ^ (tok & 7)) * VEC;
        cp_async16(kb + off, kbase + srow_ * p.k.ss + col * VEC, valid);
        cp_async16(vb + off, vbase + srow_ * p.v.ss + col * VEC, valid);
      }
      cp_async_commit();
    };
    const int nbatch = ceil_div(n, NSLOT);
    if (nbatch > 0) issue_kv(0, 0);
    for (int bi = 0; bi < nbatch; ++bi) {
      const int first = bi * NSLOT;
      const int cntb = imin(NSLOT, n - first);
      if (bi + 1 < nbatch) {
        issue_kv(first + NSLOT, (bi + 1) & 1);
        asm volatile("cp.async.wait_group 1;" ::: "memory");
      } else {
        cp_async_wait_all();
      }
      __syncthreads();
      const T* kb = kvbuf + (size_t)(bi & 1) * 2 * NSLOT * BLK;
      const T* vb = kb + (size_t)NSLOT * BLK;
      for (int slot = warp; slot < cntb; slot += kSW) {
        const int blk = list[first + slot];
        const int tok_valid = imin(BS, S - blk * BS);
        mma_block<T, D, BS>(acc, qa, smem_addr(kb + (size_t)slot * BLK), smem_addr(vb + (size_t)slot * BLK),
                            lmask[first + slot], tok_valid, scale_log2, lane);
      }
      __syncthreads();  // this stage is refilled two batches later
    }
    if (tid == 0) STEP_STAMP(13);

    // ---- warp partials -> this CTA's partial (m in log2 units, l, o) ----
    {
      float l0 = acc.l[0], l1 = acc.l[1];
      l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
      l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
      l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
      l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
      float* mine = wpart + warp * G * (D + 2);
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int r = gid + half * 8;
        if (r < G) {
          float* rp = mine + r * (D + 2);
          if (tig == 0) {
            rp[0] = acc.m[half];
            rp[1] = half ? l1 : l0;
          }
#pragma unroll
          for (int nn = 0; nn < MmaAcc<D>::NT; ++nn) {
            rp[2 + nn * 8 + tig * 2] = acc.o[nn][half * 2];
            rp[2 + nn * 8 + tig * 2 + 1] = acc.o[nn][half * 2 + 1];
          }
        }
      }
    }
    __syncthreads();
    if (tid == 0) STEP_STAMP(23);
    float* gpart = p.part + (size_t)cta * G * (D + 2);
    for (int idx = tid; idx < G * D; idx += kStepThreads) {
      const int hh = idx / D, dd = idx - hh * D;
      float M = -INFINITY;
      for (int w = 0; w < kSW; ++w) M = fmaxf(M, wpart[(w * G + hh) * (D + 2)]);
      float Ls = 0.f, O = 0.f;
      if (M != -INFINITY) {
        for (int w = 0; w < kSW; ++w) {
          const float* rp = wpart + (w * G + hh) * (D + 2);
          const float f = (rp[0] == -INFINITY) ? 0.f : exp2f(rp[0] - M);
          Ls += rp[1] * f;
          O += rp[2 + dd] * f;
        }
      }
      gpart[hh * (D + 2) + 2 + dd] = O;
      if (dd == 0) {
        gpart[hh * (D + 2)] = M;
        gpart[hh * (D + 2) + 1] = Ls;
      }
    }
    __syncthreads();
    if (tid == 0) {
      fence_acq_rel_gpu();  // release: this CTA's partial
      str_u64(p.pready + cta, tword(tag, 1u));
      STEP_STAMP(6);
    }

    // ---- the group's SPLIT partials, merged in split order by every CTA of
    //      the group for its own share of the output columns: warp w takes
    //      head w % G and half (G = 4) or all (G = 8) of the share, its lanes
    //      the splits ----
    {
      if (warp == 0) {
        PollBudget pb{p.wait_ns, 0, false};
        constexpr int NP = kStepMaxGrid / 32;
        const unsigned long long* base = p.pready + c_first + lane;
        const int np = lane < SPLIT ? ceil_div(SPLIT - lane, 32) : 0;
        unsigned long long x[NP];
#pragma unroll
        for (int i = 0; i < NP; ++i) x[i] = i < np ? ldr_u64(base + i * 32) : 0ull;
        wait_tagged_n<NP>(base, 32, x, np, tag, pb);
        if (__any_sync(0xffffffffu, pb.dead) && lane == 0) report(p.status, ADAKV_ST_WAIT_TIMEOUT);
        fence_acq_rel_gpu();  // acquire: the partials
      }
      __syncthreads();
      const size_t stride = (size_t)G * (D + 2);
      const int d_lo = muldiv(D, split, SPLIT), d_hi = muldiv(D, split + 1, SPLIT);
      constexpr int WPH = kSW / G;  // warps per head
      static_assert(kSW % G == 0, "whole warps per head");
      const int hh = warp % G, wp = warp / G;
      const int cpw = ceil_div(d_hi - d_lo, WPH);
      const int cb = d_lo + wp * cpw, ce = imin(d_hi, cb + cpw);
      const float* ph = p.part + (size_t)c_first * stride + hh * (D + 2);
      T* orow = static_cast<T*>(const_cast<void*>(p.out.data)) + b * p.out.sb + (int64_t)(kvh * G + hh) * p.out.sh;
      for (int c0 = cb; c0 < ce; c0 += 4) {
        float Ml = -INFINITY, Ll = 0.f, Ol[4] = {0.f, 0.f, 0.f, 0.f};
        for (int s0 = lane; s0 < SPLIT; s0 += 32) {
          const float* src = ph + (size_t)s0 * stride;
          const float m = __ldcg(src), l = __ldcg(src + 1);
          float o[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) o[u] = c0 + u < ce ? __ldcg(src + 2 + c0 + u) : 0.f;
          if (m > -INFINITY) {
            const float Mn = fmaxf(Ml, m);
            const float fa = Ml == -INFINITY ? 0.f : exp2f(Ml - Mn), fb = exp2f(m - Mn);
            Ll = Ll * fa + l * fb;
#pragma unroll
            for (int u = 0; u < 4; ++u) Ol[u] = Ol[u] * fa + o[u] * fb;
            Ml = Mn;
          }
        }
        const float M = warp_max(Ml);
        const float f = Ml == -INFINITY ? 0.f : exp2f(Ml - M);
        const float Ls = warp_sum(Ll * f);
        float O[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) O[u] = warp_sum(Ol[u] * f);
        const float ol = lane == 0 ? O[0] : lane == 1 ? O[1] : lane == 2 ? O[2] : O[3];
        if (lane < 4 && c0 + lane < ce) orow[c0 + lane] = from_f32<T>(Ls > 0.f ? ol / Ls : 0.f);
        if (p.lse && split == SPLIT - 1 && wp == 0 && c0 == cb && lane == 0)
          p.lse[row0 + hh] = (Ls > 0.f && M > -INFINITY) ? M * 0.6931471805599453f + logf(Ls) : -INFINITY;
      }
    }
  }

  // peers may still read this CTA's s_part until they arrive
  if (head_cta) asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");

  // ---------------------------------------------------------------- call tag
  // The last CTA to finish advances the call counter (every CTA read it at
  // its start), so the next call's words carry a new tag.
  __syncthreads();
  if (tid == 0) {
    STEP_STAMP(7);
    unsigned prev;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(p.epoch + 1) : "memory");
    if (prev == (unsigned)(GRID - 1)) {
      p.epoch[1] = 0u;
      p.epoch[0] = tag;
    }
  }
}

// ---------------------------------------------------------------------------
// last step's block scores -> float rows (either path's layout)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) step_scores_kernel(bool fused, const float* fscores,
                                                          int fs_stride, const float* scores,
                                                          int score_stride, int nb, float* out,
                                                          int out_stride) {
  const int r = blockIdx.x;
  for (int j = threadIdx.x; j < nb; j += blockDim.x) {
    float v;
    if (fused) v = fscores[(size_t)r * fs_stride + j];
    else v = scores[(size_t)r * score_stride + j];
    out[(size_t)r * out_stride + j] = v;
  }
}

cudaError_t launch_step_scores(bool fused, const float* fscores, int fs_stride,
                               const float* scores, int score_stride, int rows, int nb, float* out,
                               int out_stride, cudaStream_t st) {
  step_scores_kernel<<<rows, 256, 0, st>>>(fused, fscores, fs_stride, scores, score_stride, nb, out,
                                           out_stride);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
template <typename F>
static cudaError_t for_each_step(int dtype, int D, int g, F&& f) {
#define ADAKV_STEP_CASE(TT, DD, GG) \
  if (D == DD && g == GG) return f(step_kernel<TT, DD, GG>);
#define ADAKV_STEP_T(TT) ADAKV_STEP_CASE(TT, 128, 4) ADAKV_STEP_CASE(TT, 128, 8)
  if (dtype == ADAKV_DTYPE_BF16) {
    ADAKV_STEP_T(__nv_bfloat16)
  } else if (dtype == ADAKV_DTYPE_F16) {
    ADAKV_STEP_T(__half)
  }
#undef ADAKV_STEP_T
#undef ADAKV_STEP_CASE
  return cudaErrorInvalidValue;
}

bool step_kernel_built(int dtype, int D, int bs, int g) {
  return (dtype == ADAKV_DTYPE_BF16 || dtype == ADAKV_DTYPE_F16) && D == 128 && bs == 16 &&
         (g == 4 || g == 8);
}

size_t step_smem_bytes(int D, int g, int nb_max, int min_split, int csize, int* nbt, int* slice_cap) {
  const int sc = ceil_div(imax(nb_max, 1), imax(min_split, 1)) + 1;
  int t = 8;
  StepSmem s = step_smem_layout(D, g, nb_max, t, sc, csize);
  while (s.total > kStepSmemMax && t > 1) {
    --t;
    s = step_smem_layout(D, g, nb_max, t, sc, csize);
  }
  if (nbt) *nbt = t;
  if (slice_cap) *slice_cap = sc;
  return s.total;
}

cudaError_t step_kernels_init() {
  for (int dt : {ADAKV_DTYPE_F16, ADAKV_DTYPE_BF16})
    for (int g : {4, 8}) {
      cudaError_t e = for_each_step(dt, 128, g, [](auto kern) {
        return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kStepSmemMax);
      });
      if (e != cudaSuccess) return e;
    }
  return cudaSuccess;
}

cudaError_t launch_step(const StepParams& p, int dtype, int D, int g, int grid, size_t smem,
                        cudaStream_t st, const LaunchOpts& o) {
  LaunchOpts oc = o;
  oc.cluster_x = (unsigned)p.csize;
  return for_each_step(dtype, D, g, [&](auto kern) {
    return launch_ex(kern, dim3(grid), dim3(kStepThreads), smem, st, oc, p);
  });
}

int step_active_clusters(int dtype, int D, int g, int csize, size_t smem) {
  int n = 0;
  const cudaError_t e = for_each_step(dtype, D, g, [&](auto kern) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(csize, 1, 1);
    cfg.blockDim = dim3(kStepThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = csize;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
  });
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return 0;
  }
  return n;
}

}  // namespace adakv
