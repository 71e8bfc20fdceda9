// (b) Centroid block estimator, with (a) the step's KV append fused in.
//
// scores[b, h, j] = q[b, h] . centroid[b, h / g, j] (unscaled, float32): the
// reference's einsum("hd,hbd->hb") over GQA-expanded centroids
// (adakv/estimator.py:73-74, adakv/attention.py:187-189) with the expansion
// folded away -- every centroid row is read from HBM once and scored against
// all g query heads of its KV head.
//
// Persistent grid, one CTA per SM.  The work is the list of 64-row chunks of
// every (sequence, KV head) centroid table; each CTA owns a contiguous range of
// it.  A producer warp streams chunks through a 4-stage shared-memory ring with
// 1-D bulk copies (the TMA engine, one CTA per copy), each stage also carrying the g
// query rows of the chunk's KV head; completion is signalled on per-stage
// mbarriers (transaction bytes) and stages are released by the 8 consumer warps
// through a second set of mbarriers.  A consumer lane owns D/32 dims of a row
// and keeps the matching query slices in registers; 32 (row, head) partial dot
// products are finished with one 31-shuffle butterfly reduce-scatter.
//
// Fused append (adakv/runtime.py:43-60): when the step appends n_new tokens, a
// tenth warp writes them into the K/V cache in place, recomputes every touched
// block's centroid from its tokens (token-order float32 sum, one IEEE division:
// bit-identical to a rebuild), stores it, and scores it against the group's
// queries.  Consumers skip those rows, so there is no ordering hazard between
// the refresh and the bulk copies of the same chunk.
//
// Bytes from HBM per step: the float32 centroid table (B * Hkv * nb * D * 4) plus
// q; the block scores (B * Hq * nb * 4) are written once and stay in L2.
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

// E consecutive elements of T -> fp32 (E * sizeof(T) is 4, 8 or 16 bytes).
// Pure register arithmetic: taking the address of a local word would push it
// to local memory and serialise the surrounding loads.
__device__ __forceinline__ float lo16_f32(uint32_t w, __nv_bfloat16*) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float hi16_f32(uint32_t w, __nv_bfloat16*) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ float lo16_f32(uint32_t w, __half*) {
  return __half2float(__ushort_as_half((unsigned short)(w & 0xFFFFu)));
}
__device__ __forceinline__ float hi16_f32(uint32_t w, __half*) {
  return __half2float(__ushort_as_half((unsigned short)(w >> 16)));
}

template <typename T, int E>
__device__ __forceinline__ void load_vec(const T* p, float (&out)[E]) {
  if constexpr (sizeof(T) == 4 && E == 4) {
    const float4 v = *reinterpret_cast<const float4*>(p);
    out[0] = v.x; out[1] = v.y; out[2] = v.z; out[3] = v.w;
  } else if constexpr (sizeof(T) == 4 && E == 2) {
    const float2 v = *reinterpret_cast<const float2*>(p);
    out[0] = v.x; out[1] = v.y;
  } else if constexpr (sizeof(T) == 2 && E == 4) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    out[0] = lo16_f32(u.x, (T*)nullptr); out[1] = hi16_f32(u.x, (T*)nullptr);
    out[2] = lo16_f32(u.y, (T*)nullptr); out[3] = hi16_f32(u.y, (T*)nullptr);
  } else if constexpr (sizeof(T) == 2 && E == 2) {
    const uint32_t u = *reinterpret_cast<const uint32_t*>(p);
    out[0] = lo16_f32(u, (T*)nullptr); out[1] = hi16_f32(u, (T*)nullptr);
  } else {
#pragma unroll
    for (int e = 0; e < E; ++e) out[e] = to_f32(p[e]);
  }
}

template <typename T, int E>
__device__ __forceinline__ void copy_vec(T* dst, const T* src) {
  constexpr int BYTES = E * (int)sizeof(T);
  if constexpr (BYTES == 16) {
    *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
  } else if constexpr (BYTES == 8) {
    *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(src);
  } else if constexpr (BYTES == 4) {
    *reinterpret_cast<uint32_t*>(dst) = *reinterpret_cast<const uint32_t*>(src);
  } else {
#pragma unroll
    for (int e = 0; e < E; ++e) dst[e] = src[e];
  }
}

// E elements of T as one raw register word (8 or 16 bytes) and its fp32 unpack
template <typename T, int E> struct RawVec;
template <> struct RawVec<float, 4> {
  using type = float4;
  __device__ __forceinline__ static void unpack(const float4& v, float (&o)[4]) {
    o[0] = v.x; o[1] = v.y; o[2] = v.z; o[3] = v.w;
  }
};
template <> struct RawVec<float, 2> {
  using type = float2;
  __device__ __forceinline__ static void unpack(const float2& v, float (&o)[2]) { o[0] = v.x; o[1] = v.y; }
};
template <typename H> struct RawVec16x4 {
  using type = uint2;
  __device__ __forceinline__ static void unpack(const uint2& u, float (&o)[4]) {
    o[0] = lo16_f32(u.x, (H*)nullptr); o[1] = hi16_f32(u.x, (H*)nullptr);
    o[2] = lo16_f32(u.y, (H*)nullptr); o[3] = hi16_f32(u.y, (H*)nullptr);
  }
};
template <typename H> struct RawVec16x2 {
  using type = uint32_t;
  __device__ __forceinline__ static void unpack(const uint32_t& u, float (&o)[2]) {
    o[0] = lo16_f32(u, (H*)nullptr); o[1] = hi16_f32(u, (H*)nullptr);
  }
};
template <> struct RawVec<__nv_bfloat16, 4> : RawVec16x4<__nv_bfloat16> {};
template <> struct RawVec<__half, 4> : RawVec16x4<__half> {};
template <> struct RawVec<__nv_bfloat16, 2> : RawVec16x2<__nv_bfloat16> {};
template <> struct RawVec<__half, 2> : RawVec16x2<__half> {};

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

template <typename T, int D, int GP>
__global__ void __launch_bounds__(kEstThreads, 1) estimate_kernel(EstParams p) {
  constexpr int E = D / 32;                             // floats per lane per row
  constexpr int R = 32 / GP;                            // rows per reduce-scatter group
  constexpr int RPW = kEstRows / kEstConsumerWarps;     // rows per consumer warp (8)
  constexpr int NG = RPW / R;                           // groups per warp
  constexpr int TILE_F = kEstRows * D;                  // floats of centroid rows per stage
  static_assert(RPW % R == 0, "rows per warp must be a multiple of the group rows");
  extern __shared__ __align__(128) float ring[];       // [stages][stage_f], then 2x[B+1] ints
  __shared__ __align__(8) uint64_t full_bar[kEstMaxStages];
  __shared__ __align__(8) uint64_t empty_bar[kEstMaxStages];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int stages = p.stages;
  const int qrow = D * (int)sizeof(T);                        // bytes of one q row
  const int stage_f = TILE_F + (p.g * qrow + 15) / 16 * 4;    // floats per stage (16-B multiple)
  int* seq_base = reinterpret_cast<int*>(ring + stages * stage_f);  // [B+1] first chunk of seq
  int* seq_cph = seq_base + p.B + 1;                                 // [B] chunks per KV head
  const float Tf = p.temperature;
  const bool unit_t = (Tf == 1.0f);

  if (tid == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], kEstConsumerWarps);
    }
  }
  __syncthreads();
  const bool appending = p.n_new > 0 && p.k_new.data != nullptr;

  auto chunk_of = [&](int c, int& b, int& kvh, int& ch) {
    int lo = 0, hi = p.B;
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (seq_base[mid] <= c) lo = mid; else hi = mid;
    }
    b = lo;
    const int r = c - seq_base[b];
    kvh = r / seq_cph[b];
    ch = r - kvh * seq_cph[b];
  };
  // the chunk after (b, kvh, ch) in the list (sequences without chunks skipped)
  auto chunk_next = [&](int& b, int& kvh, int& ch) {
    if (++ch == seq_cph[b]) {
      ch = 0;
      if (++kvh == p.Hkv) {
        kvh = 0;
        do {
          ++b;
        } while (b < p.B && seq_cph[b] == 0);
      }
    }
  };

  if (warp == kEstConsumerWarps) {
    // ---------------- producer ----------------
    // The centroid table and q are inputs of this call (written before it by
    // kernels that complete first), so the stream starts before
    // griddepcontrol.wait, overlapping the previous kernel's tail.  Rows this
    // call's append refreshes are skipped by the consumers, so reading them
    // early is harmless.
    int carry = 0;
    for (int base = 0; base < p.B; base += 32) {  // per-sequence chunk prefix, one warp
      const int b = base + lane;
      int cnt = 0;
      if (b < p.B) {
        const int S = seq_len_of(p.seq_lens, b, p.max_seq_len);
        const bool ok = S > 0 && S <= p.max_seq_len;
        if (!ok && blockIdx.x == 0) report(p.status, ADAKV_ST_BAD_SEQ_LEN);
        const int cph = ok ? ceil_div(ceil_div(S, p.bs), kEstRows) : 0;
        seq_cph[b] = cph;
        cnt = cph * p.Hkv;
      }
      int incl = cnt;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      if (b < p.B) seq_base[b] = carry + incl - cnt;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) seq_base[p.B] = carry;
    named_bar_sync(1, (kEstConsumerWarps + 1) * 32);  // publish the chunk map to the consumers
    if (lane == 0) {
      const int total = carry;
      const int c_begin = (int)((int64_t)total * blockIdx.x / gridDim.x);
      const int c_end = (int)((int64_t)total * (blockIdx.x + 1) / gridDim.x);
      int b = 0, kvh = 0, ch = 0;
      if (c_begin < c_end) chunk_of(c_begin, b, kvh, ch);
      if constexpr (GP >= 8) {
        int s = 0, ph = 0;  // ring slot of the chunk and its use count's parity
        int nb_b = -1, nb = 0;  // sequence whose block count is in nb
        int run = -1;           // (sequence, KV head) whose queries the consumers hold
        for (int c = c_begin, i = 0; c < c_end; ++c, ++i) {
          if (i >= stages && !mbar_wait_bounded(&empty_bar[s], ph ^ 1)) {
            report(p.status, ADAKV_ST_WAIT_TIMEOUT);
            break;
          }
          if (b != nb_b) {
            nb_b = b;
            nb = ceil_div(seq_len_of(p.seq_lens, b, p.max_seq_len), p.bs);
          }
          const int row0 = ch * kEstRows;
          const int nrows = imin(kEstRows, nb - row0);
          float* st = ring + s * stage_f;
          // the query rows travel with the first chunk of each run only (the
          // consumers keep them in registers)
          const bool with_q = b * p.Hkv + kvh != run;
          run = b * p.Hkv + kvh;
          mbar_arrive_expect_tx(&full_bar[s],
                                (uint32_t)nrows * D * 4u + (with_q ? (uint32_t)(p.g * qrow) : 0u));
          bulk_g2s(st, p.cent + ((int64_t)(b * p.Hkv + kvh) * p.nb_cap + row0) * D,
                   (uint32_t)nrows * D * 4u, &full_bar[s]);
          if (with_q) {
            const T* qsrc = static_cast<const T*>(p.q.data) + b * p.q.sb + (int64_t)kvh * p.g * p.q.sh;
            for (int j = 0; j < p.g; ++j)
              bulk_g2s(reinterpret_cast<char*>(st + TILE_F) + j * qrow, qsrc + j * p.q.sh, qrow,
                       &full_bar[s]);
          }
          chunk_next(b, kvh, ch);
          if (++s == stages) {
            s = 0;
            ph ^= 1;
          }
        }
      } else {  // groups of 4: q rows in every stage (measured faster there)
        int s = 0, ph = 0;  // ring slot of the chunk and its use count's parity
        for (int c = c_begin, i = 0; c < c_end; ++c, ++i) {
          if (i >= stages && !mbar_wait_bounded(&empty_bar[s], ph ^ 1)) {
            report(p.status, ADAKV_ST_WAIT_TIMEOUT);
            break;
          }
          const int S = seq_len_of(p.seq_lens, b, p.max_seq_len);
          const int nb = ceil_div(S, p.bs);
          const int row0 = ch * kEstRows;
          const int nrows = imin(kEstRows, nb - row0);
          float* st = ring + s * stage_f;
          mbar_arrive_expect_tx(&full_bar[s], (uint32_t)nrows * D * 4u + (uint32_t)(p.g * qrow));
          bulk_g2s(st, p.cent + ((int64_t)(b * p.Hkv + kvh) * p.nb_cap + row0) * D,
                   (uint32_t)nrows * D * 4u, &full_bar[s]);
          const T* qsrc = static_cast<const T*>(p.q.data) + b * p.q.sb + (int64_t)kvh * p.g * p.q.sh;
          for (int j = 0; j < p.g; ++j)
            bulk_g2s(reinterpret_cast<char*>(st + TILE_F) + j * qrow, qsrc + j * p.q.sh, qrow,
                     &full_bar[s]);
          chunk_next(b, kvh, ch);
          if (++s == stages) {
            s = 0;
            ph ^= 1;
          }
        }
      }
    }
    pdl_wait();
  } else if (warp == kEstConsumerWarps + 1) {
    // ---------------- fused append + per-call bookkeeping ----------------
    // Loads of the touched blocks' old tokens and of the new tokens go out
    // first, ahead of the bulk stream (old tokens were written by calls that
    // completed before this grid launched); every write waits for the
    // previous grid, which may still be reading the slots rewritten here.
    using Raw = typename RawVec<T, E>::type;
    bool waited = false;
    // the rows the append refreshes are scored here; their softmax partial
    // goes to the last stats slot of each row (empty when nothing is appended)
    auto store_tail = [&](int b, int kvh, const SoftPart& t) {
      if (p.stats && lane < p.g)
        soft_store(p.stats + ((int64_t)(b * p.Hq + kvh * p.g + lane) * p.stats_stride +
                              p.stats_stride - 1) * kStatF, t);
    };
    if (!appending) {
      for (int pair = blockIdx.x; pair < p.B * p.Hkv; pair += gridDim.x)
        store_tail(pair / p.Hkv, pair % p.Hkv, soft_empty());
    }
    if (appending) {
      for (int pair = blockIdx.x; pair < p.B * p.Hkv; pair += gridDim.x) {
        const int b = pair / p.Hkv, kvh = pair - b * p.Hkv;
        const int S = seq_len_of(p.seq_lens, b, p.max_seq_len);
        SoftPart tail = soft_empty();
        if (S <= 0 || S > p.max_seq_len || S < p.n_new) {
          store_tail(b, kvh, tail);
          continue;
        }
        const int S_old = S - p.n_new;
        const int nb = ceil_div(S, p.bs);
        const int sink = imin(p.n_sink, nb), local = imin(p.n_local, nb);
        const int d = lane * E;
        T* kc = static_cast<T*>(const_cast<void*>(p.k.data)) + b * p.k.sb + kvh * p.k.sh + d;
        T* vc = static_cast<T*>(const_cast<void*>(p.v.data)) + b * p.v.sb + kvh * p.v.sh + d;
        const T* kn = static_cast<const T*>(p.k_new.data) + b * p.k_new.sb + kvh * p.k_new.sh + d;
        const T* vn = static_cast<const T*>(p.v_new.data) + b * p.v_new.sb + kvh * p.v_new.sh + d;
        const T* qb = static_cast<const T*>(p.q.data) + b * p.q.sb + (int64_t)kvh * p.g * p.q.sh + d;
        for (int blk = S_old / p.bs; blk < nb; ++blk) {
          const int t0 = blk * p.bs, t1 = imin(t0 + p.bs, S);
          float acc[E];
#pragma unroll
          for (int e = 0; e < E; ++e) acc[e] = 0.f;
          for (int base = t0; base < t1; base += 16) {
            Raw x[16];
#pragma unroll
            for (int u = 0; u < 16; ++u) {
              const int t = base + u;
              if (t < t1) {
                const T* src = (t >= S_old) ? kn + (int64_t)(t - S_old) * p.k_new.ss
                                            : kc + (int64_t)t * p.k.ss;
                x[u] = *reinterpret_cast<const Raw*>(src);
              }
            }
            if (!waited) {
              pdl_wait();
              waited = true;
            }
#pragma unroll
            for (int u = 0; u < 16; ++u) {
              const int t = base + u;
              if (t < t1 && t >= S_old) {
                *reinterpret_cast<Raw*>(kc + (int64_t)t * p.k.ss) = x[u];
                *reinterpret_cast<Raw*>(vc + (int64_t)t * p.v.ss) =
                    *reinterpret_cast<const Raw*>(vn + (int64_t)(t - S_old) * p.v_new.ss);
              }
            }
#pragma unroll
            for (int u = 0; u < 16; ++u) {
              const int t = base + u;
              if (t < t1) {
                float xf[E];
                RawVec<T, E>::unpack(x[u], xf);
#pragma unroll
                for (int e = 0; e < E; ++e) acc[e] = (t == t0) ? xf[e] : __fadd_rn(acc[e], xf[e]);
              }
            }
          }
          const float n = (float)(t1 - t0);
          float cen[E];
#pragma unroll
          for (int e = 0; e < E; ++e) cen[e] = __fdiv_rn(acc[e], n);
          float* crow = p.cent + ((int64_t)(b * p.Hkv + kvh) * p.nb_cap + blk) * D + d;
#pragma unroll
          for (int e = 0; e < E; ++e) crow[e] = cen[e];
          for (int j = 0; j < p.g; ++j) {
            float qv[E];
            load_vec<T, E>(qb + j * p.q.sh, qv);
            float part = 0.f;
#pragma unroll
            for (int e = 0; e < E; ++e) part = fmaf(qv[e], cen[e], part);
#pragma unroll
            for (int o = 16; o; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
            if (lane == 0)
              p.scores[(int64_t)(b * p.Hq + kvh * p.g + j) * p.score_stride + blk] = part;
            if (lane == j)
              soft_add(tail, part, unit_t ? part : __fdiv_rn(part, Tf),
                       !(blk < sink || blk >= nb - local));
          }
        }
        store_tail(b, kvh, tail);
      }
    }
    if (!waited) pdl_wait();
    if (blockIdx.x == 0 && lane == 0 && p.epoch) atomicAdd(p.epoch, 1u);
    // clear the plan's weight-exchange tags of this call's rows (the plan kernel
    // starts after this grid completes, so no stale tag can satisfy its barrier)
    if (p.slots) {
      for (int r = blockIdx.x * 32 + lane; r < p.B * p.Hq * kPlanSlotsPerRow; r += gridDim.x * 32)
        p.slots[r].word = 0ull;
    }
    if (p.counters) {
      for (int r = blockIdx.x * 32 + lane; r < p.B * p.Hkv; r += gridDim.x * 32) p.counters[r] = 0u;
    }
  } else {
    // ---------------- consumers ----------------
    named_bar_sync(1, (kEstConsumerWarps + 1) * 32);  // chunk map written by the producer warp
    const int total = seq_base[p.B];
    const int c_begin = (int)((int64_t)total * blockIdx.x / gridDim.x);
    const int c_end = (int)((int64_t)total * (blockIdx.x + 1) / gridDim.x);
    float qr[GP][E];  // the group's query slices, loaded when the (sequence, KV head) changes
    int qrun = -1;
    int b = 0, kvh = 0, ch = 0;
    if (c_begin < c_end) chunk_of(c_begin, b, kvh, ch);
    int s = 0, ph = 0;  // ring slot of the chunk and its use count's parity
    int S_b = -1, S = 0;
    for (int c = c_begin; c < c_end; ++c) {
      if (b != S_b) {  // the sequence's length, read once per sequence
        S_b = b;
        S = seq_len_of(p.seq_lens, b, p.max_seq_len);
      }
      // a lane that gives up makes the whole warp give up: the shuffles below
      // need every lane
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&full_bar[s], ph))) {
        if (lane == 0) report(p.status, ADAKV_ST_WAIT_TIMEOUT);
        break;
      }
      const int nb = ceil_div(S, p.bs);
      const int row0 = ch * kEstRows;
      const int nrows = imin(kEstRows, nb - row0);
      // rows refreshed by the append warp are scored there
      const int skip_from = appending ? (S - p.n_new) / p.bs - row0 : nrows;
      const int lim = imin(nrows, skip_from);
      const float* tile = ring + s * stage_f;
      // groups of 8+ heads: only the first chunk of a run carries q (producer)
      if (GP < 8 || b * p.Hkv + kvh != qrun) {
        qrun = b * p.Hkv + kvh;
        const T* qs = reinterpret_cast<const T*>(tile + TILE_F);
#pragma unroll
        for (int j = 0; j < GP; ++j) {
          if (j < p.g) {
            load_vec<T, E>(qs + j * D + lane * E, qr[j]);
          } else {
#pragma unroll
            for (int e = 0; e < E; ++e) qr[j][e] = 0.f;
          }
        }
      }
      float scs[NG];  // this lane's scores of the chunk (kept for the softmax partial)
#pragma unroll
      for (int grp = 0; grp < NG; ++grp) {
        const int rbase = warp * RPW + grp * R;
        float v[32];
#pragma unroll
        for (int r = 0; r < R; ++r) {
          float cr[E];
          lds_row<E>(tile + (rbase + r) * D + lane * E, cr);
#pragma unroll
          for (int j = 0; j < GP; ++j) {
            float acc = 0.f;
#pragma unroll
            for (int e = 0; e < E; ++e) acc = fmaf(qr[j][e], cr[e], acc);
            v[r * GP + j] = acc;
          }
        }
        const float sc = warp_reduce_scatter32(v, lane);
        scs[grp] = sc;
        const int row = rbase + lane / GP, j = lane % GP;
        if (j < p.g && row < lim)
          p.scores[(int64_t)(b * p.Hq + kvh * p.g + j) * p.score_stride + row0 + row] = sc;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_bar[s]);  // the stage refills while the partial is built
      if (p.stats) {
        // Softmax partial of this warp's rows of each head: maxima over the
        // lanes of a head first (independent xor shuffles), then one exp per
        // score relative to the head's warp max, then xor sums.
        const int sink = imin(p.n_sink, nb), local = imin(p.n_local, nb);
        float zv[NG];
        bool ok[NG], cont[NG];
        float m = -INFINITY, mxl = -INFINITY, cmxl = -INFINITY, csl = 0.f, cql = 0.f;
#pragma unroll
        for (int grp = 0; grp < NG; ++grp) {
          const int row = warp * RPW + grp * R + lane / GP, j = lane % GP;
          const int blk = row0 + row;
          ok[grp] = j < p.g && row < lim;
          cont[grp] = ok[grp] && !(blk < sink || blk >= nb - local);
          zv[grp] = unit_t ? scs[grp] : __fdiv_rn(scs[grp], Tf);
          if (ok[grp]) {
            m = fmaxf(m, zv[grp]);
            mxl = fmaxf(mxl, scs[grp]);
          }
          if (cont[grp]) {
            cmxl = fmaxf(cmxl, scs[grp]);
            csl += scs[grp];
            cql = fmaf(scs[grp], scs[grp], cql);
          }
        }
#pragma unroll
        for (int o = GP; o < 32; o <<= 1) {
          m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
          mxl = fmaxf(mxl, __shfl_xor_sync(0xffffffffu, mxl, o));
          cmxl = fmaxf(cmxl, __shfl_xor_sync(0xffffffffu, cmxl, o));
        }
        float zl = 0.f, al = 0.f;
#pragma unroll
        for (int grp = 0; grp < NG; ++grp) {
          if (ok[grp]) {
            const float d = zv[grp] - m;
            const float e = expf(d);
            zl += e;
            al = fmaf(e, d, al);
          }
        }
#pragma unroll
        for (int o = GP; o < 32; o <<= 1) {
          zl += __shfl_xor_sync(0xffffffffu, zl, o);
          al += __shfl_xor_sync(0xffffffffu, al, o);
          csl += __shfl_xor_sync(0xffffffffu, csl, o);
          cql += __shfl_xor_sync(0xffffffffu, cql, o);
        }
        const SoftPart part{mxl, cmxl, csl, cql, m, zl, al};
        if (lane < p.g)
          soft_store(p.stats + ((int64_t)(b * p.Hq + kvh * p.g + lane) * p.stats_stride +
                                ch * kEstConsumerWarps + warp) * kStatF, part);
      }
      chunk_next(b, kvh, ch);
      if (++s == stages) {
        s = 0;
        ph ^= 1;
      }
    }
    pdl_wait();  // (no-op for ordering here; keeps every thread's wait uniform)
  }
  pdl_launch_dependents();
}

int estimate_stage_bytes(int dtype, int D, int g) {
  const int tile = kEstRows * D * 4;
  const int q = (g * D * (dtype == ADAKV_DTYPE_F32 ? 4 : 2) + 15) / 16 * 16;
  return tile + q;
}

int estimate_stages(int dtype, int D, int g, int B) {
  const size_t fixed = sizeof(int) * (2 * (size_t)B + 2);
  const size_t room = kEstSmemBudget > fixed ? kEstSmemBudget - fixed : 0;
  const int st = (int)(room / estimate_stage_bytes(dtype, D, g));
  return imax(2, imin(kEstMaxStages, st));
}

size_t estimate_smem_bytes(int dtype, int D, int g, int B) {
  return (size_t)estimate_stages(dtype, D, g, B) * estimate_stage_bytes(dtype, D, g) +
         sizeof(int) * (2 * (size_t)B + 2);
}

template <typename F>
static cudaError_t for_each_estimate(int dtype, int D, int g, F&& f) {
#define ADAKV_EST_G(TT, DD)                                      \
  if (D == DD) {                                                 \
    if (g <= 4) return f(estimate_kernel<TT, DD, 4>);            \
    if (g <= 8) return f(estimate_kernel<TT, DD, 8>);            \
    if (g <= 16) return f(estimate_kernel<TT, DD, 16>);          \
  }
  if (dtype == ADAKV_DTYPE_F32) {
    ADAKV_EST_G(float, 64) ADAKV_EST_G(float, 128)
  } else if (dtype == ADAKV_DTYPE_F16) {
    ADAKV_EST_G(__half, 64) ADAKV_EST_G(__half, 128)
  } else if (dtype == ADAKV_DTYPE_BF16) {
    ADAKV_EST_G(__nv_bfloat16, 64) ADAKV_EST_G(__nv_bfloat16, 128)
  }
#undef ADAKV_EST_G
  return cudaErrorInvalidValue;
}

cudaError_t estimate_kernels_init() {
  for (int dt = 0; dt < 3; ++dt)
    for (int D : {64, 128})
      for (int g : {4, 8, 16}) {
        const size_t smem = kEstSmemBudget + 1024;
        cudaError_t e = for_each_estimate(dt, D, g, [&](auto kern) {
          return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        });
        if (e != cudaSuccess) return e;
      }
  return cudaSuccess;
}

cudaError_t launch_estimate(const EstParams& p, int dtype, int D, int nb_max, int grid,
                            cudaStream_t st, const LaunchOpts& o) {
  (void)nb_max;
  const size_t smem = estimate_smem_bytes(dtype, D, p.g, p.B);
  return for_each_estimate(dtype, D, p.g, [&](auto kern) {
    return launch_ex(kern, dim3(grid), dim3(kEstThreads), smem, st, o, p);
  });
}

}  // namespace adakv
