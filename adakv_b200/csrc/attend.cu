// (d) Fused ragged block-sparse split-KV flash decode over the GQA union.
//
// out[b, h] = softmax_t((q[b, h] . K[b, h/g, t]) * sm_scale) . V[b, h/g, t] over the
// tokens t of head h's selected blocks (tokens >= seq_len masked): the semantics
// of the reference kernel (adakv/kernels/block_sparse_decode.py:51-100) and of
// the oracle (adakv/reference.py:76-80).
//
// Grid (SPLIT, Hkv, B).  The g query heads of a KV group select overlapping
// block sets; every CTA of the group ORs their selection bitmaps into the
// union and takes the SPLIT-th share of it (the split-KV axis), so each
// selected K/V block is read from HBM exactly once for the whole group.  A CTA
// gathers its blocks with 16-byte cp.async copies (zero-fill past seq_len)
// into a two-stage shared-memory ring and computes online-softmax partials of
// all g heads; each block is masked per head by the head's own selection.
// Partials (m, l, o) go to the workspace; the last CTA of the group to finish
// (an atomic arrival count, reset by that CTA) merges the SPLIT partials in
// split order and writes out[b, h] for the group.  No CTA waits on another.
//
// Tensor-core path (bf16 / fp16): the g rows of the group are the M = 16
// rows of an m16n8k16 MMA tile (attend_mma.cuh), 8 warps split the blocks of
// a batch.  CUDA-core path (fp32): 1-4 warps per query head, a token row is
// spread over D * 4 / 16 lanes and dot products finish with xor shuffles.
//
// HBM traffic: the union of the group's selected K/V blocks
// (bs * D * sizeof(T) * 2 bytes per block) plus the bitmaps, q, out and the
// partials (g * (D + 2) * 4 bytes per CTA, L2 resident).
#include <type_traits>

#include "attend_mma.cuh"
#include "kernels.h"

namespace adakv {

constexpr int kAttendMaxThreads = 512;  // CUDA-core path: g <= 16 warps
constexpr int kAttendMmaWarps = 8;

// shared-memory carve-up of one attend CTA (host and device agree on it)
struct AttendSmem {
  size_t kv, uw, list, mask, wpart, merge, total;
};

// Warps of one CTA: tensor-core path, kAttendMmaWarps split the blocks;
// CUDA-core path, 1-4 warps per query head.
__host__ __device__ inline int attend_warps(bool mma, int g) {
  if (mma) return kAttendMmaWarps;
  int wph = 16 / g;
  wph = wph < 1 ? 1 : (wph > 4 ? 4 : wph);
  return g * wph;
}

__host__ __device__ inline AttendSmem attend_smem_layout(int elt, int D, int BS, int nslot, int g,
                                                         int nw_max, int slice_cap, int split,
                                                         bool mma) {
  auto al = [](size_t x) { return (x + 127) / 128 * 128; };
  const int nwarps = attend_warps(mma, g);
  const int prow = mma ? g : 1;  // per-warp partial rows
  AttendSmem s;
  s.kv = 0;
  s.uw = s.kv + al((size_t)2 * 2 * nslot * BS * D * elt);  // 2 stages x (K, V)
  s.list = s.uw + al((size_t)nw_max * 4);
  s.mask = s.list + al((size_t)slice_cap * 4);
  s.wpart = s.mask + al((size_t)slice_cap * 4);
  s.merge = s.wpart + al((size_t)nwarps * prow * (D + 2) * 4);
  s.total = s.merge + al((size_t)(2 * split * g + g) * 4);
  return s;
}

template <typename T, int D, int BS, bool MMA>
__global__ void __launch_bounds__(MMA ? kAttendMmaWarps * 32 : kAttendMaxThreads) attend_kernel(AttendParams p) {
  constexpr int VEC = 16 / sizeof(T);       // elements per 16-byte chunk
  constexpr int LPT = D / VEC;              // lanes per token row (CUDA-core path)
  constexpr int TPP = 32 / LPT;             // token rows per warp pass
  constexpr int PASSES = BS / TPP;
  constexpr int ROWC = D / VEC;             // 16-byte chunks per token row
  constexpr int BLK = BS * D;               // elements of one K (or V) block
  static_assert(LPT <= 32 && BS % TPP == 0, "unsupported tile shape");
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ int scan_scratch[33];
  __shared__ int s_last;

  const int split = blockIdx.x, SPLIT = gridDim.x;
  const int kvh = blockIdx.y, b = blockIdx.z;
  const int grp = b * p.Hkv + kvh;
  const int nthr = blockDim.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nwarps = nthr >> 5;
  const int g = p.g, NSLOT = p.nbt;
  const AttendSmem L =
      attend_smem_layout(sizeof(T), D, BS, NSLOT, g, p.nw_max, p.slice_cap, SPLIT, MMA);
  T* kvbuf = reinterpret_cast<T*>(smem + L.kv);                // [2][K, V][NSLOT][BS][D]
  uint32_t* uw = reinterpret_cast<uint32_t*>(smem + L.uw);     // [nw_max] union words
  int* list = reinterpret_cast<int*>(smem + L.list);           // [slice_cap] block ids
  uint32_t* lmask = reinterpret_cast<uint32_t*>(smem + L.mask);  // [slice_cap] head bits
  float* wpart = reinterpret_cast<float*>(smem + L.wpart);     // per-warp partials
  float* mf = reinterpret_cast<float*>(smem + L.merge);        // merge: [SPLIT][g] factors
  float* ml = mf + SPLIT * g;                                  // [g] merged maxima
  float* mL = ml + SPLIT * g;                                  // [g] merged denominators

  // inputs of the whole step (written before the estimator ran): load them
  // before waiting for the plan
  int S = seq_len_of(p.seq_lens, b, p.max_seq_len);
  if (S < 0 || S > p.max_seq_len) S = 0;
  const int nb = ceil_div(S, BS);
  const int nw = ceil_div(nb, 32);
  const int row0 = b * p.Hq + kvh * g;
  const T* kbase = static_cast<const T*>(p.k.data) + b * p.k.sb + kvh * p.k.sh;
  const T* vbase = static_cast<const T*>(p.v.data) + b * p.v.sb + kvh * p.v.sh;
  const T* qbase = static_cast<const T*>(p.q.data) + b * p.q.sb + (int64_t)kvh * g * p.q.sh;
  MmaAcc<D> acc;
  uint32_t qa[D / 16][4];
  float qf[VEC];
  float m_run = -INFINITY, l_run = 0.f, o[VEC];
  const int gid = lane >> 2, tig = lane & 3;
  if constexpr (MMA) {
#pragma unroll
    for (int nn = 0; nn < MmaAcc<D>::NT; ++nn)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc.o[nn][e] = 0.f;
    acc.m[0] = acc.m[1] = -INFINITY;
    acc.l[0] = acc.l[1] = 0.f;
    // A fragments of q: rows = query heads of the group (rows >= g are zero)
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int row = gid + (e & 1) * 8;
        const int col = ks * 16 + (e >> 1) * 8 + tig * 2;
        qa[ks][e] = row < g ? *reinterpret_cast<const uint32_t*>(qbase + (int64_t)row * p.q.sh + col)
                            : 0u;
      }
    }
  } else {
    const int WPH = nwarps / g;
    const int head = warp / WPH;
    const int d0 = (lane % LPT) * VEC;
    const uint4 u = *reinterpret_cast<const uint4*>(qbase + (int64_t)head * p.q.sh + d0);
    Unpack16<T>::run(u, qf);
#pragma unroll
    for (int e = 0; e < VEC; ++e) o[e] = 0.f;
  }
  const float scale_log2 = p.sm_scale * 1.4426950408889634f;
  pdl_wait();

  // ---- union of the group's selection bitmaps; this CTA's share of it ----
  // Each thread ORs a run of consecutive words, four words' loads in flight
  // at a time; the share is then enumerated from the union in shared memory
  // and every listed block's head mask is fetched in one parallel pass.
  const int wpt = ceil_div(nw, nthr);
  const int w0 = imin(tid * wpt, nw), w1 = imin(w0 + wpt, nw);
  int cnt = 0;
  for (int wb = w0; wb < w1; wb += 4) {
    uint32_t u4[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (wb + k < w1) {
#pragma unroll
        for (int hh = 0; hh < 16; ++hh)
          if (hh < g) u4[k] |= p.bitmap[(int64_t)(row0 + hh) * p.bm_words + wb + k];
      }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (wb + k < w1) {
        uw[wb + k] = u4[k];
        cnt += __popc(u4[k]);
      }
    }
  }
  const int before = block_exclusive_scan(cnt, scan_scratch);
  const int U = scan_scratch[32];
  const int lo = (int)((int64_t)U * split / SPLIT), hi = (int)((int64_t)U * (split + 1) / SPLIT);
  if (before < hi && before + cnt > lo) {
    int rk = before;
    for (int w = w0; w < w1 && rk < hi; ++w) {
      uint32_t u = uw[w];
      const int pc = __popc(u);
      if (rk + pc <= lo) {  // the whole word lies before this CTA's share
        rk += pc;
        continue;
      }
      while (u && rk < hi) {
        const int bit = __ffs(u) - 1;
        u &= u - 1u;
        if (rk >= lo) list[rk - lo] = w * 32 + bit;
        ++rk;
      }
    }
  }
  __syncthreads();
  for (int i = tid; i < hi - lo; i += nthr) {
    const int id = list[i], w = id >> 5, bit = id & 31;
    uint32_t m = 0;
#pragma unroll
    for (int hh = 0; hh < 16; ++hh)
      if (hh < g) m |= ((p.bitmap[(int64_t)(row0 + hh) * p.bm_words + w] >> bit) & 1u) << hh;
    lmask[i] = m;
  }
  __syncthreads();
  const int n = hi - lo;

  // ---- two-stage gather ring + compute, NSLOT blocks per stage ----
  auto issue = [&](int first, int stage) {
    const int cntb = imin(NSLOT, n - first);
    T* kb = kvbuf + (size_t)stage * 2 * NSLOT * BLK;
    T* vb = kb + (size_t)NSLOT * BLK;
    const int chunks = cntb * BS * ROWC;
    for (int c = tid; c < chunks; c += nthr) {
      const int slot = c / (BS * ROWC);
      const int rem = c - slot * (BS * ROWC);
      const int tok = rem / ROWC, col = rem - tok * ROWC;
      const int pos = list[first + slot] * BS + tok;
      const bool valid = pos < S;
      const int64_t srow = valid ? (int64_t)pos : 0;
      const int pcol = MMA ? (col ^ (tok & 7)) : col;  // swizzle for ldmatrix
      const size_t off = (size_t)slot * BLK + tok * D + pcol * VEC;
      cp_async16(kb + off, kbase + srow * p.k.ss + col * VEC, valid);
      cp_async16(vb + off, vbase + srow * p.v.ss + col * VEC, valid);
    }
    cp_async_commit();
  };
  int seen = 0;
  const int nbatch = ceil_div(n, NSLOT);
  if (nbatch > 0) issue(0, 0);
  for (int bi = 0; bi < nbatch; ++bi) {
    const int first = bi * NSLOT;
    const int cntb = imin(NSLOT, n - first);
    if (bi + 1 < nbatch) {
      issue(first + NSLOT, (bi + 1) & 1);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      cp_async_wait_all();
    }
    __syncthreads();
    const T* kb = kvbuf + (size_t)(bi & 1) * 2 * NSLOT * BLK;
    const T* vb = kb + (size_t)NSLOT * BLK;
    if constexpr (MMA) {
      for (int slot = warp; slot < cntb; slot += nwarps) {
        const int blk = list[first + slot];
        const int tok_valid = imin(BS, S - blk * BS);
        mma_block<T, D, BS>(acc, qa, smem_addr(kb + (size_t)slot * BLK),
                            smem_addr(vb + (size_t)slot * BLK), lmask[first + slot], tok_valid,
                            scale_log2, lane);
      }
    } else {
      const int WPH = nwarps / g;
      const int head = warp / WPH, sub = warp - head * WPH;
      const int d0 = (lane % LPT) * VEC;
      const int tl = lane / LPT;
      for (int slot = 0; slot < cntb; ++slot) {
        if (!((lmask[first + slot] >> head) & 1u)) continue;  // warp-uniform
        if ((seen++ % WPH) != sub) continue;
        const int blk = list[first + slot];
        const T* kt = kb + (size_t)slot * BLK;
        const T* vt = vb + (size_t)slot * BLK;
        float sc[PASSES];
#pragma unroll
        for (int pp = 0; pp < PASSES; ++pp) {
          const int tok = pp * TPP + tl;
          const uint4 u = *reinterpret_cast<const uint4*>(kt + tok * D + d0);
          float kf[VEC];
          Unpack16<T>::run(u, kf);
          float part = 0.f;
#pragma unroll
          for (int e = 0; e < VEC; ++e) part = fmaf(qf[e], kf[e], part);
#pragma unroll
          for (int off = LPT / 2; off >= 1; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
          sc[pp] = (blk * BS + tok < S) ? part * scale_log2 : -INFINITY;
        }
        float mb = sc[0];
#pragma unroll
        for (int pp = 1; pp < PASSES; ++pp) mb = fmaxf(mb, sc[pp]);
#pragma unroll
        for (int off = LPT; off < 32; off <<= 1) mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, off));
        const float m_new = fmaxf(m_run, mb);
        if (m_new == -INFINITY) continue;
        const float alpha = exp2f(m_run - m_new);
        float l_part = 0.f;
#pragma unroll
        for (int e = 0; e < VEC; ++e) o[e] *= alpha;
#pragma unroll
        for (int pp = 0; pp < PASSES; ++pp) {
          const int tok = pp * TPP + tl;
          const float pt = exp2f(sc[pp] - m_new);
          l_part += pt;
          const uint4 u = *reinterpret_cast<const uint4*>(vt + tok * D + d0);
          float vf[VEC];
          Unpack16<T>::run(u, vf);
#pragma unroll
          for (int e = 0; e < VEC; ++e) o[e] = fmaf(pt, vf[e], o[e]);
        }
        l_run = l_run * alpha + l_part;
        m_run = m_new;
      }
    }
    __syncthreads();  // this stage is refilled two batches later
  }

  // ---- warp partials -> this CTA's partial of each head (max in log2 units) ----
  float* gpart = p.part + ((size_t)grp * SPLIT + split) * g * (D + 2);  // [g][m, l, o[D]]
  if constexpr (MMA) {
    float l0 = acc.l[0], l1 = acc.l[1];
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    float* mine = wpart + warp * g * (D + 2);  // [g][D + 2] = m, l, o[D]
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int row = gid + half * 8;
      if (row < g) {
        float* rp = mine + row * (D + 2);
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
    __syncthreads();
    for (int idx = tid; idx < g * D; idx += nthr) {
      const int hh = idx / D, d = idx - hh * D;
      float M = -INFINITY;
      for (int w = 0; w < nwarps; ++w) M = fmaxf(M, wpart[(w * g + hh) * (D + 2)]);
      float Ls = 0.f, O = 0.f;
      if (M != -INFINITY) {
        for (int w = 0; w < nwarps; ++w) {
          const float* rp = wpart + (w * g + hh) * (D + 2);
          const float f = (rp[0] == -INFINITY) ? 0.f : exp2f(rp[0] - M);
          Ls += rp[1] * f;
          O += rp[2 + d] * f;
        }
      }
      gpart[hh * (D + 2) + 2 + d] = O;
      if (d == 0) {
        gpart[hh * (D + 2)] = M;
        gpart[hh * (D + 2) + 1] = Ls;
      }
    }
  } else {
#pragma unroll
    for (int off = LPT; off < 32; off <<= 1) {
      l_run += __shfl_xor_sync(0xffffffffu, l_run, off);
#pragma unroll
      for (int e = 0; e < VEC; ++e) o[e] += __shfl_xor_sync(0xffffffffu, o[e], off);
    }
    const int d0 = (lane % LPT) * VEC;
    float* mine = wpart + warp * (D + 2);
    if (lane < LPT) {
#pragma unroll
      for (int e = 0; e < VEC; ++e) mine[2 + d0 + e] = o[e];
    }
    if (lane == 0) {
      mine[0] = m_run;
      mine[1] = l_run;
    }
    __syncthreads();
    const int WPH = nwarps / g;
    for (int idx = tid; idx < g * D; idx += nthr) {
      const int hh = idx / D, d = idx - hh * D;
      const float* wp = wpart + hh * WPH * (D + 2);
      float M = -INFINITY;
      for (int w = 0; w < WPH; ++w) M = fmaxf(M, wp[w * (D + 2)]);
      float Ls = 0.f, O = 0.f;
      if (M != -INFINITY) {
        for (int w = 0; w < WPH; ++w) {
          const float mw = wp[w * (D + 2)];
          const float f = (mw == -INFINITY) ? 0.f : exp2f(mw - M);
          Ls += wp[w * (D + 2) + 1] * f;
          O += wp[w * (D + 2) + 2 + d] * f;
        }
      }
      gpart[hh * (D + 2) + 2 + d] = O;
      if (d == 0) {
        gpart[hh * (D + 2)] = M;
        gpart[hh * (D + 2) + 1] = Ls;
      }
    }
  }

  // ---- the last CTA of the group merges the SPLIT partials ----
  // Arrival is one acq_rel atomic by thread 0 after the CTA barrier: release
  // publishes this CTA's partial (ordered before it by the barrier), acquire
  // makes the other CTAs' partials visible to the merging CTA.
  __syncthreads();
  if (tid == 0) {
    unsigned prev;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;"
                 : "=r"(prev)
                 : "l"(p.counters + grp)
                 : "memory");
    s_last = prev == (unsigned)(SPLIT - 1);
  }
  __syncthreads();
  if (!s_last) {
    pdl_launch_dependents();
    return;
  }
  const float* gp0 = p.part + (size_t)grp * SPLIT * g * (D + 2);
  const size_t stride = (size_t)g * (D + 2);  // between splits
  // per-head max over splits and merge factors: warp w takes heads w, w + nwarps, ...
  static_assert(kAttendMaxSplit <= 64, "two splits per lane");
  for (int hh = warp; hh < g; hh += nwarps) {
    float m2[2], l2[2];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int s2 = lane + 32 * q;
      const float* pp = gp0 + s2 * stride + hh * (D + 2);
      m2[q] = s2 < SPLIT ? __ldcg(pp) : -INFINITY;
      l2[q] = s2 < SPLIT ? __ldcg(pp + 1) : 0.f;
    }
    const float M = warp_max(fmaxf(m2[0], m2[1]));
    float Ls = 0.f;
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int s2 = lane + 32 * q;
      const float f = (M == -INFINITY || m2[q] == -INFINITY) ? 0.f : exp2f(m2[q] - M);
      if (s2 < SPLIT) mf[s2 * g + hh] = f;
      Ls += l2[q] * f;
    }
    Ls = warp_sum(Ls);
    if (lane == 0) {
      mL[hh] = Ls;
      ml[hh] = M;
    }
  }
  __syncthreads();
  for (int idx = tid; idx < g * D; idx += nthr) {
    const int hh = idx / D, d = idx - hh * D;
    const float* src = gp0 + (size_t)hh * (D + 2) + 2 + d;
    float O = 0.f;
    for (int s0 = 0; s0 < SPLIT; s0 += 32) {  // up to 32 loads in flight per round trip
      float v[32];
#pragma unroll
      for (int u = 0; u < 32; ++u) v[u] = s0 + u < SPLIT ? __ldcg(src + (size_t)(s0 + u) * stride) : 0.f;
#pragma unroll
      for (int u = 0; u < 32; ++u)
        if (s0 + u < SPLIT) O += mf[(s0 + u) * g + hh] * v[u];
    }
    const float Ls = mL[hh];
    const float res = Ls > 0.f ? O / Ls : 0.f;
    if (p.out_f32) {
      p.out_f32[(int64_t)(row0 + hh) * D + d] = res;
    } else {
      T* orow = static_cast<T*>(const_cast<void*>(p.out.data)) + b * p.out.sb +
                (int64_t)(kvh * g + hh) * p.out.sh;
      orow[d] = from_f32<T>(res);
    }
  }
  if (p.lse && tid < g) {
    // merged max M is in log2 units of (score * sm_scale): lse = M ln 2 + ln L
    const float M = ml[tid];
    const float Ls = mL[tid];
    p.lse[row0 + tid] = (Ls > 0.f && M > -INFINITY) ? M * 0.6931471805599453f + logf(Ls) : -INFINITY;
  }
  if (tid == 0) p.counters[grp] = 0u;  // ready for the next call
  pdl_launch_dependents();
}

// Stand-alone attend: caller-given (block_table, sel_lens) -> per-head bitmaps.
// Duplicate ids collapse to one bit; ids outside [0, nb) are flagged and skipped.
__global__ void __launch_bounds__(256) table_bitmap_kernel(TableParams p) {
  extern __shared__ uint32_t sbits[];
  const int h = blockIdx.x, b = blockIdx.y, row = b * p.Hq + h;
  pdl_wait();
  if (h == 0 && b == 0 && p.counters)
    for (int i = threadIdx.x; i < p.ncounters; i += blockDim.x) p.counters[i] = 0u;
  int S = seq_len_of(p.seq_lens, b, p.max_seq_len);
  if (S < 0 || S > p.max_seq_len) {
    if (threadIdx.x == 0 && h == 0) report(p.status, ADAKV_ST_BAD_SEQ_LEN);
    S = 0;
  }
  const int nb = ceil_div(S, p.bs);
  const int nw = ceil_div(nb, 32);
  for (int w = threadIdx.x; w < nw; w += blockDim.x) sbits[w] = 0u;
  __syncthreads();
  int k = p.sel_lens[row];
  if (k < 0 || k > p.table_width) {
    if (threadIdx.x == 0) report(p.status, ADAKV_ST_BAD_SEL_LEN);
    k = k < 0 ? 0 : p.table_width;
  }
  const int* trow = p.block_table + (int64_t)row * p.table_width;
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    const int blk = trow[i] - p.block_offset;
    if (blk < 0 || blk >= nb) {
      if (!p.local_only) report(p.status, ADAKV_ST_BAD_BLOCK_ID);
    } else {
      atomicOr(&sbits[blk >> 5], 1u << (blk & 31));
    }
  }
  __syncthreads();
  for (int w = threadIdx.x; w < nw; w += blockDim.x) p.bitmap[(int64_t)row * p.bm_words + w] = sbits[w];
  pdl_launch_dependents();
}

template <typename F>
static cudaError_t for_each_attend(int dtype, int D, int bs, F&& f) {
#define ADAKV_ATT_CASE(TT, DD, BB) \
  if (D == DD && bs == BB) return f(attend_kernel<TT, DD, BB, !std::is_same<TT, float>::value>, (int)sizeof(TT));
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

bool attend_uses_mma(int dtype) { return dtype != ADAKV_DTYPE_F32; }

int attend_threads(int dtype, int g) { return 32 * attend_warps(attend_uses_mma(dtype), g); }

size_t attend_smem_bytes(int dtype, int D, int bs, int nbt, int g, int nw_max, int slice_cap,
                         int split) {
  return attend_smem_layout(dtype == ADAKV_DTYPE_F32 ? 4 : 2, D, bs, nbt, g, nw_max, slice_cap,
                            split, attend_uses_mma(dtype))
      .total;
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
  return cudaFuncSetAttribute(table_bitmap_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              64 * 1024);
}

cudaError_t launch_attend(const AttendParams& p, int dtype, int D, int bs, int split,
                          cudaStream_t st, const LaunchOpts& o) {
  const size_t smem = attend_smem_bytes(dtype, D, bs, p.nbt, p.g, p.nw_max, p.slice_cap, split);
  return for_each_attend(dtype, D, bs, [&](auto kern, int) {
    return launch_ex(kern, dim3(split, p.Hkv, p.B), dim3(attend_threads(dtype, p.g)), smem, st, o, p);
  });
}

// Merge of per-shard attention outputs of one query head (sequence-sharded
// decode): out = sum_n exp(lse_n - LSE) o_n with LSE = log sum_n exp(lse_n);
// rows with no selected token anywhere (every lse_n = -inf) produce zeros.
template <typename T>
__global__ void __launch_bounds__(128) combine_kernel(CombineParams p) {
  const int row = blockIdx.x;
  pdl_wait();
  float M = -INFINITY;
  for (int n = 0; n < p.n_parts; ++n) M = fmaxf(M, p.lse[n * p.lse_stride + row]);
  float den = 0.f;
  for (int n = 0; n < p.n_parts; ++n) {
    const float l = p.lse[n * p.lse_stride + row];
    den += (M == -INFINITY || l == -INFINITY) ? 0.f : expf(l - M);
  }
  const int b = row / p.Hq, h = row - b * p.Hq;
  T* orow = static_cast<T*>(const_cast<void*>(p.out.data)) + b * p.out.sb + (int64_t)h * p.out.sh;
  for (int d = threadIdx.x; d < p.D; d += blockDim.x) {
    float acc = 0.f;
    for (int n = 0; n < p.n_parts; ++n) {
      const float l = p.lse[n * p.lse_stride + row];
      if (M == -INFINITY || l == -INFINITY) continue;
      acc += expf(l - M) * p.parts[n * p.part_stride + (int64_t)row * p.D + d];
    }
    orow[d] = from_f32<T>(den > 0.f ? acc / den : 0.f);
  }
  pdl_launch_dependents();
}

cudaError_t launch_combine(const CombineParams& p, int dtype, cudaStream_t st, const LaunchOpts& o) {
  if (dtype == ADAKV_DTYPE_F32)
    return launch_ex(combine_kernel<float>, dim3(p.rows), dim3(128), 0, st, o, p);
  if (dtype == ADAKV_DTYPE_F16)
    return launch_ex(combine_kernel<__half>, dim3(p.rows), dim3(128), 0, st, o, p);
  return launch_ex(combine_kernel<__nv_bfloat16>, dim3(p.rows), dim3(128), 0, st, o, p);
}

cudaError_t launch_table_bitmap(const TableParams& p, cudaStream_t st, const LaunchOpts& o) {
  const int nw_max = ceil_div(ceil_div(p.max_seq_len, p.bs), 32);
  return launch_ex(table_bitmap_kernel, dim3(p.Hq, p.B), dim3(256), (size_t)nw_max * 4, st, o, p);
}

}  // namespace adakv
