// (d) Fused ragged block-sparse split-KV flash decode over the GQA union.
//
// out[b, h] = softmax_t((q[b, h] . K[b, h/g, t]) * sm_scale) . V[b, h/g, t] over the
// tokens t of head h's selected blocks (tokens >= seq_len masked): the semantics
// of the reference kernel (adakv/kernels/block_sparse_decode.py:51-100) and of
// the oracle (adakv/reference.py:76-80).
//
// One thread-block cluster per (sequence, KV head).  The g query heads of the
// group select overlapping block sets; the cluster reads their selection
// bitmaps, forms the union, and splits the union evenly over its CTAs, so every
// selected K/V block is read from HBM exactly once for the whole group (the
// split-KV axis).  Each CTA gathers its blocks with 16-byte cp.async copies
// (zero-fill past seq_len) into a double-buffered shared-memory ring, and warp
// h of the CTA runs the online softmax of query head h over the blocks whose
// head bit is set: a token row is spread over D*sizeof(T)/16 lanes, dot products
// finish with xor shuffles, the lane keeps its 16-byte slice of the output.
// The per-CTA partials (m, l, o) are merged across the cluster through
// distributed shared memory -- no global scratch, no atomics, no second kernel.
//
// HBM traffic: the union of the group's selected K/V blocks
// (bs * D * sizeof(T) * 2 bytes per block) plus the selection bitmaps, q and out.
#include <cooperative_groups.h>

#include "kernels.h"

namespace adakv {

namespace cg = cooperative_groups;

constexpr int kAttendMaxThreads = 512;  // g <= 16 warps

__device__ __forceinline__ void cp_async_wait_one() {
  asm volatile("cp.async.wait_group 1;" ::: "memory");
}

// shared-memory carve-up of one attend CTA (host and device agree on it)
struct AttendSmem {
  size_t kv, hw, list, mask, part, total;
};

__host__ __device__ inline AttendSmem attend_smem_layout(int elt, int D, int BS, int nbt, int g,
                                                         int nw_max, int slice_cap) {
  auto al = [](size_t x) { return (x + 15) / 16 * 16; };
  AttendSmem s;
  s.kv = 0;
  s.hw = s.kv + al((size_t)2 * 2 * nbt * BS * D * elt);
  s.list = s.hw + al((size_t)g * nw_max * 4);
  s.mask = s.list + al((size_t)slice_cap * 4);
  s.part = s.mask + al((size_t)slice_cap * 4);
  s.total = s.part + al((size_t)(32 + g * D) * 4);
  return s;
}

template <typename T, int D, int BS>
__global__ void __launch_bounds__(kAttendMaxThreads) attend_kernel(AttendParams p) {
  constexpr int VEC = 16 / sizeof(T);       // elements per 16-byte chunk
  constexpr int LPT = D / VEC;              // lanes per token row
  constexpr int TPP = 32 / LPT;             // token rows per warp pass
  constexpr int PASSES = BS / TPP;
  constexpr int ROWC = D / VEC;             // 16-byte chunks per token row
  constexpr int BLK = BS * D;               // elements of one K (or V) block
  static_assert(LPT <= 32 && BS % TPP == 0, "unsupported tile shape");
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ int scan_scratch[33];

  cg::cluster_group cl = cg::this_cluster();
  const int rank = (int)cl.block_rank();
  const int CL = (int)cl.num_blocks();
  const int kvh = blockIdx.y, b = blockIdx.z;
  const int nthr = blockDim.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = p.g, NBT = p.nbt;
  const AttendSmem L = attend_smem_layout(sizeof(T), D, BS, NBT, g, p.nw_max, p.slice_cap);
  T* kbuf = reinterpret_cast<T*>(smem + L.kv);                 // [2][NBT][BS][D]
  T* vbuf = kbuf + (size_t)2 * NBT * BLK;
  uint32_t* hw = reinterpret_cast<uint32_t*>(smem + L.hw);     // [g][nw_max] head words
  int* list = reinterpret_cast<int*>(smem + L.list);           // [slice_cap] block ids
  uint32_t* lmask = reinterpret_cast<uint32_t*>(smem + L.mask);  // [slice_cap] head bits
  float* pm = reinterpret_cast<float*>(smem + L.part);         // [16] running max per head
  float* pl = pm + 16;                                         // [16] denominators
  float* po = pl + 16;                                         // [g][D] numerators

  pdl_wait();
  int S = seq_len_of(p.seq_lens, b, p.max_seq_len);
  if (S < 0 || S > p.max_seq_len) S = 0;
  const int nb = ceil_div(S, BS);
  const int nw = ceil_div(nb, 32);
  const int row0 = b * p.Hq + kvh * g;

  // ---- the group's selection bitmaps and their union ----
  for (int idx = tid; idx < g * nw; idx += nthr) {
    const int hh = idx / nw, w = idx - hh * nw;
    hw[hh * p.nw_max + w] = p.bitmap[(int64_t)(row0 + hh) * p.bm_words + w];
  }
  __syncthreads();
  auto uni = [&](int w) -> uint32_t {
    uint32_t u = 0;
    for (int hh = 0; hh < g; ++hh) u |= hw[hh * p.nw_max + w];
    return u;
  };
  const int wpt = ceil_div(nw, nthr);
  const int w0 = imin(tid * wpt, nw), w1 = imin(w0 + wpt, nw);
  int cnt = 0;
  for (int w = w0; w < w1; ++w) cnt += __popc(uni(w));
  const int before = block_exclusive_scan(cnt, scan_scratch);
  const int U = scan_scratch[32];
  const int lo = (int)((int64_t)U * rank / CL), hi = (int)((int64_t)U * (rank + 1) / CL);
  int rk = before;
  for (int w = w0; w < w1 && rk < hi; ++w) {
    uint32_t u = uni(w);
    while (u && rk < hi) {
      const int bit = __ffs(u) - 1;
      u &= u - 1u;
      if (rk >= lo) {
        uint32_t m = 0;
        for (int hh = 0; hh < g; ++hh) m |= ((hw[hh * p.nw_max + w] >> bit) & 1u) << hh;
        list[rk - lo] = w * 32 + bit;
        lmask[rk - lo] = m;
      }
      ++rk;
    }
  }
  __syncthreads();
  const int n = hi - lo;

  // ---- gather: double-buffered batches of NBT blocks ----
  const T* kbase = static_cast<const T*>(p.k.data) + b * p.k.sb + kvh * p.k.sh;
  const T* vbase = static_cast<const T*>(p.v.data) + b * p.v.sb + kvh * p.v.sh;
  auto issue = [&](int batch) {
    const int first = batch * NBT;
    const int cntb = imin(NBT, n - first);
    if (cntb > 0) {
      T* kd = kbuf + (size_t)(batch & 1) * NBT * BLK;
      T* vd = vbuf + (size_t)(batch & 1) * NBT * BLK;
      const int chunks = cntb * BS * ROWC;
      for (int c = tid; c < chunks; c += nthr) {
        const int slot = c / (BS * ROWC);
        const int rem = c - slot * (BS * ROWC);
        const int tok = rem / ROWC, col = rem - tok * ROWC;
        const int pos = list[first + slot] * BS + tok;
        const bool valid = pos < S;
        const int64_t srow = valid ? (int64_t)pos : 0;
        const size_t off = (size_t)slot * BLK + tok * D + col * VEC;
        cp_async16(kd + off, kbase + srow * p.k.ss + col * VEC, valid);
        cp_async16(vd + off, vbase + srow * p.v.ss + col * VEC, valid);
      }
    }
    cp_async_commit();
  };
  issue(0);
  issue(1);

  const int d0 = (lane % LPT) * VEC;
  const int tl = lane / LPT;
  float qf[VEC];
  {
    const uint4 u = *reinterpret_cast<const uint4*>(static_cast<const T*>(p.q.data) + b * p.q.sb +
                                                    (int64_t)(kvh * g + warp) * p.q.sh + d0);
    Unpack16<T>::run(u, qf);
  }
  float m_run = -INFINITY, l_run = 0.f;
  float o[VEC];
#pragma unroll
  for (int e = 0; e < VEC; ++e) o[e] = 0.f;

  const int nbatches = ceil_div(n, NBT);
  for (int bi = 0; bi < nbatches; ++bi) {
    cp_async_wait_one();
    __syncthreads();
    const T* kt = kbuf + (size_t)(bi & 1) * NBT * BLK;
    const T* vt = vbuf + (size_t)(bi & 1) * NBT * BLK;
    const int first = bi * NBT;
    const int cntb = imin(NBT, n - first);
    for (int slot = 0; slot < cntb; ++slot) {
      if (!((lmask[first + slot] >> warp) & 1u)) continue;  // warp-uniform
      const int blk = list[first + slot];
      float sc[PASSES];
#pragma unroll
      for (int pp = 0; pp < PASSES; ++pp) {
        const int tok = pp * TPP + tl;
        const uint4 u = *reinterpret_cast<const uint4*>(kt + (size_t)slot * BLK + tok * D + d0);
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
      if (m_new == -INFINITY) continue;
      const float alpha = expf(m_run - m_new);
      float l_part = 0.f;
#pragma unroll
      for (int e = 0; e < VEC; ++e) o[e] *= alpha;
#pragma unroll
      for (int pp = 0; pp < PASSES; ++pp) {
        const int tok = pp * TPP + tl;
        const float pt = expf(sc[pp] - m_new);
        l_part += pt;
        const uint4 u = *reinterpret_cast<const uint4*>(vt + (size_t)slot * BLK + tok * D + d0);
        float vf[VEC];
        Unpack16<T>::run(u, vf);
#pragma unroll
        for (int e = 0; e < VEC; ++e) o[e] = fmaf(pt, vf[e], o[e]);
      }
      l_run = l_run * alpha + l_part;
      m_run = m_new;
    }
    __syncthreads();  // the buffer is refilled next
    issue(bi + 2);
  }
  cp_async_wait_all();

  // ---- per-CTA partial of each head ----
#pragma unroll
  for (int off = LPT; off < 32; off <<= 1) {
    l_run += __shfl_xor_sync(0xffffffffu, l_run, off);
#pragma unroll
    for (int e = 0; e < VEC; ++e) o[e] += __shfl_xor_sync(0xffffffffu, o[e], off);
  }
  if (lane < LPT) {
#pragma unroll
    for (int e = 0; e < VEC; ++e) po[warp * D + d0 + e] = o[e];
  }
  if (lane == 0) {
    pm[warp] = m_run;
    pl[warp] = l_run;
  }
  cl.sync();

  // ---- cluster merge: CTA `rank` finalises heads rank, rank + CL, ... ----
  for (int hh = rank; hh < g; hh += CL) {
    float M = -INFINITY;
    for (int c = 0; c < CL; ++c) M = fmaxf(M, *cl.map_shared_rank(&pm[hh], c));
    T* orow = static_cast<T*>(const_cast<void*>(p.out.data)) + b * p.out.sb +
              (int64_t)(kvh * g + hh) * p.out.sh;
    for (int d = tid; d < D; d += nthr) {
      float Lsum = 0.f, O = 0.f;
      if (M != -INFINITY) {
        for (int c = 0; c < CL; ++c) {
          const float mc = *cl.map_shared_rank(&pm[hh], c);
          const float f = (mc == -INFINITY) ? 0.f : expf(mc - M);
          Lsum += *cl.map_shared_rank(&pl[hh], c) * f;
          O += *cl.map_shared_rank(&po[hh * D + d], c) * f;
        }
      }
      orow[d] = from_f32<T>(Lsum > 0.f ? O / Lsum : 0.f);
    }
  }
  cl.sync();  // keep this CTA's shared memory alive until every reader is done
  pdl_launch_dependents();
}

// Stand-alone attend: caller-given (block_table, sel_lens) -> per-head bitmaps.
// Duplicate ids collapse to one bit; ids outside [0, nb) are flagged and skipped.
__global__ void __launch_bounds__(256) table_bitmap_kernel(TableParams p) {
  extern __shared__ uint32_t sbits[];
  const int h = blockIdx.x, b = blockIdx.y, row = b * p.Hq + h;
  pdl_wait();
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
    const int blk = trow[i];
    if (blk < 0 || blk >= nb) {
      report(p.status, ADAKV_ST_BAD_BLOCK_ID);
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

size_t attend_smem_bytes(int dtype, int D, int bs, int nbt, int g, int nw_max, int slice_cap) {
  return attend_smem_layout(dtype == ADAKV_DTYPE_F32 ? 4 : 2, D, bs, nbt, g, nw_max, slice_cap).total;
}

cudaError_t attend_kernels_init() {
  for (int dt = 0; dt < 3; ++dt)
    for (int D : {64, 128})
      for (int bs : {16, 32}) {
        cudaError_t e = for_each_attend(dt, D, bs, [](auto kern, int) {
          cudaError_t r = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)kAttendSmemMax);
          if (r != cudaSuccess) return r;
          return cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        });
        if (e != cudaSuccess) return e;
      }
  return cudaFuncSetAttribute(table_bitmap_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              64 * 1024);
}

int attend_max_cluster(int dtype, int D, int bs, int g, size_t smem) {
  int best = 1;
  for_each_attend(dtype, D, bs, [&](auto kern, int) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(16, 1, 1);
    cfg.blockDim = dim3(32 * g, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 16;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    cudaError_t e = cudaOccupancyMaxPotentialClusterSize(&n, kern, &cfg);
    if (e == cudaSuccess && n > 0) best = n;
    return e;
  });
  int c = 1;
  while (c * 2 <= best && c * 2 <= 16) c *= 2;
  return c;
}

cudaError_t launch_attend(const AttendParams& p, int dtype, int D, int bs, int cluster,
                          cudaStream_t st, const LaunchOpts& o) {
  const size_t smem = attend_smem_bytes(dtype, D, bs, p.nbt, p.g, p.nw_max, p.slice_cap);
  LaunchOpts oc = o;
  oc.cluster_x = (unsigned)cluster;
  return for_each_attend(dtype, D, bs, [&](auto kern, int) {
    return launch_ex(kern, dim3(cluster, p.Hkv, p.B), dim3(32 * p.g), smem, st, oc, p);
  });
}

cudaError_t launch_table_bitmap(const TableParams& p, cudaStream_t st, const LaunchOpts& o) {
  const int nw_max = ceil_div(ceil_div(p.max_seq_len, p.bs), 32);
  return launch_ex(table_bitmap_kernel, dim3(p.Hq, p.B), dim3(256), (size_t)nw_max * 4, st, o, p);
}

}  // namespace adakv
