// Tensor-core (mma.sync m16n8k16, bf16/fp16 in, fp32 accumulate) attention of
// the g query heads of one KV group over one 16- or 32-token K/V block.
//
// The g query rows form the M = 16 rows of the MMA (rows >= g are zero and
// masked); tokens are N for q.K^T and K for P.V.  K/V tiles sit in shared
// memory as [token][D] rows of 16-byte chunks, chunk c of token t stored at
// c ^ (t & 7) so that ldmatrix (K) and ldmatrix.trans (V) read 8 rows without
// bank conflicts.  The q.K^T accumulators are reused in registers as the
// A operand of P.V (FlashAttention-2 register layout), with the probabilities
// rounded to the input type.
#pragma once

#include "common.cuh"

namespace adakv {

template <typename T> struct MmaType;
template <> struct MmaType<__nv_bfloat16> {
  static constexpr const char* name = "bf16";
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
  }
};
template <> struct MmaType<__half> {
  static constexpr const char* name = "f16";
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    const __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
  }
};

template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  if constexpr (sizeof(T) == 2 && std::is_same<T, __nv_bfloat16>::value) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// byte offset of 16-byte chunk `chunk` of token row `tok` in a swizzled tile
template <int D, typename T>
__device__ __forceinline__ uint32_t swz_off(int tok, int chunk) {
  constexpr int ROW = D * (int)sizeof(T);
  return (uint32_t)(tok * ROW + ((chunk ^ (tok & 7)) << 4));
}

// Per-warp online-softmax state for the 16 MMA rows this lane touches
// (rows gid and gid + 8), and the output accumulators for all D columns.
template <int D>
struct MmaAcc {
  static constexpr int NT = D / 8;  // output n-tiles
  float o[NT][4];
  float m[2], l[2];
};

// One K/V block (BS tokens) for all query rows of the group.
//   qa:     A fragments of q, [D/16][4] (rows >= g are zero)
//   ktile:  shared address of the swizzled K block, vtile likewise
//   rowok:  bit r set = query row r takes part for this block
//   tok_valid: number of tokens of the block below seq_len
template <typename T, int D, int BS>
__device__ __forceinline__ void mma_block(MmaAcc<D>& acc, const uint32_t (&qa)[D / 16][4],
                                          uint32_t ktile, uint32_t vtile, uint32_t rowok,
                                          int tok_valid, float scale_log2, int lane) {
  constexpr int KS = D / 16;   // k-steps of q.K^T
  constexpr int NTS = BS / 8;  // token n-tiles of S
  const int gid = lane >> 2, tig = lane & 3;
  float s[NTS][4];
#pragma unroll
  for (int j = 0; j < NTS; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) s[j][e] = 0.f;
  // S = q K^T: one ldmatrix.x4 gives both b-fragments of two token n-tiles
#pragma unroll
  for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
    for (int jp = 0; jp < NTS; jp += 2) {
      const int mi = lane >> 3, r = lane & 7;
      const int tok = (jp + (mi >> 1)) * 8 + r;
      const int chunk = ks * 2 + (mi & 1);
      uint32_t b[4];
      ldsm_x4(b, ktile + swz_off<D, T>(tok, chunk));
      mma16816<T>(s[jp], qa[ks], b[0], b[1]);
      mma16816<T>(s[jp + 1], qa[ks], b[2], b[3]);
    }
  }
  // mask: rows not selecting this block, padding rows, tokens past seq_len
  const bool r0ok = (rowok >> gid) & 1u, r1ok = (rowok >> (gid + 8)) & 1u;
  float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
  for (int j = 0; j < NTS; ++j) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int t = j * 8 + tig * 2 + e;
      const bool tv = t < tok_valid;
      s[j][e] = (r0ok && tv) ? s[j][e] * scale_log2 : -INFINITY;
      s[j][2 + e] = (r1ok && tv) ? s[j][2 + e] * scale_log2 : -INFINITY;
      mx0 = fmaxf(mx0, s[j][e]);
      mx1 = fmaxf(mx1, s[j][2 + e]);
    }
  }
  mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
  mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
  mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
  mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
  const float mn0 = fmaxf(acc.m[0], mx0), mn1 = fmaxf(acc.m[1], mx1);
  // scores are pre-multiplied by log2(e): exp(x) == exp2(x * log2(e))
  const float al0 = (mn0 == -INFINITY) ? 1.f : exp2f(acc.m[0] - mn0);
  const float al1 = (mn1 == -INFINITY) ? 1.f : exp2f(acc.m[1] - mn1);
  float ls0 = 0.f, ls1 = 0.f;
  uint32_t pa[NTS / 2][4];
#pragma unroll
  for (int j = 0; j < NTS; ++j) {
    float p[4];
    p[0] = (mn0 == -INFINITY) ? 0.f : exp2f(s[j][0] - mn0);
    p[1] = (mn0 == -INFINITY) ? 0.f : exp2f(s[j][1] - mn0);
    p[2] = (mn1 == -INFINITY) ? 0.f : exp2f(s[j][2] - mn1);
    p[3] = (mn1 == -INFINITY) ? 0.f : exp2f(s[j][3] - mn1);
    ls0 += p[0] + p[1];
    ls1 += p[2] + p[3];
    // accumulator (n-tile j) -> A fragment of P.V (k-step j / 2)
    pa[j >> 1][(j & 1) * 2 + 0] = MmaType<T>::pack(p[0], p[1]);
    pa[j >> 1][(j & 1) * 2 + 1] = MmaType<T>::pack(p[2], p[3]);
  }
  acc.m[0] = mn0;
  acc.m[1] = mn1;
  acc.l[0] = acc.l[0] * al0 + ls0;
  acc.l[1] = acc.l[1] * al1 + ls1;
#pragma unroll
  for (int n = 0; n < MmaAcc<D>::NT; ++n) {
    acc.o[n][0] *= al0;
    acc.o[n][1] *= al0;
    acc.o[n][2] *= al1;
    acc.o[n][3] *= al1;
  }
  // O += P V: ldmatrix.trans gives the b-fragments of two output n-tiles
#pragma unroll
  for (int kt = 0; kt < BS / 16; ++kt) {
#pragma unroll
    for (int np = 0; np < MmaAcc<D>::NT; np += 2) {
      const int mi = lane >> 3, r = lane & 7;
      const int tok = kt * 16 + (mi & 1) * 8 + r;
      const int chunk = np + (mi >> 1);
      uint32_t b[4];
      ldsm_x4_trans(b, vtile + swz_off<D, T>(tok, chunk));
      mma16816<T>(acc.o[np], pa[kt], b[0], b[1]);
      mma16816<T>(acc.o[np + 1], pa[kt], b[2], b[3]);
    }
  }
}

}  // namespace adakv
