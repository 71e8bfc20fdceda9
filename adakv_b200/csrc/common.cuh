// Shared device helpers and launch-parameter structs for the AdaKV decode path.
//
// Everything here is sm_100a-only device code or host/device arithmetic that
// both the launchers and the kernels need (per-sequence budget bounds, the
// workspace layout).  No torch types appear anywhere in this library.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/adakv_b200.h"

namespace adakv {

// ---------------------------------------------------------------------------
// constants
// ---------------------------------------------------------------------------
constexpr int kEstRows = 64;          // centroid rows (blocks) per estimator chunk
constexpr uint64_t kWaitLimitNs = 200ull * 1000ull * 1000ull;  // bounded spin: 200 ms

// ---------------------------------------------------------------------------
// parameter structs (host -> device by value)
// ---------------------------------------------------------------------------
struct View {          // [B, H, S, D] view, D contiguous
  const void* data;
  int64_t sb, sh, ss;  // element strides
};

struct SelectCfg {
  double avg_budget;
  double temperature;
  int k_min, k_max, n_sink, n_local, c_min, policy;
  double nucleus_p;
};

__host__ __device__ inline int ceil_div(int a, int b) { return (a + b - 1) / b; }
__host__ __device__ inline int imin(int a, int b) { return a < b ? a : b; }
__host__ __device__ inline int imax(int a, int b) { return a > b ? a : b; }

// Per-sequence budget bounds, exactly as the reference derives them:
// reference.py:71-73 passes min(k_min, nb), min(k_max, nb) and
// floor = min(sink, nb) + min(local, nb) + c_min; budget.py:75-77 then sets
// lo = min(max(floor, k_min, 1), nb), hi = min(k_max, nb),
// target = clip(avg, lo, hi); selector.py:41-49 clamps each head to
// [min(sink + local + c_min, nb), nb].
struct SeqBudget {
  int nb, sink, local, floor_sel, lo, hi;
  double target;
};

__host__ __device__ inline SeqBudget seq_budget(int nb, const SelectCfg& c) {
  SeqBudget r;
  r.nb = nb;
  r.sink = imin(c.n_sink, nb);
  r.local = imin(c.n_local, nb);
  r.floor_sel = imin(r.sink + r.local + c.c_min, nb);
  const int floor_b = r.sink + r.local + c.c_min;
  r.lo = imin(imax(imax(floor_b, imin(c.k_min, nb)), 1), nb);
  r.hi = imin(imin(c.k_max, nb), nb);
  double t = c.avg_budget;
  t = t < (double)r.lo ? (double)r.lo : t;   // np.clip = min(max(x, lo), hi)
  t = t > (double)r.hi ? (double)r.hi : t;
  r.target = t;
  return r;
}

// Realised selected-block count of one head (budget.py:45-86 + selector.py:53-54).
// `w` is the head's entropy weight, `sum_w` the sequence's sum over heads.
__host__ __device__ inline int head_count(const SeqBudget& s, const SelectCfg& c, double w,
                                          double sum_w, int n_heads) {
  const int nb = s.nb;
  if (nb <= 0) return 0;
  double k;
  if (nb <= 1) {
    k = (double)imin(imax(imin(c.k_min, nb), 1), nb);
  } else if (c.policy == ADAKV_POLICY_FIXED) {
    k = rint(s.target);
  } else {
    const double surplus = (s.target - s.lo > 0.0 ? s.target - s.lo : 0.0) * (double)n_heads;
    const double extra = surplus * w / (sum_w > 1e-9 ? sum_w : 1e-9);
    double x = rint((double)s.lo + extra);
    x = x < (double)s.lo ? (double)s.lo : x;
    x = x > (double)s.hi ? (double)s.hi : x;
    k = x;
  }
  long long kk = (long long)k;
  if (kk < s.floor_sel) kk = s.floor_sel;
  if (kk > nb) kk = nb;
  return (int)kk;
}

// Largest per-head count any sequence of this geometry can produce.
inline int table_width_for(int nb_cap, const SelectCfg& c) {
  int w = imax(imax(c.k_max, c.n_sink + c.n_local + imax(c.c_min, 0)), 1);
  return imin(w, imax(nb_cap, 1));
}

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// ---------------------------------------------------------------------------
// device helpers
// ---------------------------------------------------------------------------
#ifdef __CUDACC__

// (the memory clobber keeps the read in place relative to barriers and memory
// operations, so timestamps and time limits measure what they bracket)
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t) : : "memory");
  return t;
}

// order-preserving float -> uint32 map; NaN sorts below everything
__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return 0u;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Status words live at the start of a workspace (16 bytes reserved): bytes
// 0..3 collect the ADAKV_ST_* bits, bytes 8..15 optionally hold the device
// address of a host-mapped word (adakv_set_status_sink) that is written on
// every report, so that a host can see a failure without synchronising.
__device__ __forceinline__ void report(uint32_t* status, uint32_t bits) {
  if (status) {
    atomicOr(status, bits);
    uint32_t* sink = *reinterpret_cast<uint32_t* volatile*>(reinterpret_cast<char*>(status) + 8);
    if (sink) asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(sink), "r"(bits) : "memory");
  }
}

// --- tagged 64-bit words (call tag << 32 | 32-bit payload) ------------------
// A word written whole with one 64-bit store is read whole by one 64-bit
// load, so a reader that sees this call's tag also sees this call's payload;
// words of earlier calls carry older tags.  No counter has to be reset.
__device__ __forceinline__ unsigned long long tword(uint32_t tag, uint32_t bits) {
  return (static_cast<unsigned long long>(tag) << 32) | bits;
}
__device__ __forceinline__ bool tag_is(unsigned long long w, uint32_t tag) {
  return static_cast<uint32_t>(w >> 32) == tag;
}
__device__ __forceinline__ unsigned long long ldr_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void ldr_u64x2(const unsigned long long* p, unsigned long long& a,
                                          unsigned long long& b) {
  asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ void str_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

// One thread's bounded wait budget for a phase: the first wait starts the
// clock; once `limit` ns have passed the thread stops waiting (`dead`) and
// uses whatever it reads, and the caller reports ADAKV_ST_WAIT_TIMEOUT.
struct PollBudget {
  uint64_t limit;
  uint64_t t0;
  bool dead;
};

// Words w[i] (i < n) of base[i * stride], first read already in w: re-read
// every word that does not carry `tag` yet, all of a round's loads in flight
// together, until each one does or the budget runs out.  One round trip
// after the last word lands, however many words were late.
template <int N>
__device__ __forceinline__ void wait_tagged_n(const unsigned long long* base, size_t stride,
                                              unsigned long long (&w)[N], int n, uint32_t tag,
                                              PollBudget& pb) {
  while (!pb.dead) {
    bool all = true;
#pragma unroll
    for (int i = 0; i < N; ++i)
      if (i < n && !tag_is(w[i], tag)) all = false;
    if (all) return;
    const uint64_t now = globaltimer_ns();
    if (pb.t0 == 0) {
      pb.t0 = now;
    } else if (now - pb.t0 > pb.limit) {
      pb.dead = true;
      return;
    }
#pragma unroll
    for (int i = 0; i < N; ++i)
      if (i < n && !tag_is(w[i], tag)) w[i] = ldr_u64(base + i * stride);
  }
}

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_add_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Re-read *p until its tag is `tag` (w = the first read), within the budget.
__device__ __forceinline__ unsigned long long wait_tagged(const unsigned long long* p,
                                                          unsigned long long w, uint32_t tag,
                                                          PollBudget& pb) {
  if (tag_is(w, tag) || pb.dead) return w;
  if (pb.t0 == 0) pb.t0 = globaltimer_ns();
  while (true) {
    w = ldr_u64(p);
    if (tag_is(w, tag)) return w;
    if (globaltimer_ns() - pb.t0 > pb.limit) {
      pb.dead = true;
      return w;
    }
  }
}

__device__ __forceinline__ int seq_len_of(const int* seq_lens, int b, int max_seq_len) {
  return seq_lens ? seq_lens[b] : max_seq_len;
}

// fp32 <- one element
__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

// Unpack one 16-byte word holding 16/sizeof(T) elements of T into fp32.
template <typename T> struct Unpack16;
template <> struct Unpack16<float> {
  static constexpr int N = 4;
  __device__ __forceinline__ static void run(const uint4& u, float* f) {
    f[0] = __uint_as_float(u.x); f[1] = __uint_as_float(u.y);
    f[2] = __uint_as_float(u.z); f[3] = __uint_as_float(u.w);
  }
};
template <> struct Unpack16<__nv_bfloat16> {
  static constexpr int N = 8;
  __device__ __forceinline__ static void run(const uint4& u, float* f) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
  }
};
template <> struct Unpack16<__half> {
  static constexpr int N = 8;
  __device__ __forceinline__ static void run(const uint4& u, float* f) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
      float2 v = __half22float2(h);
      f[2 * i] = v.x;
      f[2 * i + 1] = v.y;
    }
  }
};

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// --- mbarrier + 1-D bulk copy (TMA engine, one CTA per copy) ---------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase; false after kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
  }
  return true;
}

// Global -> shared bulk copy completing on `bar` (addresses 16-B aligned,
// bytes a multiple of 16).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// --- cp.async (16 B, zero-fill when !valid) --------------------------------
__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  const uint32_t n = valid ? 16u : 0u;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src),
               "r"(n)
               : "memory");
}
// the first `bytes` (0..16) of 16 B; the rest of the destination zero-filled
__device__ __forceinline__ void cp_async16_n(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// named barrier among `count` threads (a multiple of 32) of the CTA
__device__ __forceinline__ void named_bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// --- programmatic dependent launch ------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// --- reductions -------------------------------------------------------------
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Butterfly reduce-scatter of 32 per-lane partial values: afterwards lane l
// holds the warp-wide sum of slot l in v[0] (31 shuffles for 32 sums).
__device__ __forceinline__ float warp_reduce_scatter32(float (&v)[32], int lane) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < off; ++i) {
      const float send = upper ? v[i] : v[i + off];
      const float keep = upper ? v[i + off] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
  return v[0];
}

// Exclusive block-wide prefix sum of one int per thread (blockDim multiple of 32).
// `scratch` needs 33 ints of shared memory.  Returns the exclusive prefix; the
// block total is left in scratch[32].
__device__ __forceinline__ int block_exclusive_scan(int v, int* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) scratch[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int t = lane < nwarps ? scratch[lane] : 0;
    int s = t;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    if (lane < nwarps) scratch[lane] = s - t;  // exclusive warp offsets
    if (lane == 31) scratch[32] = s;
  }
  __syncthreads();
  const int res = scratch[warp] + x - v;
  __syncthreads();
  return res;
}

#endif  // __CUDACC__

}  // namespace adakv
