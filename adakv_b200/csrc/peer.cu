// All-gather of small per-rank payloads between the GPUs of one node through
// peer-mapped memory (CUDA IPC over NVLink / NVSwitch).  It stands in for an
// NCCL all-gather whose fixed cost (about 11 us per call inside a CUDA graph
// on two B200s, measured) dominates the sequence-sharded decode step, whose
// exchanges are 0.5 KB - 0.5 MB.
//
// Each rank owns one exchange buffer (peer_layout): `world` slots of
// slot_bytes, then world * kPeerChunks 64-bit flag words, then one 64-bit
// tag word.  A put copies this rank's payload into slot `rank` of every
// rank's buffer (its own included), kPeerChunks chunks per destination, one
// CTA each: the CTA's stores, a CTA barrier, then thread 0's system-scope
// fence and one store of the call tag into the destination's flag word
// (rank, chunk).  A wait polls the local buffer's flag words until every one
// carries the tag or a later one (bounded by a wall-clock limit; on expiry it
// reports ADAKV_ST_WAIT_TIMEOUT and returns), fences, then advances the
// local tag.  The tag counts the completed exchanges on this buffer, which
// is the same number on every rank, so flag words are never cleared.  A rank
// may post its next payload before a slower rank has read the previous one
// only if the caller lets it: a payload must have been consumed everywhere
// before the next exchange on that buffer starts (in the sharded decode
// step, each exchange depends on the previous one, so it has).  Measured on
// two B200s inside a CUDA graph: 9.5 us for 512 B and 11.0 us for 514 KB per
// rank, against 12.4 and 19.6 us for an NCCL all-gather.
//
// Puts only ever write remote memory and waits only read local memory; no
// kernel waits on another kernel of the same GPU.
#include "kernels.h"

namespace adakv {

namespace {

__device__ __forceinline__ unsigned long long* peer_flags(unsigned char* buf, int world,
                                                          size_t slot_bytes) {
  return reinterpret_cast<unsigned long long*>(buf + (size_t)world * slot_bytes);
}
__device__ __forceinline__ unsigned long long* peer_tag(unsigned char* buf, int world,
                                                        size_t slot_bytes) {
  return peer_flags(buf, world, slot_bytes) + (size_t)world * kPeerChunks;
}

__global__ void __launch_bounds__(kPeerThreads) peer_put_kernel(PeerParams p) {
  const int c = blockIdx.x, d = blockIdx.y, tid = threadIdx.x;
  pdl_wait();  // the payload comes from the previous kernel
  const unsigned long long tag = *peer_tag(p.local, p.world, p.slot_bytes) + 1ull;
  const size_t n16 = p.bytes / 16;
  const size_t per = (n16 + kPeerChunks - 1) / kPeerChunks;
  const size_t a = (size_t)c * per, b = a + per < n16 ? a + per : n16;
  const uint4* src = reinterpret_cast<const uint4*>(p.src);
  unsigned char* dbuf = p.dsts[d];
  uint4* dst = reinterpret_cast<uint4*>(dbuf + (size_t)p.rank * p.slot_bytes);
  for (size_t i = a + tid; i < b; i += kPeerThreads) dst[i] = src[i];
  __syncthreads();  // the CTA's stores are ordered before thread 0's fence (cumulative)
  if (tid == 0) {
    unsigned long long* f = peer_flags(dbuf, p.world, p.slot_bytes) + (size_t)p.rank * kPeerChunks + c;
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(f), "l"(tag) : "memory");
  }
  pdl_launch_dependents();
}

__global__ void __launch_bounds__(kPeerThreads) peer_wait_kernel(PeerParams p) {
  __shared__ int s_late;
  const int tid = threadIdx.x;
  pdl_wait();
  unsigned long long* tagp = peer_tag(p.local, p.world, p.slot_bytes);
  const unsigned long long tag = *tagp + 1ull;
  const unsigned long long* flags = peer_flags(p.local, p.world, p.slot_bytes);
  if (tid == 0) s_late = 0;
  __syncthreads();
  const int n = p.world * kPeerChunks;
  const uint64_t t0 = globaltimer_ns();
  for (int i = tid; i < n; i += kPeerThreads) {
    while (true) {
      unsigned long long v;
      asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(flags + i) : "memory");
      if (v >= tag) break;  // a faster rank's next tag counts too
      if (globaltimer_ns() - t0 > p.wait_ns) {
        s_late = 1;
        break;
      }
    }
  }
  asm volatile("fence.acq_rel.sys;" ::: "memory");  // the payloads are read after this
  __syncthreads();
  if (tid == 0) {
    if (s_late) report(p.status, ADAKV_ST_WAIT_TIMEOUT);
    *tagp = tag;
  }
  pdl_launch_dependents();
}

}  // namespace

size_t peer_buffer_bytes(int world, size_t slot_bytes) {
  return (size_t)world * slot_bytes + ((size_t)world * kPeerChunks + 2) * sizeof(unsigned long long);
}

cudaError_t launch_peer_put(const PeerParams& p, cudaStream_t st, const LaunchOpts& o) {
  return launch_ex(peer_put_kernel, dim3(kPeerChunks, p.world), dim3(kPeerThreads), 0, st, o, p);
}

cudaError_t launch_peer_wait(const PeerParams& p, cudaStream_t st, const LaunchOpts& o) {
  return launch_ex(peer_wait_kernel, dim3(1), dim3(kPeerThreads), 0, st, o, p);
}

}  // namespace adakv
