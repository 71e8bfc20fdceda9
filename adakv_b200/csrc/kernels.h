// Launch-parameter structs and launcher entry points shared by the kernel
// translation units and the C-ABI layer (capi.cu).
#pragma once

#include <utility>

#include "common.cuh"

namespace adakv {

// ---------------------------------------------------------------------------
// (a) centroid build / append / refresh (stand-alone entry points)
// ---------------------------------------------------------------------------
struct CentroidParams {
  View k, v;            // caches [B, Hkv, S, D]
  View k_new, v_new;    // [B, Hkv, n_new, D] (append only)
  const int* seq_lens;  // length after append; NULL -> max_seq_len
  int max_seq_len;
  int B, Hkv, bs, nb_cap;
  int n_new;            // 0: build every block
  float* cent;          // [B, Hkv, nb_cap, D]
  uint32_t* status;
};

// weight-exchange slot of one (sequence, query head) for the plan barrier:
// one 64-bit word, call tag in the high half (never 0 once written), the
// head's float32 entropy bits in the low half; written and read whole
struct __align__(8) PlanSlot {
  unsigned long long word;
};

// ---------------------------------------------------------------------------
// (b) estimator (+ fused append of the step's new tokens)
// ---------------------------------------------------------------------------
constexpr int kEstMaxStages = 8;       // TMA ring depth limit
constexpr int kStatF = 8;              // floats per softmax partial
constexpr size_t kEstSmemBudget = 200 * 1024;  // dynamic shared memory of one estimator CTA
constexpr int kEstConsumerWarps = 8;   // 8 warps x 8 rows = kEstRows
constexpr int kEstThreads = (kEstConsumerWarps + 2) * 32;  // + producer warp + refresh warp
constexpr int kEstMaxBatch = 2048;     // sequences per launch (per-sequence chunk prefix in smem)

struct EstParams {
  View q;                 // [B, Hq, D]
  float* cent;            // [B, Hkv, nb_cap, D]
  int nb_cap;
  const int* seq_lens;    // NULL -> max_seq_len
  int max_seq_len;
  int B, Hq, Hkv, g, bs;
  float* scores;          // [B, Hq, score_stride]
  int score_stride;
  uint32_t* epoch;        // incremented once per launch (per-call tag for the plan barrier)
  PlanSlot* slots;        // [B*Hq*kPlanSlotsPerRow] exchange slots: cleared here, before the plan
  uint32_t* counters;     // [B*Hkv] attend arrival counts: cleared here, before the attend
  // Per-(head, 64-block chunk, consumer warp) softmax partials for the plan
  // (nullable): stats[(row * stats_stride + chunk * 8 + warp) * 8 + {max s,
  // content max, content sum, content sum of squares, m = max z,
  // sum e^(z - m), sum e^(z - m) (z - m)}], z = s / temperature; the last
  // slot of a row holds the rows the fused append scored.
  float* stats;
  int stats_stride;
  int n_sink, n_local;    // forced blocks (excluded from the content statistics)
  float temperature;      // max(T, 1e-6) as float
  // fused append: n_new > 0 and k_new.data != NULL
  View k, v, k_new, v_new;
  int n_new;
  int stages;             // ring depth (estimate_stages)
  uint32_t* status;
};

// ---------------------------------------------------------------------------
// (c) plan: entropy budget + per-sequence weight exchange + top-k
// ---------------------------------------------------------------------------
constexpr int kPlanThreads = 512;
constexpr int kPlanSmemMaxKeys = 32 * 1024;   // slice staged in shared memory up to this many blocks
constexpr int kPlanMaxBlocks = 512 * 1024;    // longest sequence in blocks (bitmap words in smem)
constexpr size_t kPlanSmemMax = 184 * 1024;   // opt-in dynamic shared memory of one plan CTA
constexpr int kPlanMaxCluster = 8;            // CTAs splitting one head's score row
constexpr int kPlanSlotsPerRow = 2 * kPlanMaxCluster;  // exchange words per (sequence, head)

// shared-memory layout of one plan CTA for a cluster size and longest row
struct PlanLayout {
  int csize;       // CTAs per (sequence, head)
  int slice_cap;   // blocks per CTA (multiple of 32)
  bool smem_keys;  // slice staged in shared memory (else re-read from L2)
  size_t smem;     // dynamic shared memory bytes
};

struct PlanParams {
  const int* seq_lens;
  int max_seq_len;
  int B, Hq, bs;
  SelectCfg cfg;
  const float* scores;
  int score_stride;
  const uint32_t* epoch;
  PlanSlot* slots;          // [B*Hq*kPlanSlotsPerRow]
  int* sel_lens;            // [B*Hq] out
  int* block_table;         // [B*Hq, table_width] out, ascending block ids
  int table_width;
  const float* stats;       // estimator partials (EstParams::stats) or NULL
  int stats_stride;
  uint32_t* bitmap;         // [B*Hq, bm_words] out, bit j = block j selected
  int bm_words;
  int csize;                // CTAs of the cluster splitting each row
  int slice_cap;            // blocks per CTA (PlanLayout::slice_cap)
  int seqs_per_round;       // grid = seqs_per_round * Hq * csize CTAs
  uint32_t* status;
  uint64_t wait_ns;         // bound of the entropy exchange wait
  int debug_flags;          // test-only: bit 0 = head 0 never publishes its entropy
};

// ---------------------------------------------------------------------------
// (d) attend: one cluster per (sequence, KV head) over the union of the group's blocks
// ---------------------------------------------------------------------------
constexpr size_t kAttendSmemMax = 200 * 1024;  // opt-in dynamic shared memory of one attend CTA
constexpr int kAttendCtaTarget = 148;  // CTAs per launch the split-KV axis aims for (B200 SMs)
constexpr int kAttendMaxSplit = 64;    // CTAs per (sequence, KV head)
constexpr int kAttendMaxSlice = 8192;  // union blocks one CTA takes at most

struct AttendParams {
  View q, k, v, out;
  const int* seq_lens;
  int max_seq_len;
  int B, Hq, Hkv, g;
  float sm_scale;
  const uint32_t* bitmap;   // [B*Hq, bm_words]
  int bm_words;
  int nw_max;               // ceil(ceil(max_seq_len / bs) / 32)
  int slice_cap;            // >= union blocks one CTA can get
  int nbt;                  // blocks per stage of the two-stage gather ring
  float* part;              // [B*Hkv*split, g, D + 2] partials (m, l, o)
  uint32_t* counters;       // [B*Hkv] arrival counts (zero between calls)
  float* out_f32;           // optional [B*Hq, D] float32 output instead of `out`
  float* lse;               // optional [B*Hq] natural-log sum of exp of the scaled scores
  uint32_t* status;
};

struct CombineParams {      // log-sum-exp merge of per-shard attention outputs
  const float* parts;       // part n: parts + n * part_stride, [rows, D]
  const float* lse;         // part n: lse + n * lse_stride, [rows]
  int64_t part_stride, lse_stride;
  int n_parts, rows, D;
  View out;                 // rows = b * Hq + h -> out[b, h, :]
  int Hq;
};

struct ImportanceParams {   // H2O / SnapKV per-key attention importance (importance.cu)
  View q, k;                // [B, Hq, S, D] prompt queries, [B, Hkv, S, D] keys
  int B, Hq, Hkv, S;
  int n_query;              // the last n_query query rows attend (S: H2O, the window: SnapKV)
  float scale;
  float* row_m;             // [B, Hq, n_query] row max of the scaled logits (workspace)
  float* row_l;             // [B, Hq, n_query] row sum of exp(logit - max) (workspace)
  float* imp;               // [B * Hq, imp_stride] float32 out
  int imp_stride;
};

// ---------------------------------------------------------------------------
// (a)-(d) one decode step in one persistent kernel (step.cu)
// ---------------------------------------------------------------------------
constexpr int kStepThreads = 256;       // 8 warps: estimator consumers, selection, MMA attend
constexpr int kStepRows = 64;           // centroid rows per estimator ring stage
constexpr int kStepStages = 6;          // estimator ring depth
constexpr int kStepMaxDesc = 192;       // ring stages one CTA streams at most
constexpr int kStepMaxBatch = 32;       // sequences per call
constexpr int kStepMaxHeads = 128;      // B * Hq (one selection CTA per query head)
constexpr int kStepMaxBlocks = 32768;   // blocks per sequence (the score row is staged in smem)
constexpr int kStepMaxGrid = 256;       // CTAs (one per SM)
constexpr int kStepCandCap = 1024;      // boundary-bucket members ranked exactly
constexpr size_t kStepSmemMax = 220 * 1024;

struct StepParams {
  View q, k, v, out, k_new, v_new;
  float* cent;                 // [B, Hkv, nb_cap, D] float32
  int nb_cap;
  const int* seq_lens;
  int max_seq_len;
  int B, Hq, Hkv, bs;
  int n_new;                   // tokens appended by this step (0: none)
  SelectCfg cfg;
  float sm_scale;
  int* block_table;            // [B*Hq, table_width] out, ascending block ids
  int table_width;
  int* sel_lens;               // [B*Hq] out
  float* lse;                  // optional [B*Hq]
  // workspace (tagged words: call tag << 32 | payload)
  uint32_t* status;
  uint32_t* epoch;             // [0] calls completed, [1] CTAs done in this call
  unsigned long long* arrive;  // CTAs past the estimator phase, over all calls (monotonic)
  float* scores;               // [B*Hq, fs_stride] block scores (plain floats)
  int fs_stride;
  float* piece;                // [(B*Hkv + grid) * g, 8] score statistics (SoftPart) of the
                               // rows one CTA scored for one (sequence, KV head), per head
  unsigned long long* hslot;   // [B*Hq] entropy of each head (tagged)
  uint32_t* bitmap;            // [B*Hq, fb_stride] selection bitmaps
  int fb_stride;
  unsigned long long* ready;   // [B*Hq, csize] a cluster rank's bitmap words are out (tagged, release)
  float* part;                 // [grid, g, D + 2] attention partials (m, l, o) per CTA
  unsigned long long* pready;  // [grid] a CTA's partial is complete (tagged, release)
  int csize;                   // CTAs (one cluster) per query head in the selection phase
  int nbt;                     // K/V blocks per gather stage
  int slice_cap;               // union blocks one attend CTA takes at most
  int nb_max;                  // ceil(max_seq_len / bs)
  uint64_t wait_ns;            // bound of every device-side wait
  int debug_flags;             // test-only: bit 0 = head 0 never publishes its entropy,
                               // bit 1 = record per-CTA phase timestamps in `timeline`
  unsigned long long* timeline;  // [grid, kStepTimelineSlots] globaltimer stamps (debug)
};
constexpr int kStepTimelineSlots = 24;

// (b') minmax (Quest) estimator: tables and scores
struct MinmaxParams {
  View k, q;
  const int* seq_lens;
  int max_seq_len;
  int B, Hq, Hkv, g, bs, nb_cap;
  int n_new;                // build: 0 (every block); refresh: blocks touched by the last n_new tokens
  float* kmin;              // [B, Hkv, nb_cap, D] float32
  float* kmax;
  float* scores;            // [B*Hq, score_stride] (score kernel)
  int score_stride;
};

struct TableParams {        // block table -> per-head bitmaps (stand-alone attend)
  const int* block_table;
  int table_width;
  const int* sel_lens;
  const int* seq_lens;
  int max_seq_len;
  int B, Hq, bs;
  uint32_t* bitmap;
  int bm_words;
  uint32_t* counters;       // [ncounters] attend arrival counts: cleared here, before the attend
  int ncounters;
  int block_offset;         // table ids are global; this cache holds blocks from here on
  int local_only;           // 1: ids outside [block_offset, block_offset + nb) are skipped silently
  uint32_t* status;
};

// ---------------------------------------------------------------------------
// sequence-sharded selection from exchanged statistics (shard_select.cu)
// ---------------------------------------------------------------------------
constexpr int kShardThreads = 1024;
constexpr int kShardListCap = 4096;     // candidates one shard keeps per head at most
constexpr int kShardStageCap = 32768;   // score-row floats staged in shared memory
constexpr int kShardSortBuckets = 2048; // counting-sort buckets of the candidate keys
constexpr int kShardStatD = 8;          // doubles of one head's statistics record
constexpr int kShardFinishThreads = 512;
constexpr int kShardFinishStage = 160 * 1024;       // candidate lists staged in shared memory up to
constexpr size_t kShardFinishSmemMax = 200 * 1024;  // opt-in dynamic shared memory of a finish CTA
constexpr int kShardMaxWorld = 64;

// One rank's exchange record: Hq statistics records of kShardStatD doubles
// (max score, content max, content sum, content sum of squares, max z,
// Z = sum e^(z - max z), A = sum e^(z - max z) (z - max z), candidates kept),
// then Hq candidate lists of cap_pad 64-bit keys (order key of the score << 32
// | ~global block id), sorted descending.
struct ShardSelParams {
  const float* scores;        // [Hq, score_stride] this shard's score rows
  int score_stride;
  int n_local, block_lo;      // blocks of this shard and its first global block
  int nb;                     // blocks of the whole sequence
  int Hq;
  SelectCfg cfg;
  int cap, cap_pad;           // candidates per head at most, list stride
  size_t xstride;             // bytes between ranks' exchange records in xall
  int world, rank;
  unsigned char* xmine;       // this rank's exchange record (prep writes it)
  const unsigned char* xall;  // [world] exchange records in rank order
  double* cc_mine;            // [Hq] this shard's clamp term (clamp writes it)
  const double* cc_all;       // [world, Hq] every shard's clamp term (NULL: none)
  int table_width;            // the whole sequence's per-head count cap
  int* block_table;           // [Hq, out_width] this rank's selected global block ids
  int out_width;
  int* sel_lens;              // [Hq]
  uint32_t* status;
};

// ---------------------------------------------------------------------------
// all-gather of small payloads through peer-mapped memory (peer.cu)
// ---------------------------------------------------------------------------
constexpr int kPeerChunks = 16;    // CTAs (and flag words) per (source, destination)
constexpr int kPeerThreads = 256;
constexpr int kPeerMaxWorld = 16;

struct PeerParams {
  const void* src;                 // this rank's payload (16-byte aligned)
  size_t bytes;                    // payload bytes, a multiple of 16, <= slot_bytes
  int world, rank;
  unsigned char* const* dsts;      // device array [world]: every rank's buffer, mapped here
  size_t slot_bytes;               // a multiple of 16
  unsigned char* local;            // this rank's buffer
  uint32_t* status;                // optional ADAKV_ST_* word
  uint64_t wait_ns;                // bound of the wait
};

// ---------------------------------------------------------------------------
// launch helper: cudaLaunchKernelEx with optional PDL / cooperative / cluster
// ---------------------------------------------------------------------------
struct LaunchOpts {
  bool pdl = false;         // programmatic dependent launch on the previous kernel
  bool coop = false;        // all CTAs co-resident (they wait on one another)
  unsigned cluster_x = 0;   // thread-block cluster size along x (0: none)
};

template <typename... KArgs, typename... Args>
inline cudaError_t launch_ex(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                             cudaStream_t st, const LaunchOpts& o, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[3];
  unsigned n = 0;
  if (o.pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (o.coop) {
    attr[n].id = cudaLaunchAttributeCooperative;
    attr[n].val.cooperative = 1;
    ++n;
  }
  if (o.cluster_x) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = o.cluster_x;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// ---------------------------------------------------------------------------
// launchers (one per translation unit)
// ---------------------------------------------------------------------------
cudaError_t launch_centroid(const CentroidParams& p, int dtype, int D, int blocks_per_seq,
                            cudaStream_t stream);
cudaError_t launch_estimate(const EstParams& p, int dtype, int D, int nb_max, int grid,
                            cudaStream_t stream, const LaunchOpts& o);
cudaError_t launch_plan(const PlanParams& p, const PlanLayout& l, int grid, cudaStream_t stream,
                        const LaunchOpts& o);
cudaError_t launch_attend(const AttendParams& p, int dtype, int D, int bs, int split,
                          cudaStream_t stream, const LaunchOpts& o);
cudaError_t launch_table_bitmap(const TableParams& p, cudaStream_t stream, const LaunchOpts& o);
cudaError_t launch_minmax_build(const MinmaxParams& p, int dtype, int D, int blocks_per_seq,
                                cudaStream_t stream);
cudaError_t launch_minmax_score(const MinmaxParams& p, int dtype, int D, int nb_max,
                                cudaStream_t stream);
cudaError_t launch_combine(const CombineParams& p, int dtype, cudaStream_t stream, const LaunchOpts& o);
cudaError_t launch_importance(const ImportanceParams& p, int dtype, int D, cudaStream_t stream);
cudaError_t launch_stage(const void* src, void* dst, size_t bytes, cudaStream_t stream);
// sharded selection: stage 0 = statistics + candidates, 1 = clamp term, 2 = budgets + table
cudaError_t launch_shard_select(int stage, const ShardSelParams& p, cudaStream_t stream,
                                const LaunchOpts& o);
size_t shard_finish_smem(int Hq, int world, int cap_pad);
cudaError_t shard_kernels_init();
size_t peer_buffer_bytes(int world, size_t slot_bytes);
cudaError_t launch_peer_put(const PeerParams& p, cudaStream_t stream, const LaunchOpts& o);
cudaError_t launch_peer_wait(const PeerParams& p, cudaStream_t stream, const LaunchOpts& o);
cudaError_t launch_step(const StepParams& p, int dtype, int D, int g, int grid, size_t smem,
                        cudaStream_t stream, const LaunchOpts& o);
cudaError_t launch_step_scores(bool fused, const float* fscores,
                               int fs_stride, const float* scores, int score_stride, int rows,
                               int nb, float* out, int out_stride, cudaStream_t stream);
cudaError_t step_kernels_init();
// dynamic shared memory of the step kernel and its gather-ring depth
size_t step_smem_bytes(int D, int g, int nb_max, int min_split, int csize, int* nbt, int* slice_cap);
// clusters of `csize` step CTAs with `smem` bytes that can be resident at once
int step_active_clusters(int dtype, int D, int g, int csize, size_t smem);
bool step_kernel_built(int dtype, int D, int bs, int g);

// once per device (current device): opt-in shared memory / cluster sizes
cudaError_t estimate_kernels_init();
cudaError_t plan_kernels_init();
cudaError_t attend_kernels_init();
size_t estimate_smem_bytes(int dtype, int D, int g, int B);
int estimate_stages(int dtype, int D, int g, int B);
PlanLayout plan_layout(int nb_max, int csize);
// clusters of the plan kernel with layout `l` that can be resident at once
int plan_active_clusters(const PlanLayout& l, bool nucleus);
size_t attend_smem_bytes(int dtype, int D, int bs, int nbt, int g, int nw_max, int slice_cap,
                         int split);

#ifdef __CUDACC__
// Softmax partial of a set of blocks of one query head: max score, content
// max / sum / sum of squares (sink and local blocks excluded), and
// (m, Z, A) = (max z, sum e^(z - m), sum e^(z - m) (z - m)), z = s / T.
struct SoftPart {
  float mx, cmx, cs, cq, m, Z, A;
};

__device__ __forceinline__ SoftPart soft_empty() {
  return SoftPart{-INFINITY, -INFINITY, 0.f, 0.f, -INFINITY, 0.f, 0.f};
}

__device__ __forceinline__ void soft_add(SoftPart& a, float s, float z, bool content) {
  a.mx = fmaxf(a.mx, s);
  if (content) {
    a.cmx = fmaxf(a.cmx, s);
    a.cs += s;
    a.cq = fmaf(s, s, a.cq);
  }
  if (z > a.m) {
    const float f = a.m == -INFINITY ? 0.f : expf(a.m - z);
    a.A = f * fmaf(a.Z, a.m == -INFINITY ? 0.f : a.m - z, a.A);
    a.Z = fmaf(a.Z, f, 1.f);
    a.m = z;
  } else {
    const float e = expf(z - a.m);
    a.Z += e;
    a.A = fmaf(e, z - a.m, a.A);
  }
}

__device__ __forceinline__ void soft_merge(SoftPart& a, const SoftPart& b) {
  a.mx = fmaxf(a.mx, b.mx);
  a.cmx = fmaxf(a.cmx, b.cmx);
  a.cs += b.cs;
  a.cq += b.cq;
  const float m = fmaxf(a.m, b.m);
  if (m == -INFINITY) return;
  const float fa = a.m == -INFINITY ? 0.f : expf(a.m - m);
  const float fb = b.m == -INFINITY ? 0.f : expf(b.m - m);
  const float Aa = a.m == -INFINITY ? 0.f : fa * fmaf(a.Z, a.m - m, a.A);
  const float Ab = b.m == -INFINITY ? 0.f : fb * fmaf(b.Z, b.m - m, b.A);
  a.Z = a.Z * fa + b.Z * fb;
  a.A = Aa + Ab;
  a.m = m;
}

__device__ __forceinline__ SoftPart soft_shfl_xor(const SoftPart& a, int o) {
  SoftPart r;
  r.mx = __shfl_xor_sync(0xffffffffu, a.mx, o);
  r.cmx = __shfl_xor_sync(0xffffffffu, a.cmx, o);
  r.cs = __shfl_xor_sync(0xffffffffu, a.cs, o);
  r.cq = __shfl_xor_sync(0xffffffffu, a.cq, o);
  r.m = __shfl_xor_sync(0xffffffffu, a.m, o);
  r.Z = __shfl_xor_sync(0xffffffffu, a.Z, o);
  r.A = __shfl_xor_sync(0xffffffffu, a.A, o);
  return r;
}

__device__ __forceinline__ void soft_store(float* dst, const SoftPart& a) {
  reinterpret_cast<float4*>(dst)[0] = make_float4(a.mx, a.cmx, a.cs, a.cq);
  reinterpret_cast<float4*>(dst)[1] = make_float4(a.m, a.Z, a.A, 0.f);
}

// the same from L2 (a record another CTA of this kernel wrote)
__device__ __forceinline__ SoftPart soft_load_cg(const float* src) {
  const float4 u = __ldcg(reinterpret_cast<const float4*>(src));
  const float4 w = __ldcg(reinterpret_cast<const float4*>(src) + 1);
  return SoftPart{u.x, u.y, u.z, u.w, w.x, w.y, w.z};
}

__device__ __forceinline__ SoftPart soft_load(const float* src) {
  const float4 u = reinterpret_cast<const float4*>(src)[0];
  const float4 w = reinterpret_cast<const float4*>(src)[1];
  return SoftPart{u.x, u.y, u.z, u.w, w.x, w.y, w.z};
}
#endif  // __CUDACC__

}  // namespace adakv
