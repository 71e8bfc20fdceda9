// extern "C" entry points declared in include/adakv_b200.h.
//
// Host-side responsibilities: validate every argument before anything is
// launched (the reference raises ValueError / asserts in the same places,
// adakv/attention.py:192,200,226, adakv/runtime.py:97), derive the workspace
// layout, size grids from host-known bounds (no device->host synchronisation
// anywhere on the decode path), and enqueue the kernels on the caller's stream.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <atomic>
#include <map>
#include <unordered_map>
#include <mutex>
#include <tuple>
#include <string>

#include "kernels.h"

using namespace adakv;

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

#define CUDA_TRY(expr)                                                                  \
  do {                                                                                  \
    cudaError_t e_ = (expr);                                                            \
    if (e_ != cudaSuccess)                                                              \
      return fail(ADAKV_ERR_CUDA, "%s failed: %s", #expr, cudaGetErrorString(e_));     \
  } while (0)

// ---------------------------------------------------------------------------
// per-device state (opt-in shared memory, SM count)
// ---------------------------------------------------------------------------
struct DeviceState {
  bool ready = false;
  int num_sms = 0;
  bool step_ok = false;                            // the one-kernel step can run one CTA per SM
  std::map<int, int> plan_ctas;                    // nb_max * 16 + cluster -> resident plan clusters
  std::map<std::tuple<int, int, int, size_t>, int> step_clusters;  // (dtype, g, csize, smem) -> resident
};

// Test-only knobs (adakv_debug_knob), all off by default.
std::atomic<int64_t> g_dbg_wait_ns{0};   // bound of device waits in ns (0: kWaitLimitNs)
std::atomic<int> g_dbg_flags{0};         // bit 0: head 0 never publishes its entropy
std::atomic<int> g_dbg_path{0};          // decode step: 0 automatic, 1 three kernels, 2 one kernel
std::atomic<int> g_dbg_cluster{0};       // one-kernel step: largest selection cluster (0: 8)

uint64_t wait_limit_ns() {
  const int64_t v = g_dbg_wait_ns.load();
  return v > 0 ? (uint64_t)v : kWaitLimitNs;
}
constexpr int kMaxDevices = 64;
DeviceState g_dev[kMaxDevices];
std::mutex g_dev_mu;

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("ADAKV_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

int device_state(DeviceState** out) {
  int dev = 0;
  CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(ADAKV_ERR_UNSUPPORTED, "device index %d", dev);
  std::lock_guard<std::mutex> lock(g_dev_mu);
  DeviceState& s = g_dev[dev];
  if (!s.ready) {
    CUDA_TRY(cudaDeviceGetAttribute(&s.num_sms, cudaDevAttrMultiProcessorCount, dev));
    CUDA_TRY(estimate_kernels_init());
    CUDA_TRY(plan_kernels_init());
    CUDA_TRY(attend_kernels_init());
    CUDA_TRY(step_kernels_init());
    CUDA_TRY(shard_kernels_init());
    s.step_ok = s.num_sms >= 1;
    s.ready = true;
  }
  *out = &s;
  return ADAKV_OK;
}

int elt_size(int dtype) { return dtype == ADAKV_DTYPE_F32 ? 4 : 2; }

// ---------------------------------------------------------------------------
// validation
// ---------------------------------------------------------------------------
int check_geometry(const adakv_geometry* g) {
  if (!g) return fail(ADAKV_ERR_INVALID, "geometry is NULL");
  if (g->batch < 1) return fail(ADAKV_ERR_INVALID, "batch must be >= 1 (got %d)", g->batch);
  if (g->n_q_heads < 1 || g->n_kv_heads < 1)
    return fail(ADAKV_ERR_INVALID, "head counts must be >= 1 (Hq=%d Hkv=%d)", g->n_q_heads,
                g->n_kv_heads);
  if (g->n_q_heads % g->n_kv_heads)
    return fail(ADAKV_ERR_INVALID, "n_q_heads must be a multiple of n_kv_heads (Hq=%d Hkv=%d)",
                g->n_q_heads, g->n_kv_heads);
  if (g->n_q_heads > 128)
    return fail(ADAKV_ERR_UNSUPPORTED,
                "n_q_heads %d > 128 (the per-sequence entropy exchange covers at most 128 heads)",
                g->n_q_heads);
  if (g->n_q_heads / g->n_kv_heads > 16)
    return fail(ADAKV_ERR_UNSUPPORTED, "GQA group size %d > 16", g->n_q_heads / g->n_kv_heads);
  if (g->head_dim != 64 && g->head_dim != 128)
    return fail(ADAKV_ERR_UNSUPPORTED, "head_dim must be 64 or 128 (got %d)", g->head_dim);
  if (g->block_size != 16 && g->block_size != 32)
    return fail(ADAKV_ERR_UNSUPPORTED, "block_size must be 16 or 32 (got %d)", g->block_size);
  if (g->dtype < ADAKV_DTYPE_F32 || g->dtype > ADAKV_DTYPE_BF16)
    return fail(ADAKV_ERR_INVALID, "unknown dtype %d", g->dtype);
  if (g->max_seq_len < 1) return fail(ADAKV_ERR_INVALID, "max_seq_len must be >= 1");
  const int nb = ceil_div(g->max_seq_len, g->block_size);
  if (g->nb_cap < nb)
    return fail(ADAKV_ERR_INVALID, "nb_cap %d < ceil(max_seq_len / block_size) = %d", g->nb_cap, nb);
  if (nb > kPlanMaxBlocks)
    return fail(ADAKV_ERR_UNSUPPORTED, "max_seq_len / block_size = %d blocks > %d", nb, kPlanMaxBlocks);
  if (g->batch > kEstMaxBatch)
    return fail(ADAKV_ERR_UNSUPPORTED, "batch %d > %d", g->batch, kEstMaxBatch);
  if ((int64_t)g->batch * g->n_q_heads > (1 << 24))
    return fail(ADAKV_ERR_UNSUPPORTED, "batch * n_q_heads too large");
  return ADAKV_OK;
}

int check_view(const adakv_view* v, const char* name, int dtype, bool tokens) {
  if (!v || !v->data) return fail(ADAKV_ERR_INVALID, "%s is NULL", name);
  if (reinterpret_cast<uintptr_t>(v->data) % 16)
    return fail(ADAKV_ERR_INVALID, "%s data must be 16-byte aligned", name);
  const int64_t e = elt_size(dtype);
  if ((v->stride_b * e) % 16 || (v->stride_h * e) % 16 || (tokens && (v->stride_s * e) % 16))
    return fail(ADAKV_ERR_INVALID, "%s strides must be multiples of 16 bytes", name);
  if (v->stride_b < 0 || v->stride_h < 0 || (tokens && v->stride_s < 0))
    return fail(ADAKV_ERR_INVALID, "%s strides must be non-negative", name);
  return ADAKV_OK;
}

int check_params(const adakv_select_params* sp) {
  if (!sp) return fail(ADAKV_ERR_INVALID, "select params are NULL");
  if (!std::isfinite(sp->avg_budget) || sp->avg_budget < 0)
    return fail(ADAKV_ERR_INVALID, "avg_budget must be finite and >= 0");
  if (!std::isfinite(sp->temperature))
    return fail(ADAKV_ERR_INVALID, "temperature must be finite");
  if (sp->k_min < 0 || sp->k_max < 1 || sp->n_sink_blocks < 0 || sp->n_local_blocks < 0 ||
      sp->c_min < 0)
    return fail(ADAKV_ERR_INVALID,
                "need k_min >= 0, k_max >= 1, n_sink_blocks >= 0, n_local_blocks >= 0, c_min >= 0");
  if (sp->policy != ADAKV_POLICY_FIXED && sp->policy != ADAKV_POLICY_ADAPTIVE &&
      sp->policy != ADAKV_POLICY_NUCLEUS)
    return fail(ADAKV_ERR_INVALID, "unknown budget_policy %d", sp->policy);
  if (sp->policy == ADAKV_POLICY_NUCLEUS && !std::isfinite(sp->nucleus_p))
    return fail(ADAKV_ERR_INVALID, "nucleus_p must be finite");
  return ADAKV_OK;
}

SelectCfg to_cfg(const adakv_select_params* sp) {
  SelectCfg c;
  c.avg_budget = sp->avg_budget;
  c.temperature = sp->temperature;
  c.k_min = sp->k_min;
  c.k_max = sp->k_max;
  c.n_sink = sp->n_sink_blocks;
  c.n_local = sp->n_local_blocks;
  c.c_min = sp->c_min;
  c.policy = sp->policy;
  c.nucleus_p = sp->nucleus_p;
  return c;
}

View to_view(const adakv_view* v) {
  View r;
  r.data = v ? v->data : nullptr;
  r.sb = v ? v->stride_b : 0;
  r.sh = v ? v->stride_h : 0;
  r.ss = v ? v->stride_s : 0;
  return r;
}

// CTAs per (sequence, KV head) of the attend kernel: enough to cover the GPU
// once for small batches, at most kAttendMaxSlice union blocks per CTA, and
// no more CTAs than blocks.
int attend_split(const adakv_geometry* g) {
  const int groups = g->batch * g->n_kv_heads;
  const int nb_max = ceil_div(g->max_seq_len, g->block_size);
  int split = std::max(1, kAttendCtaTarget / groups);
  split = std::max(split, ceil_div(nb_max, kAttendMaxSlice));
  split = std::min(split, std::max(1, nb_max));
  return std::min(split, kAttendMaxSplit);
}

// Workspace layout (byte offsets into the caller's buffer; every region is
// 256-byte aligned).  Nothing needs resetting between calls: the plan's
// exchange slots are cleared by the estimator of the same call and the
// attend arrival counters are reset by the CTA that merges.
struct WsLayout {
  size_t status, epoch, slots, scores, stats, bitmap, part, counters, bytes;
  int score_stride, stats_stride, bm_words, split;
  // one-kernel step (present when the geometry can take it); its state words
  // sit at a fixed offset, its regions depend on B, Hq, Hkv, D and nb_cap only
  bool fused;
  size_t fstate, fscores, fpiece, fhslot, fbitmap, fready, fpart, fpready, ftimeline, fbegin, fend;
  int fs_stride, fb_stride;
};

// Geometries the one-kernel step is built for (policy and grid are checked at launch).
bool step_geometry_ok(const adakv_geometry* g) {
  const int gq = g->n_q_heads / g->n_kv_heads;
  const int nb_max = ceil_div(g->max_seq_len, g->block_size);
  return step_kernel_built(g->dtype, g->head_dim, g->block_size, gq) && g->batch <= kStepMaxBatch &&
         (int64_t)g->batch * g->n_q_heads <= kStepMaxHeads && nb_max <= kStepMaxBlocks;
}

WsLayout make_ws(const adakv_geometry* g, bool with_plan) {
  WsLayout L{};
  const int rows = g->batch * g->n_q_heads;
  L.score_stride = (int)align_up((size_t)g->nb_cap, 4);
  L.bm_words = ceil_div(g->nb_cap, 32);
  L.split = attend_split(g);
  const int gq = g->n_q_heads / g->n_kv_heads;
  size_t o = 0;
  auto take = [&](size_t bytes) { size_t at = o; o = align_up(o + bytes, 256); return at; };
  L.status = take(16);
  L.fstate = take(32);  // one-kernel step: calls completed, CTAs done, arrival counter
  L.epoch = take(16);
  L.fused = with_plan && step_geometry_ok(g);
  L.fbegin = o;
  if (L.fused) {
    L.fs_stride = (int)align_up((size_t)g->nb_cap, 4);
    L.fb_stride = (int)align_up((size_t)ceil_div(g->nb_cap, 32), 2);
    L.fscores = take(4 * (size_t)rows * L.fs_stride);
    L.fpiece = take(32 * (size_t)(g->batch * g->n_kv_heads + kStepMaxGrid) * 8 * gq);  // x warps
    L.fhslot = take(8 * (size_t)rows);
    L.fbitmap = take(4 * (size_t)rows * L.fb_stride);
    L.fready = take(8 * (size_t)rows * 8);  // one word per cluster rank (<= 8)
    L.fpart = take(4 * (size_t)kStepMaxGrid * gq * (g->head_dim + 2));
    L.fpready = take(8 * (size_t)kStepMaxGrid);
    L.ftimeline = take(8 * (size_t)kStepMaxGrid * kStepTimelineSlots);
  }
  L.fend = o;
  L.slots = with_plan ? take(sizeof(PlanSlot) * rows * kPlanSlotsPerRow) : 0;
  L.scores = with_plan ? take(sizeof(float) * (size_t)rows * L.score_stride) : 0;
  L.stats_stride = ceil_div(g->nb_cap, kEstRows) * kEstConsumerWarps + 1;
  L.stats = with_plan ? take(sizeof(float) * kStatF * (size_t)rows * L.stats_stride) : 0;
  L.bitmap = take(sizeof(uint32_t) * (size_t)rows * L.bm_words);
  L.part = take(sizeof(float) * (size_t)g->batch * g->n_kv_heads * L.split * gq * (g->head_dim + 2));
  L.counters = take(sizeof(uint32_t) * (size_t)g->batch * g->n_kv_heads);
  L.bytes = o;
  return L;
}

template <typename T>
T* ws_at(void* ws, size_t off) {
  return reinterpret_cast<T*>(static_cast<char*>(ws) + off);
}

int check_workspace(void* ws, size_t bytes, size_t need) {
  if (!ws) return fail(ADAKV_ERR_INVALID, "workspace is NULL");
  if (reinterpret_cast<uintptr_t>(ws) % 256)
    return fail(ADAKV_ERR_INVALID, "workspace must be 256-byte aligned");
  if (bytes < need)
    return fail(ADAKV_ERR_INVALID, "workspace too small: %zu < %zu bytes", bytes, need);
  return ADAKV_OK;
}

// budget + top-k (plan kernel) over score rows already on the device; the
// exchange slots of the workspace must be cleared before it runs
int enqueue_select(const DeviceState* ds, const adakv_geometry* g, const adakv_select_params* sp,
                   const float* scores, int score_stride, const float* stats,
                   const int32_t* seq_lens, int32_t* block_table, int32_t table_width,
                   int32_t* sel_lens, void* ws, const WsLayout& L, cudaStream_t st) {
  const int nb_max = ceil_div(g->max_seq_len, g->block_size);
  const bool pdl = pdl_enabled();
  PlanParams pp{};
  pp.seq_lens = seq_lens;
  pp.max_seq_len = g->max_seq_len;
  pp.B = g->batch;
  pp.Hq = g->n_q_heads;
  pp.bs = g->block_size;
  pp.cfg = to_cfg(sp);
  pp.scores = scores;
  pp.score_stride = score_stride;
  pp.stats = stats;
  pp.stats_stride = L.stats_stride;
  pp.epoch = ws_at<uint32_t>(ws, L.epoch);
  pp.slots = ws_at<PlanSlot>(ws, L.slots);
  pp.sel_lens = sel_lens;
  pp.block_table = block_table;
  pp.table_width = table_width;
  pp.bitmap = ws_at<uint32_t>(ws, L.bitmap);
  pp.bm_words = L.bm_words;
  pp.status = ws_at<uint32_t>(ws, L.status);
  pp.wait_ns = wait_limit_ns();
  pp.debug_flags = g_dbg_flags.load();
  // Cluster size: the largest C in {8, 4, 2} whose slices keep >= 1024 blocks,
  // with all B * Hq * C CTAs resident at once and at most one per SM (one
  // round); else C = 1 with as many sequences per round as are resident.
  // The clusters of a sequence wait on one another (entropy exchange), so the
  // grid never exceeds what is resident once the estimator drains; the
  // exchange is also bounded in time.
  auto active = [&](const PlanLayout& l) {
    std::lock_guard<std::mutex> lock(g_dev_mu);
    const bool nucleus = sp->policy == ADAKV_POLICY_NUCLEUS;
    const int key = (nb_max * 16 + l.csize) * 2 + (nucleus ? 1 : 0);
    auto it = ds->plan_ctas.find(key);
    if (it == ds->plan_ctas.end())
      it = const_cast<DeviceState*>(ds)->plan_ctas.emplace(key, plan_active_clusters(l, nucleus)).first;
    return it->second;
  };
  const int64_t heads = (int64_t)g->batch * g->n_q_heads;
  PlanLayout lay = plan_layout(nb_max, 1);
  for (int c = kPlanMaxCluster; c >= 2; c /= 2) {
    if (ceil_div(nb_max, c) < 1024 || heads * c > ds->num_sms) continue;
    const PlanLayout l = plan_layout(nb_max, c);
    if (l.smem > kPlanSmemMax || active(l) < heads) continue;
    lay = l;
    break;
  }
  if (lay.smem > kPlanSmemMax)
    return fail(ADAKV_ERR_UNSUPPORTED, "sequence too long for the plan kernel's shared memory");
  const int clusters = active(lay);
  if (clusters < g->n_q_heads)
    return fail(ADAKV_ERR_UNSUPPORTED, "n_q_heads %d exceeds the co-resident plan clusters (%d)",
                g->n_q_heads, clusters);
  pp.csize = lay.csize;
  pp.slice_cap = lay.slice_cap;
  pp.seqs_per_round = std::max(1, std::min(g->batch, clusters / g->n_q_heads));
  const int plan_grid = pp.seqs_per_round * g->n_q_heads * lay.csize;
  LaunchOpts op;
  op.pdl = pdl;
  CUDA_TRY(launch_plan(pp, lay, plan_grid, st, op));
  return ADAKV_OK;
}

// estimator (+ fused append) and the plan kernel; shared by adakv_plan and
// adakv_decode_step
int enqueue_plan(const DeviceState* ds, const adakv_geometry* g, const adakv_select_params* sp,
                 const adakv_view* q, float* centroid, const int32_t* seq_lens,
                 const adakv_view* k, const adakv_view* v, const adakv_view* k_new,
                 const adakv_view* v_new, int n_new, int32_t* block_table, int32_t table_width,
                 int32_t* sel_lens, void* ws, const WsLayout& L, cudaStream_t st) {
  const int nb_max = ceil_div(g->max_seq_len, g->block_size);
  uint32_t* status = ws_at<uint32_t>(ws, L.status);
  const bool pdl = pdl_enabled();

  EstParams ep{};
  ep.q = to_view(q);
  ep.cent = centroid;
  ep.nb_cap = g->nb_cap;
  ep.seq_lens = seq_lens;
  ep.max_seq_len = g->max_seq_len;
  ep.B = g->batch;
  ep.Hq = g->n_q_heads;
  ep.Hkv = g->n_kv_heads;
  ep.g = g->n_q_heads / g->n_kv_heads;
  ep.bs = g->block_size;
  ep.scores = ws_at<float>(ws, L.scores);
  ep.score_stride = L.score_stride;
  ep.epoch = ws_at<uint32_t>(ws, L.epoch);
  ep.slots = ws_at<PlanSlot>(ws, L.slots);
  ep.counters = ws_at<uint32_t>(ws, L.counters);
  ep.stats = ws_at<float>(ws, L.stats);
  ep.stats_stride = L.stats_stride;
  ep.n_sink = sp->n_sink_blocks;
  ep.n_local = sp->n_local_blocks;
  ep.temperature = (float)(sp->temperature > 1e-6 ? sp->temperature : 1e-6);
  if (n_new > 0) {
    ep.k = to_view(k);
    ep.v = to_view(v);
    ep.k_new = to_view(k_new);
    ep.v_new = to_view(v_new);
    ep.n_new = n_new;
  }
  ep.status = status;
  ep.stages = estimate_stages(g->dtype, g->head_dim, ep.g, g->batch);
  const int64_t chunks = (int64_t)g->batch * g->n_kv_heads * ceil_div(nb_max, kEstRows);
  const int est_grid = (int)std::max<int64_t>(1, std::min<int64_t>(ds->num_sms, chunks));
  LaunchOpts oe;
  oe.pdl = pdl;
  CUDA_TRY(launch_estimate(ep, g->dtype, g->head_dim, nb_max, est_grid, st, oe));

  return enqueue_select(ds, g, sp, ep.scores, ep.score_stride, ep.stats, seq_lens, block_table,
                        table_width, sel_lens, ws, L, st);
}

// attend over the bitmaps in the workspace
int enqueue_attend(const DeviceState* ds, const adakv_geometry* g, const adakv_view* q,
                   const adakv_view* k, const adakv_view* v, const adakv_view* out,
                   const int32_t* seq_lens, float sm_scale, void* ws, const WsLayout& L,
                   cudaStream_t st, float* out_f32 = nullptr, float* lse = nullptr) {
  (void)ds;
  const int nb_max = ceil_div(g->max_seq_len, g->block_size);
  const int gq = g->n_q_heads / g->n_kv_heads;
  AttendParams ap{};
  ap.q = to_view(q);
  ap.k = to_view(k);
  ap.v = to_view(v);
  ap.out = to_view(out);
  ap.seq_lens = seq_lens;
  ap.max_seq_len = g->max_seq_len;
  ap.B = g->batch;
  ap.Hq = g->n_q_heads;
  ap.Hkv = g->n_kv_heads;
  ap.g = gq;
  ap.sm_scale = sm_scale;
  ap.bitmap = ws_at<uint32_t>(ws, L.bitmap);
  ap.bm_words = L.bm_words;
  ap.nw_max = ceil_div(nb_max, 32);
  ap.status = ws_at<uint32_t>(ws, L.status);
  ap.out_f32 = out_f32;
  ap.lse = lse;
  ap.part = ws_at<float>(ws, L.part);
  ap.counters = ws_at<uint32_t>(ws, L.counters);
  const int split = L.split;
  ap.slice_cap = ceil_div(nb_max, split) + 1;
  // blocks per stage of the gather ring: up to 8 (64 KB of K+V per stage for
  // bf16, D 128, bs 16), fewer when the rest of the shared memory needs room
  const size_t per_block = (size_t)g->block_size * g->head_dim * elt_size(g->dtype) * 2;
  ap.nbt = (int)std::max<size_t>(1, std::min<size_t>(8, (64 * 1024) / per_block));
  size_t smem =
      attend_smem_bytes(g->dtype, g->head_dim, g->block_size, ap.nbt, gq, ap.nw_max, ap.slice_cap, split);
  while (smem > kAttendSmemMax && ap.nbt > 1) {
    --ap.nbt;
    smem = attend_smem_bytes(g->dtype, g->head_dim, g->block_size, ap.nbt, gq, ap.nw_max,
                             ap.slice_cap, split);
  }
  if (smem > kAttendSmemMax)
    return fail(ADAKV_ERR_UNSUPPORTED, "sequence too long for the attend kernel's shared memory");
  LaunchOpts oa;
  oa.pdl = pdl_enabled();
  CUDA_TRY(launch_attend(ap, g->dtype, g->head_dim, g->block_size, split, st, oa));
  return ADAKV_OK;
}

// Which decode-step path last wrote a workspace's scores (adakv_read_scores).
std::unordered_map<const void*, bool> g_last_fused;
// Layout of the one-kernel step's regions last used in a workspace: when it
// changes (first use, another geometry on a shared buffer) its state words
// and tagged regions are zeroed, so no stale word can carry a current tag.
std::unordered_map<const void*, std::pair<size_t, size_t>> g_step_layout;

void note_path(const void* ws, bool fused) {
  std::lock_guard<std::mutex> lock(g_dev_mu);
  g_last_fused[ws] = fused;
}

// Launch shape of the one-kernel step.
struct StepPlan {
  int grid, csize, nbt, slice_cap;
  size_t smem;
};

// The one-kernel step for this call, or why not (the three-kernel chain then
// runs).  The chain is the default: on B200 at 131072 tokens it measures
// 42.6 us per step against 49.8 us for the one-kernel step, whose selection
// phase is latency-bound on a fraction of the SMs and which, holding every
// SM, cannot overlap the next kernel's start.  ADAKV_FUSED=1 (or the
// step-path knob) selects the one-kernel step.
// The cluster size is the largest of 8 / 4 / 2 / 1 CTAs per query head that
// keeps every CTA of the grid resident (one per SM) and slices of >= 256 blocks.
bool step_applies(DeviceState* ds, const adakv_geometry* g, const adakv_select_params* sp,
                  const WsLayout& L, StepPlan* out) {
  const int path = g_dbg_path.load();
  if (path == 1 || !L.fused || !ds->step_ok) return false;
  static const bool env_on = [] {
    const char* e = getenv("ADAKV_FUSED");
    return e && e[0] == '1';
  }();
  if (!env_on && path != 2) return false;
  if (sp->policy == ADAKV_POLICY_NUCLEUS) return false;
  const int gq = g->n_q_heads / g->n_kv_heads;
  const int nb_max = ceil_div(g->max_seq_len, g->block_size);
  const int heads = g->batch * g->n_q_heads, groups = g->batch * g->n_kv_heads;
  const int64_t rows = (int64_t)groups * nb_max;
  const int cmax = g_dbg_cluster.load() > 0 ? g_dbg_cluster.load() : 8;
  for (int c : {8, 4, 2, 1}) {
    if (c > cmax || gq * c > 32 || (c > 1 && nb_max / c < 256)) continue;
    int grid = std::min(ds->num_sms, kStepMaxGrid) / c * c;
    if (grid < heads * c || grid < groups) continue;
    StepPlan sp_{};
    sp_.csize = c;
    sp_.smem = step_smem_bytes(g->head_dim, gq, nb_max, grid / groups, c, &sp_.nbt, &sp_.slice_cap);
    if (sp_.smem > kStepSmemMax) continue;
    int active;
    {
      std::lock_guard<std::mutex> lock(g_dev_mu);
      const auto key = std::make_tuple(g->dtype, gq, c, sp_.smem);
      auto it = ds->step_clusters.find(key);
      if (it == ds->step_clusters.end())
        it = ds->step_clusters
                 .emplace(key, step_active_clusters(g->dtype, g->head_dim, gq, c, sp_.smem))
                 .first;
      active = it->second;
    }
    grid = std::min(grid, active * c);
    if (grid < heads * c || grid < groups) continue;
    // ring stages of one CTA: its rows in 64-row stages plus one per (sequence, KV head) it crosses
    const int64_t per = (rows + grid - 1) / grid;
    if ((per + kStepRows - 1) / kStepRows + std::min<int64_t>(groups, per) + 1 > kStepMaxDesc) continue;
    sp_.grid = grid;
    sp_.smem = step_smem_bytes(g->head_dim, gq, nb_max, grid / groups, c, &sp_.nbt, &sp_.slice_cap);
    *out = sp_;
    return true;
  }
  return false;
}

int enqueue_step(const adakv_geometry* g, const adakv_select_params* sp, const adakv_view* q,
                 const adakv_view* k, const adakv_view* v, const adakv_view* k_new,
                 const adakv_view* v_new, int n_new, float* centroid, const int32_t* seq_lens,
                 float sm_scale, int32_t* block_table, int32_t table_width, int32_t* sel_lens,
                 const adakv_view* out, void* ws, const WsLayout& L, const StepPlan& plan,
                 cudaStream_t st) {
  const int grid = plan.grid;
  const int gq = g->n_q_heads / g->n_kv_heads;
  const int nb_max = ceil_div(g->max_seq_len, g->block_size);
  StepParams p{};
  p.q = to_view(q);
  p.k = to_view(k);
  p.v = to_view(v);
  p.out = to_view(out);
  if (n_new > 0) {
    p.k_new = to_view(k_new);
    p.v_new = to_view(v_new);
  }
  p.cent = centroid;
  p.nb_cap = g->nb_cap;
  p.seq_lens = seq_lens;
  p.max_seq_len = g->max_seq_len;
  p.B = g->batch;
  p.Hq = g->n_q_heads;
  p.Hkv = g->n_kv_heads;
  p.bs = g->block_size;
  p.n_new = n_new;
  p.cfg = to_cfg(sp);
  p.sm_scale = sm_scale;
  p.block_table = block_table;
  p.table_width = table_width;
  p.sel_lens = sel_lens;
  p.lse = nullptr;
  p.status = ws_at<uint32_t>(ws, L.status);
  p.epoch = ws_at<uint32_t>(ws, L.fstate);
  p.arrive = ws_at<unsigned long long>(ws, L.fstate + 8);
  p.scores = ws_at<float>(ws, L.fscores);
  p.fs_stride = L.fs_stride;
  p.piece = ws_at<float>(ws, L.fpiece);
  p.hslot = ws_at<unsigned long long>(ws, L.fhslot);
  p.bitmap = ws_at<uint32_t>(ws, L.fbitmap);
  p.fb_stride = L.fb_stride;
  p.ready = ws_at<unsigned long long>(ws, L.fready);
  p.part = ws_at<float>(ws, L.fpart);
  p.pready = ws_at<unsigned long long>(ws, L.fpready);
  p.nb_max = nb_max;
  p.wait_ns = wait_limit_ns();
  p.debug_flags = g_dbg_flags.load();
  p.timeline = ws_at<unsigned long long>(ws, L.ftimeline);
  {
    const std::pair<size_t, size_t> sig(L.fend - L.fbegin, (size_t)grid * 16 + plan.csize);
    bool fresh;
    {
      std::lock_guard<std::mutex> lock(g_dev_mu);
      auto it = g_step_layout.find(ws);
      fresh = it == g_step_layout.end() || it->second != sig;
    }
    if (fresh) {
      cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
      CUDA_TRY(cudaStreamIsCapturing(st, &cs));
      if (cs != cudaStreamCaptureStatusNone)
        return fail(ADAKV_ERR_INVALID,
                    "the first adakv_decode_step on a workspace (or on a new geometry) must run "
                    "before stream capture: it initialises the workspace");
      CUDA_TRY(cudaMemsetAsync(ws_at<char>(ws, L.fstate), 0, 32, st));
      CUDA_TRY(cudaMemsetAsync(ws_at<char>(ws, L.fbegin), 0, L.fend - L.fbegin, st));
      std::lock_guard<std::mutex> lock(g_dev_mu);
      g_step_layout[ws] = sig;
    }
  }
  p.csize = plan.csize;
  p.nbt = plan.nbt;
  p.slice_cap = plan.slice_cap;
  const size_t smem = plan.smem;
  LaunchOpts o;
  o.pdl = pdl_enabled();
  CUDA_TRY(launch_step(p, g->dtype, g->head_dim, gq, grid, smem, st, o));
  note_path(ws, true);
  return ADAKV_OK;
}

int check_attend_views(const adakv_geometry* g, const adakv_view* q, const adakv_view* k,
                       const adakv_view* v, const adakv_view* out) {
  int rc;
  if ((rc = check_view(q, "q", g->dtype, false))) return rc;
  if ((rc = check_view(k, "k", g->dtype, true))) return rc;
  if ((rc = check_view(v, "v", g->dtype, true))) return rc;
  if ((rc = check_view(out, "out", g->dtype, false))) return rc;
  return ADAKV_OK;
}

}  // namespace

extern "C" {

int adakv_abi_version(void) { return ADAKV_B200_ABI_VERSION; }

const char* adakv_last_error(void) { return g_last_error.c_str(); }

int32_t adakv_plan_table_width(const adakv_geometry* geo, const adakv_select_params* sp) {
  if (check_geometry(geo) || check_params(sp)) return -1;
  return table_width_for(geo->nb_cap, to_cfg(sp));
}

size_t adakv_plan_workspace_bytes(const adakv_geometry* geo, const adakv_select_params* sp) {
  if (check_geometry(geo) || check_params(sp)) return 0;
  return make_ws(geo, true).bytes;
}

size_t adakv_attend_workspace_bytes(const adakv_geometry* geo, int32_t table_width) {
  if (check_geometry(geo)) return 0;
  if (table_width < 1) {
    fail(ADAKV_ERR_INVALID, "table_width must be >= 1");
    return 0;
  }
  return make_ws(geo, false).bytes;
}

int adakv_centroid_build(const adakv_geometry* geo, const adakv_view* k, const int32_t* seq_lens,
                         float* centroid, void* stream) {
  int rc;
  if ((rc = check_geometry(geo))) return rc;
  if ((rc = check_view(k, "k", geo->dtype, true))) return rc;
  if (!centroid || reinterpret_cast<uintptr_t>(centroid) % 16)
    return fail(ADAKV_ERR_INVALID, "centroid must be a 16-byte aligned device pointer");
  CentroidParams p{};
  p.k = to_view(k);
  p.seq_lens = seq_lens;
  p.max_seq_len = geo->max_seq_len;
  p.B = geo->batch;
  p.Hkv = geo->n_kv_heads;
  p.bs = geo->block_size;
  p.nb_cap = geo->nb_cap;
  p.n_new = 0;
  p.cent = centroid;
  p.status = nullptr;
  CUDA_TRY(launch_centroid(p, geo->dtype, geo->head_dim, ceil_div(geo->max_seq_len, geo->block_size),
                           static_cast<cudaStream_t>(stream)));
  return ADAKV_OK;
}

int adakv_kv_append(const adakv_geometry* geo, const adakv_view* k_cache, const adakv_view* v_cache,
                    const adakv_view* k_new, const adakv_view* v_new, int32_t n_new,
                    const int32_t* seq_lens, float* centroid, void* stream) {
  int rc;
  if ((rc = check_geometry(geo))) return rc;
  if ((rc = check_view(k_cache, "k_cache", geo->dtype, true))) return rc;
  if ((rc = check_view(v_cache, "v_cache", geo->dtype, true))) return rc;
  if ((rc = check_view(k_new, "k_new", geo->dtype, true))) return rc;
  if ((rc = check_view(v_new, "v_new", geo->dtype, true))) return rc;
  if (n_new < 1 || n_new > geo->max_seq_len)
    return fail(ADAKV_ERR_INVALID, "n_new must be in [1, max_seq_len] (got %d)", n_new);
  if (!centroid || reinterpret_cast<uintptr_t>(centroid) % 16)
    return fail(ADAKV_ERR_INVALID, "centroid must be a 16-byte aligned device pointer");
  CentroidParams p{};
  p.k = to_view(k_cache);
  p.v = to_view(v_cache);
  p.k_new = to_view(k_new);
  p.v_new = to_view(v_new);
  p.seq_lens = seq_lens;
  p.max_seq_len = geo->max_seq_len;
  p.B = geo->batch;
  p.Hkv = geo->n_kv_heads;
  p.bs = geo->block_size;
  p.nb_cap = geo->nb_cap;
  p.n_new = n_new;
  p.cent = centroid;
  p.status = nullptr;
  CUDA_TRY(launch_centroid(p, geo->dtype, geo->head_dim, ceil_div(n_new, geo->block_size) + 1,
                           static_cast<cudaStream_t>(stream)));
  return ADAKV_OK;
}

int adakv_centroid_refresh(const adakv_geometry* geo, const adakv_view* k, int32_t n_new,
                           const int32_t* seq_lens, float* centroid, void* stream) {
  int rc;
  if ((rc = check_geometry(geo))) return rc;
  if ((rc = check_view(k, "k", geo->dtype, true))) return rc;
  if (n_new < 1 || n_new > geo->max_seq_len)
    return fail(ADAKV_ERR_INVALID, "n_new must be in [1, max_seq_len] (got %d)", n_new);
  if (!centroid || reinterpret_cast<uintptr_t>(centroid) % 16)
    return fail(ADAKV_ERR_INVALID, "centroid must be a 16-byte aligned device pointer");
  CentroidParams p{};
  p.k = to_view(k);
  p.seq_lens = seq_lens;
  p.max_seq_len = geo->max_seq_len;
  p.B = geo->batch;
  p.Hkv = geo->n_kv_heads;
  p.bs = geo->block_size;
  p.nb_cap = geo->nb_cap;
  p.n_new = n_new;
  p.cent = centroid;
  p.status = nullptr;
  CUDA_TRY(launch_centroid(p, geo->dtype, geo->head_dim, ceil_div(n_new, geo->block_size) + 1,
                           static_cast<cudaStream_t>(stream)));
  return ADAKV_OK;
}

int adakv_plan(const adakv_geometry* geo, const adakv_select_params* sp, const adakv_view* q,
               const float* centroid, const int32_t* seq_lens, int32_t* block_table,
               int32_t table_width, int32_t* sel_lens, float* scores_out, void* workspace,
               size_t workspace_bytes, void* stream) {
  int rc;
  if ((rc = check_geometry(geo))) return rc;
  if ((rc = check_params(sp))) return rc;
  if ((rc = check_view(q, "q", geo->dtype, false))) return rc;
  if (!centroid || reinterpret_cast<uintptr_t>(centroid) % 16)
    return fail(ADAKV_ERR_INVALID, "centroid must be a 16-byte aligned device pointer");
  if (!block_table || !sel_lens) return fail(ADAKV_ERR_INVALID, "block_table / sel_lens are NULL");
  const int need_w = table_width_for(geo->nb_cap, to_cfg(sp));
  if (table_width < need_w)
    return fail(ADAKV_ERR_INVALID, "table_width %d < required %d", table_width, need_w);
  const WsLayout L = make_ws(geo, true);
  if ((rc = check_workspace(workspace, workspace_bytes, L.bytes))) return rc;
  DeviceState* ds = nullptr;
  if ((rc = device_state(&ds))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((rc = enqueue_plan(ds, geo, sp, q, const_cast<float*>(centroid), seq_lens, nullptr, nullptr,
                         nullptr, nullptr, 0, block_table, table_width, sel_lens, workspace, L, st)))
    return rc;
  note_path(workspace, false);
  if (scores_out) {
    CUDA_TRY(cudaMemcpy2DAsync(scores_out, sizeof(float) * geo->nb_cap,
                               ws_at<float>(workspace, L.scores), sizeof(float) * L.score_stride,
                               sizeof(float) * geo->nb_cap,
                               (size_t)geo->batch * geo->n_q_heads, cudaMemcpyDeviceToDevice, st));
  }
  return ADAKV_OK;
}

int adakv_attend(const adakv_geometry* geo, const adakv_view* q, const adakv_view* k,
                 const adakv_view* v, const int32_t* block_table, int32_t table_width,
                 const int32_t* sel_lens, const int32_t* seq_lens, float sm_scale,
                 const adakv_view* out, void* workspace, size_t workspace_bytes, void* stream) {
  int rc;
  if ((rc = check_geometry(geo))) return rc;
  if ((rc = check_attend_views(geo, q, k, v, out))) return rc;
  if (!block_table || !sel_lens) return fail(ADAKV_ERR_INVALID, "block_table / sel_lens are NULL");
  if (table_width < 1) return fail(ADAKV_ERR_INVALID, "table_width must be >= 1");
  if (!std::isfinite(sm_scale)) return fail(ADAKV_ERR_INVALID, "sm_scale must be finite");
  const WsLayout L = make_ws(geo, false);
  if ((rc = check_workspace(workspace, workspace_bytes, L.bytes))) return rc;
  DeviceState* ds = nullptr;
  if ((rc = device_state(&ds))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  TableParams tp{};
  tp.block_table = block_table;
  tp.table_width = table_width;
  tp.sel_lens = sel_lens;
  tp.seq_lens = seq_lens;
  tp.max_seq_len = geo->max_seq_len;
  tp.B = geo->batch;
  tp.Hq = geo->n_q_heads;
  tp.bs = geo->block_size;
  tp.bitmap = ws_at<uint32_t>(workspace, L.bitmap);
  tp.bm_words = L.bm_words;
  tp.status = ws_at<uint32_t>(workspace, L.status);
  tp.counters = ws_at<uint32_t>(workspace, L.counters);
  tp.ncounters = geo->batch * geo->n_kv_heads;
  LaunchOpts ot;
  ot.pdl = pdl_enabled();
  CUDA_TRY(launch_table_bitmap(tp, st, ot));
  return enqueue_attend(ds, geo, q, k, v, out, seq_lens, sm_scale, workspace, L, st);
}

int adakv_decode_step(const adakv_geometry* geo, const adakv_select_params* sp,
                      const adakv_view* q, const adakv_view* k, const adakv_view* v,
                      const adakv_view* k_new, const adakv_view* v_new, int32_t n_new,
                      float* centroid, const int32_t* seq_lens, float sm_scale,
                      int32_t* block_table, int32_t table_width, int32_t* sel_lens,
                      const adakv_view* out, void* workspace, size_t workspace_bytes,
                      void* stream) {
  int rc;
  if ((rc = check_geometry(geo))) return rc;
  if ((rc = check_params(sp))) return rc;
  if ((rc = check_attend_views(geo, q, k, v, out))) return rc;
  if (n_new < 0 || n_new > geo->max_seq_len)
    return fail(ADAKV_ERR_INVALID, "n_new must be in [0, max_seq_len] (got %d)", n_new);
  if (n_new > 0) {
    if ((rc = check_view(k_new, "k_new", geo->dtype, true))) return rc;
    if ((rc = check_view(v_new, "v_new", geo->dtype, true))) return rc;
  }
  if (!centroid || reinterpret_cast<uintptr_t>(centroid) % 16)
    return fail(ADAKV_ERR_INVALID, "centroid must be a 16-byte aligned device pointer");
  if (!block_table || !sel_lens) return fail(ADAKV_ERR_INVALID, "block_table / sel_lens are NULL");
  if (!std::isfinite(sm_scale)) return fail(ADAKV_ERR_INVALID, "sm_scale must be finite");
  const int need_w = table_width_for(geo->nb_cap, to_cfg(sp));
  if (table_width < need_w)
    return fail(ADAKV_ERR_INVALID, "table_width %d < required %d", table_width, need_w);
  const WsLayout L = make_ws(geo, true);
  if ((rc = check_workspace(workspace, workspace_bytes, L.bytes))) return rc;
  DeviceState* ds = nullptr;
  if ((rc = device_state(&ds))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  StepPlan plan{};
  if (step_applies(ds, geo, sp, L, &plan))
    return enqueue_step(geo, sp, q, k, v, k_new, v_new, n_new, centroid, seq_lens, sm_scale,
                        block_table, table_width, sel_lens, out, workspace, L, plan, st);
  if ((rc = enqueue_plan(ds, geo, sp, q, centroid, seq_lens, k, v, k_new, v_new, n_new,
                         block_table, table_width, sel_lens, workspace, L, st)))
    return rc;
  note_path(workspace, false);
  return enqueue_attend(ds, geo, q, k, v, out, seq_lens, sm_scale, workspace, L, st);
}

int adakv_read_scores(const adakv_geometry* geo, void* workspace, size_t workspace_bytes,
                      float* scores_out, int32_t score_stride, void* stream) {
  int rc;
  if ((rc = check_geometry(geo))) return rc;
  const WsLayout L = make_ws(geo, true);
  if ((rc = check_workspace(workspace, workspace_bytes, L.bytes))) return rc;
  if (!scores_out) return fail(ADAKV_ERR_INVALID, "scores_out is NULL");
  const int nb_max = ceil_div(geo->max_seq_len, geo->block_size);
  if (score_stride < nb_max)
    return fail(ADAKV_ERR_INVALID, "score_stride %d < blocks of max_seq_len (%d)", score_stride, nb_max);
  bool fused = false;
  {
    std::lock_guard<std::mutex> lock(g_dev_mu);
    auto it = g_last_fused.find(workspace);
    if (it == g_last_fused.end())
      return fail(ADAKV_ERR_INVALID, "no decode step or plan has run on this workspace");
    fused = it->second;
  }
  CUDA_TRY(launch_step_scores(fused, ws_at<float>(workspace, L.fscores), L.fs_stride,
                              ws_at<float>(workspace, L.scores), L.score_stride,
                              geo->batch * geo->n_q_heads, nb_max, scores_out, score_stride,
                              static_cast<cudaStream_t>(stream)));
  return ADAKV_OK;
}

int adakv_last_path(const void* workspace) {
  std::lock_guard<std::mutex> lock(g_dev_mu);
  auto it = g_last_fused.find(workspace);
  if (it == g_last_fused.end()) return 0;
  return it->second ? 2 : 1;
}

int adakv_stage(void* dst, const void* src, size_t bytes, void* stream) {
  if (!dst || !src) return fail(ADAKV_ERR_INVALID, "dst / src are NULL");
  if (bytes == 0) return ADAKV_OK;
  if (reinterpret_cast<uintptr_t>(dst) % 16 || reinterpret_cast<uintptr_t>(src) % 16)
    return fail(ADAKV_ERR_INVALID, "dst and src must be 16-byte aligned");
  cudaPointerAttributes da{}, sa{};
  CUDA_TRY(cudaPointerGetAttributes(&da, dst));
  CUDA_TRY(cudaPointerGetAttributes(&sa, src));
  if (da.type != cudaMemoryTypeDevice && da.type != cudaMemoryTypeManaged)
    return fail(ADAKV_ERR_INVALID, "dst must be device memory");
  const void* s = src;
  if (sa.type == cudaMemoryTypeHost) {
    if (!sa.devicePointer)
      return fail(ADAKV_ERR_INVALID, "src is page-locked host memory without a device mapping");
    s = sa.devicePointer;
  } else if (sa.type == cudaMemoryTypeUnregistered) {
    return fail(ADAKV_ERR_INVALID, "src must be device or page-locked host memory");
  }
  CUDA_TRY(launch_stage(s, dst, bytes, static_cast<cudaStream_t>(stream)));
  return ADAKV_OK;
}

int adakv_set_status_sink(void* workspace, uint32_t* host_word, void* stream) {
  if (!workspace) return fail(ADAKV_ERR_INVALID, "workspace is NULL");
  void* dev = nullptr;
  if (host_word) {
    const cudaError_t e = cudaHostGetDevicePointer(&dev, host_word, 0);
    if (e != cudaSuccess)
      return fail(ADAKV_ERR_INVALID, "host_word is not mapped page-locked memory: %s",
                  cudaGetErrorString(e));
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  CUDA_TRY(cudaMemcpyAsync(static_cast<char*>(workspace) + 8, &dev, sizeof(dev),
                           cudaMemcpyHostToDevice, st));
  CUDA_TRY(cudaStreamSynchronize(st));
  return ADAKV_OK;
}

int adakv_debug_timeline(const adakv_geometry* geo, void* workspace, size_t workspace_bytes,
                         uint64_t* out, int32_t max_ctas, void* stream) {
  int rc;
  if ((rc = check_geometry(geo))) return rc;
  const WsLayout L = make_ws(geo, true);
  if ((rc = check_workspace(workspace, workspace_bytes, L.bytes))) return rc;
  if (!L.fused) return fail(ADAKV_ERR_INVALID, "this geometry does not run the one-kernel step");
  if (!out || max_ctas < 1) return fail(ADAKV_ERR_INVALID, "out is NULL or max_ctas < 1");
  const int n = std::min(max_ctas, kStepMaxGrid);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  CUDA_TRY(cudaStreamSynchronize(st));
  CUDA_TRY(cudaMemcpy(out, ws_at<char>(workspace, L.ftimeline),
                      sizeof(uint64_t) * kStepTimelineSlots * (size_t)n, cudaMemcpyDeviceToHost));
  return ADAKV_OK;
}

int adakv_debug_knob(int32_t knob, int64_t value) {
  switch (knob) {
    case ADAKV_KNOB_WAIT_NS:
      if (value < 0) return fail(ADAKV_ERR_INVALID, "wait limit must be >= 0 ns");
      g_dbg_wait_ns.store(value);
      return ADAKV_OK;
    case ADAKV_KNOB_FLAGS:
      g_dbg_flags.store((int)value);
      return ADAKV_OK;
    case ADAKV_KNOB_STEP_PATH:
      if (value < 0 || value > 2) return fail(ADAKV_ERR_INVALID, "step path must be 0, 1 or 2");
      g_dbg_path.store((int)value);
      return ADAKV_OK;
    case ADAKV_KNOB_STEP_CLUSTER:
      if (value != 0 && value != 1 && value != 2 && value != 4 && value != 8)
        return fail(ADAKV_ERR_INVALID, "step cluster must be 0, 1, 2, 4 or 8");
      g_dbg_cluster.store((int)value);
      return ADAKV_OK;
    default:
      return fail(ADAKV_ERR_INVALID, "unknown knob %d", knob);
  }
}

int adakv_read_status(void* workspace, uint32_t* status, void* stream) {
  if (!workspace || !status) return fail(ADAKV_ERR_INVALID, "workspace / status are NULL");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  CUDA_TRY(cudaStreamSynchronize(st));
  CUDA_TRY(cudaMemcpy(status, workspace, sizeof(uint32_t), cudaMemcpyDeviceToHost));
  CUDA_TRY(cudaMemsetAsync(workspace, 0, sizeof(uint32_t), st));
  CUDA_TRY(cudaStreamSynchronize(st));
  return ADAKV_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// adakv_attend_noalloc: adakv_attend with its scratch (status word + selection
// bitmaps) in a fixed device array of this library instead of a caller
// workspace.  It has no counterpart in the reference.
// ---------------------------------------------------------------------------
namespace {

// Largest scratch the entry point can use.  A call needs exactly
// adakv_attend_workspace_bytes(geo, table_width) bytes of it: the status
// header, the selection bitmaps (B * Hq * ceil(nb_cap / 32) * 4 bytes), the
// split-KV partials (B * Hkv * split * (Hq / Hkv) * (head_dim + 2) * 4 bytes,
// split = CTAs per KV head, about 148 / (B * Hkv) for small batches) and the
// arrival counters, each region 256-byte aligned.  Batch 1 at 128K tokens
// (32 q / 8 KV heads, D 128) needs about 0.33 MiB.
constexpr size_t kNoAllocScratchBytes = 4u << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Per-device address of g_noalloc_scratch, resolved once with that device
// current (a __device__ symbol has one instance per device).
void* g_noalloc_addr[kMaxDevices];

int noalloc_scratch(void** out) {
  int dev = 0;
  CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(ADAKV_ERR_UNSUPPORTED, "device index %d", dev);
  std::lock_guard<std::mutex> lock(g_dev_mu);
  if (!g_noalloc_addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess)
      return fail(ADAKV_ERR_CUDA, "cudaGetSymbolAddress(scratch) failed: %s", cudaGetErrorString(e));
    if (!p || reinterpret_cast<uintptr_t>(p) % 256)
      return fail(ADAKV_ERR_CUDA, "scratch array is not 256-byte aligned");
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return ADAKV_OK;
}

}  // namespace

extern "C" {

int adakv_attend_noalloc(const adakv_geometry* geo, const adakv_view* q, const adakv_view* k,
                         const adakv_view* v, const int32_t* block_table, int32_t table_width,
                         const int32_t* sel_lens, const int32_t* seq_lens, float sm_scale,
                         const adakv_view* out, uint32_t* status, void* stream) {
  int rc;
  if ((rc = check_geometry(geo))) return rc;
  if ((rc = check_attend_views(geo, q, k, v, out))) return rc;
  if (!block_table || !sel_lens) return fail(ADAKV_ERR_INVALID, "block_table / sel_lens are NULL");
  if (table_width < 1) return fail(ADAKV_ERR_INVALID, "table_width must be >= 1");
  if (!std::isfinite(sm_scale)) return fail(ADAKV_ERR_INVALID, "sm_scale must be finite");
  if (status && reinterpret_cast<uintptr_t>(status) % 4)
    return fail(ADAKV_ERR_INVALID, "status must be a 4-byte aligned device pointer");
  const WsLayout L = make_ws(geo, false);
  if (L.bytes > kNoAllocScratchBytes)
    return fail(ADAKV_ERR_INVALID,
                "adakv_attend_noalloc needs %zu scratch bytes for this geometry "
                "(adakv_attend_workspace_bytes), above its fixed maximum of %zu; use "
                "adakv_attend with a workspace",
                L.bytes, kNoAllocScratchBytes);
  DeviceState* ds = nullptr;
  if ((rc = device_state(&ds))) return rc;
  void* ws = nullptr;
  if ((rc = noalloc_scratch(&ws))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // the status word collects this call's bits: it starts at zero every call;
  // the bitmap rows are written in full by the table kernel before use
  CUDA_TRY(cudaMemsetAsync(ws_at<uint32_t>(ws, L.status), 0, sizeof(uint32_t), st));
  TableParams tp{};
  tp.block_table = block_table;
  tp.table_width = table_width;
  tp.sel_lens = sel_lens;
  tp.seq_lens = seq_lens;
  tp.max_seq_len = geo->max_seq_len;
  tp.B = geo->batch;
  tp.Hq = geo->n_q_heads;
  tp.bs = geo->block_size;
  tp.bitmap = ws_at<uint32_t>(ws, L.bitmap);
  tp.bm_words = L.bm_words;
  tp.status = ws_at<uint32_t>(ws, L.status);
  tp.counters = ws_at<uint32_t>(ws, L.counters);
  tp.ncounters = geo->batch * geo->n_kv_heads;
  LaunchOpts ot;
  ot.pdl = false;  // follows the memset
  CUDA_TRY(launch_table_bitmap(tp, st, ot));
  if ((rc = enqueue_attend(ds, geo, q, k, v, out, seq_lens, sm_scale, ws, L, st))) return rc;
  if (status)
    CUDA_TRY(cudaMemcpyAsync(status, ws_at<uint32_t>(ws, L.status), sizeof(uint32_t),
                             cudaMemcpyDeviceToDevice, st));
  return ADAKV_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Sequence-sharded decode (one sequence split over several GPUs by blocks):
// per-shard scores, selection over the all-gathered score rows, per-shard
// attention with its log-sum-exp, and the log-sum-exp merge.
// ---------------------------------------------------------------------------
extern "C" {

int adakv_estimate(const adakv_geometry* geo, const adakv_view* q, const float* centroid,
                   const int32_t* seq_lens, float* scores, int32_t score_stride, void* workspace,
                   size_t workspace_bytes, void* stream) {
  int rc;
  if ((rc = check_geometry(geo))) return rc;
  if ((rc = check_view(q, "q", geo->dtype, false))) return rc;
  if (!centroid || reinterpret_cast<uintptr_t>(centroid) % 16)
    return fail(ADAKV_ERR_INVALID, "centroid must be a 16-byte aligned device pointer");
  if (!scores) return fail(ADAKV_ERR_INVALID, "scores is NULL");
  if (score_stride < ceil_div(geo->max_seq_len, geo->block_size))
    return fail(ADAKV_ERR_INVALID, "score_stride %d < blocks of max_seq_len", score_stride);
  const WsLayout L = make_ws(geo, true);
  if ((rc = check_workspace(workspace, workspace_bytes, L.bytes))) return rc;
  DeviceState* ds = nullptr;
  if ((rc = device_state(&ds))) return rc;
  const int nb_max = ceil_div(geo->max_seq_len, geo->block_size);
  EstParams ep{};
  ep.q = to_view(q);
  ep.cent = const_cast<float*>(centroid);
  ep.nb_cap = geo->nb_cap;
  ep.seq_lens = seq_lens;
  ep.max_seq_len = geo->max_seq_len;
  ep.B = geo->batch;
  ep.Hq = geo->n_q_heads;
  ep.Hkv = geo->n_kv_heads;
  ep.g = geo->n_q_heads / geo->n_kv_heads;
  ep.bs = geo->block_size;
  ep.scores = scores;
  ep.score_stride = score_stride;
  ep.temperature = 1.0f;
  ep.status = ws_at<uint32_t>(workspace, L.status);
  ep.stages = estimate_stages(geo->dtype, geo->head_dim, ep.g, geo->batch);
  const int64_t chunks = (int64_t)geo->batch * geo->n_kv_heads * ceil_div(nb_max, kEstRows);
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(ds->num_sms, chunks));
  LaunchOpts oe;
  oe.pdl = pdl_enabled();
  CUDA_TRY(launch_estimate(ep, geo->dtype, geo->head_dim, nb_max, grid,
                           static_cast<cudaStream_t>(stream), oe));
  return ADAKV_OK;
}

int adakv_select(const adakv_geometry* geo, const adakv_select_params* sp, const float* scores,
                 int32_t score_stride, const int32_t* seq_lens, int32_t* block_table,
                 int32_t table_width, int32_t* sel_lens, void* workspace, size_t workspace_bytes,
                 void* stream) {
  int rc;
  if ((rc = check_geometry(geo))) return rc;
  if ((rc = check_params(sp))) return rc;
  if (!scores) return fail(ADAKV_ERR_INVALID, "scores is NULL");
  if (score_stride < ceil_div(geo->max_seq_len, geo->block_size))
    return fail(ADAKV_ERR_INVALID, "score_stride %d < blocks of max_seq_len", score_stride);
  if (!block_table || !sel_lens) return fail(ADAKV_ERR_INVALID, "block_table / sel_lens are NULL");
  const int need_w = table_width_for(geo->nb_cap, to_cfg(sp));
  if (table_width < need_w)
    return fail(ADAKV_ERR_INVALID, "table_width %d < required %d", table_width, need_w);
  const WsLayout L = make_ws(geo, true);
  if ((rc = check_workspace(workspace, workspace_bytes, L.bytes))) return rc;
  DeviceState* ds = nullptr;
  if ((rc = device_state(&ds))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // the exchange slots start cleared (the estimator does this on the fused path)
  CUDA_TRY(cudaMemsetAsync(ws_at<char>(workspace, L.slots), 0,
                           sizeof(PlanSlot) * (size_t)geo->batch * geo->n_q_heads * kPlanSlotsPerRow, st));
  return enqueue_select(ds, geo, sp, scores, score_stride, nullptr, seq_lens, block_table,
                        table_width, sel_lens, workspace, L, st);
}

int adakv_attend_partial(const adakv_geometry* geo, const adakv_view* q, const adakv_view* k,
                         const adakv_view* v, const int32_t* block_table, int32_t table_width,
                         const int32_t* sel_lens, int32_t block_offset, const int32_t* seq_lens,
                         float sm_scale, float* out_f32, float* lse, void* workspace,
                         size_t workspace_bytes, void* stream) {
  int rc;
  if ((rc = check_geometry(geo))) return rc;
  if ((rc = check_view(q, "q", geo->dtype, false))) return rc;
  if ((rc = check_view(k, "k", geo->dtype, true))) return rc;
  if ((rc = check_view(v, "v", geo->dtype, true))) return rc;
  if (!block_table || !sel_lens) return fail(ADAKV_ERR_INVALID, "block_table / sel_lens are NULL");
  if (table_width < 1) return fail(ADAKV_ERR_INVALID, "table_width must be >= 1");
  if (block_offset < 0) return fail(ADAKV_ERR_INVALID, "block_offset must be >= 0");
  if (!out_f32 || !lse || reinterpret_cast<uintptr_t>(out_f32) % 16)
    return fail(ADAKV_ERR_INVALID, "out_f32 (16-byte aligned) and lse are required");
  if (!std::isfinite(sm_scale)) return fail(ADAKV_ERR_INVALID, "sm_scale must be finite");
  const WsLayout L = make_ws(geo, false);
  if ((rc = check_workspace(workspace, workspace_bytes, L.bytes))) return rc;
  DeviceState* ds = nullptr;
  if ((rc = device_state(&ds))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  TableParams tp{};
  tp.block_table = block_table;
  tp.table_width = table_width;
  tp.sel_lens = sel_lens;
  tp.seq_lens = seq_lens;
  tp.max_seq_len = geo->max_seq_len;
  tp.B = geo->batch;
  tp.Hq = geo->n_q_heads;
  tp.bs = geo->block_size;
  tp.bitmap = ws_at<uint32_t>(workspace, L.bitmap);
  tp.bm_words = L.bm_words;
  tp.counters = ws_at<uint32_t>(workspace, L.counters);
  tp.ncounters = geo->batch * geo->n_kv_heads;
  tp.block_offset = block_offset;
  tp.local_only = 1;
  tp.status = ws_at<uint32_t>(workspace, L.status);
  LaunchOpts ot;
  ot.pdl = pdl_enabled();
  CUDA_TRY(launch_table_bitmap(tp, st, ot));
  adakv_view none{};
  return enqueue_attend(ds, geo, q, k, v, &none, seq_lens, sm_scale, workspace, L, st, out_f32,
                        lse);
}

int adakv_combine(int32_t n_parts, int32_t batch, int32_t n_q_heads, int32_t head_dim,
                  int32_t dtype, const float* parts, const float* lse, const adakv_view* out,
                  void* stream) {
  int rc;
  if (n_parts < 1 || batch < 1 || n_q_heads < 1 || head_dim < 1)
    return fail(ADAKV_ERR_INVALID, "n_parts, batch, n_q_heads and head_dim must be >= 1");
  if (dtype < ADAKV_DTYPE_F32 || dtype > ADAKV_DTYPE_BF16)
    return fail(ADAKV_ERR_INVALID, "unknown dtype %d", dtype);
  if (!parts || !lse) return fail(ADAKV_ERR_INVALID, "parts / lse are NULL");
  if ((rc = check_view(out, "out", dtype, false))) return rc;
  CombineParams cp{};
  cp.parts = parts;
  cp.lse = lse;
  cp.n_parts = n_parts;
  cp.rows = batch * n_q_heads;
  cp.D = head_dim;
  cp.part_stride = (int64_t)cp.rows * head_dim;
  cp.lse_stride = cp.rows;
  cp.out = to_view(out);
  cp.Hq = n_q_heads;
  LaunchOpts oc;
  oc.pdl = pdl_enabled();
  CUDA_TRY(launch_combine(cp, dtype, static_cast<cudaStream_t>(stream), oc));
  return ADAKV_OK;
}

int adakv_combine_packed(int32_t n_parts, int32_t batch, int32_t n_q_heads, int32_t head_dim,
                         int32_t dtype, const float* packed, int64_t part_stride,
                         const adakv_view* out, void* stream) {
  int rc;
  if (n_parts < 1 || batch < 1 || n_q_heads < 1 || head_dim < 1)
    return fail(ADAKV_ERR_INVALID, "n_parts, batch, n_q_heads and head_dim must be >= 1");
  if (dtype < ADAKV_DTYPE_F32 || dtype > ADAKV_DTYPE_BF16)
    return fail(ADAKV_ERR_INVALID, "unknown dtype %d", dtype);
  const int64_t rows = (int64_t)batch * n_q_heads;
  if (!packed || part_stride < rows * (head_dim + 1))
    return fail(ADAKV_ERR_INVALID, "packed is NULL or part_stride %lld < rows * (head_dim + 1)",
                (long long)part_stride);
  if ((rc = check_view(out, "out", dtype, false))) return rc;
  CombineParams cp{};
  cp.parts = packed;
  cp.lse = packed + rows * head_dim;
  cp.part_stride = part_stride;
  cp.lse_stride = part_stride;
  cp.n_parts = n_parts;
  cp.rows = (int)rows;
  cp.D = head_dim;
  cp.out = to_view(out);
  cp.Hq = n_q_heads;
  LaunchOpts oc;
  oc.pdl = pdl_enabled();
  CUDA_TRY(launch_combine(cp, dtype, static_cast<cudaStream_t>(stream), oc));
  return ADAKV_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Sequence-sharded selection from exchanged statistics: no score rows cross
// between ranks, only per-head statistics, candidate lists and clamp terms.
// ---------------------------------------------------------------------------
namespace {

struct ShardGeo {
  int nb, cap, cap_pad, table_width;
  SelectCfg cfg;
  size_t record_bytes;
};

int shard_geo(const adakv_geometry* geo, const adakv_select_params* sp, ShardGeo* g) {
  int rc;
  if ((rc = check_geometry(geo))) return rc;
  if ((rc = check_params(sp))) return rc;
  if (geo->batch != 1)
    return fail(ADAKV_ERR_INVALID, "the sharded selection takes one sequence (batch %d)", geo->batch);
  if (sp->policy == ADAKV_POLICY_NUCLEUS)
    return fail(ADAKV_ERR_UNSUPPORTED,
                "the nucleus policy ranks the whole row's mass: exchange the rows (adakv_select)");
  g->cfg = to_cfg(sp);
  g->nb = ceil_div(geo->max_seq_len, geo->block_size);
  g->table_width = table_width_for(geo->nb_cap, g->cfg);
  const SeqBudget sb = seq_budget(g->nb, g->cfg);
  const int kmax = std::min(std::min(std::max(sb.hi, sb.floor_sel), g->nb), g->table_width);
  const int n_forced = (sb.sink + sb.local >= g->nb) ? g->nb : sb.sink + sb.local;
  g->cap = std::max(0, kmax - n_forced);
  if (g->cap > kShardListCap)
    return fail(ADAKV_ERR_UNSUPPORTED, "%d candidates per head exceed the sharded selection's %d",
                g->cap, kShardListCap);
  if (align_up((size_t)geo->n_q_heads * sizeof(double), 16) + kShardFinishStage > kShardFinishSmemMax)
    return fail(ADAKV_ERR_UNSUPPORTED, "n_q_heads %d too large for the sharded selection",
                geo->n_q_heads);
  g->cap_pad = (g->cap + 1) / 2 * 2;
  g->record_bytes = (size_t)geo->n_q_heads * (kShardStatD * sizeof(double) +
                                              (size_t)g->cap_pad * sizeof(unsigned long long));
  return ADAKV_OK;
}

int shard_range_ok(const ShardGeo& g, const float* scores, int32_t score_stride, int32_t block_lo,
                   int32_t n_local) {
  if (block_lo < 0 || n_local < 0 || (int64_t)block_lo + n_local > g.nb)
    return fail(ADAKV_ERR_INVALID, "shard [%d, %d + %d) outside the sequence's %d blocks", block_lo,
                block_lo, n_local, g.nb);
  if (n_local > 0 && (!scores || score_stride < n_local))
    return fail(ADAKV_ERR_INVALID, "scores is NULL or score_stride %d < n_local %d", score_stride,
                n_local);
  return ADAKV_OK;
}

int shard_records_ok(const ShardGeo& g, const void* records, size_t record_stride, int32_t world) {
  if (world < 1 || world > kShardMaxWorld)
    return fail(ADAKV_ERR_INVALID, "world %d outside [1, %d]", world, kShardMaxWorld);
  if (!records || reinterpret_cast<uintptr_t>(records) % 16 || record_stride % 16 ||
      record_stride < g.record_bytes)
    return fail(ADAKV_ERR_INVALID,
                "records must be 16-byte aligned, record_stride a multiple of 16 and >= %zu",
                g.record_bytes);
  return ADAKV_OK;
}

ShardSelParams shard_params(const adakv_geometry* geo, const ShardGeo& g, const float* scores,
                            int32_t score_stride, int32_t block_lo, int32_t n_local) {
  ShardSelParams p{};
  p.scores = scores;
  p.score_stride = score_stride;
  p.n_local = n_local;
  p.block_lo = block_lo;
  p.nb = g.nb;
  p.Hq = geo->n_q_heads;
  p.cfg = g.cfg;
  p.cap = g.cap;
  p.cap_pad = g.cap_pad;
  p.table_width = g.table_width;
  p.world = 1;
  return p;
}

}  // namespace

extern "C" {

size_t adakv_shard_record_bytes(const adakv_geometry* geo, const adakv_select_params* sp) {
  ShardGeo g;
  if (!geo || !sp || shard_geo(geo, sp, &g) != ADAKV_OK) return 0;
  return g.record_bytes;
}

int adakv_shard_prep(const adakv_geometry* geo, const adakv_select_params* sp, const float* scores,
                     int32_t score_stride, int32_t block_lo, int32_t n_local, void* record,
                     void* stream) {
  int rc;
  ShardGeo g;
  if ((rc = shard_geo(geo, sp, &g))) return rc;
  if ((rc = shard_range_ok(g, scores, score_stride, block_lo, n_local))) return rc;
  if (!record || reinterpret_cast<uintptr_t>(record) % 16)
    return fail(ADAKV_ERR_INVALID, "record must be a 16-byte aligned device pointer");
  DeviceState* ds = nullptr;
  if ((rc = device_state(&ds))) return rc;
  ShardSelParams p = shard_params(geo, g, scores, score_stride, block_lo, n_local);
  p.xmine = static_cast<unsigned char*>(record);
  LaunchOpts o;
  o.pdl = pdl_enabled();
  CUDA_TRY(launch_shard_select(0, p, static_cast<cudaStream_t>(stream), o));
  return ADAKV_OK;
}

int adakv_shard_clamp(const adakv_geometry* geo, const adakv_select_params* sp, const float* scores,
                      int32_t score_stride, int32_t block_lo, int32_t n_local, const void* records,
                      size_t record_stride, int32_t world, double* cc, void* stream) {
  int rc;
  ShardGeo g;
  if ((rc = shard_geo(geo, sp, &g))) return rc;
  if ((rc = shard_range_ok(g, scores, score_stride, block_lo, n_local))) return rc;
  if ((rc = shard_records_ok(g, records, record_stride, world))) return rc;
  if (!cc) return fail(ADAKV_ERR_INVALID, "cc is NULL");
  DeviceState* ds = nullptr;
  if ((rc = device_state(&ds))) return rc;
  ShardSelParams p = shard_params(geo, g, scores, score_stride, block_lo, n_local);
  p.xall = static_cast<const unsigned char*>(records);
  p.xstride = record_stride;
  p.world = world;
  p.cc_mine = cc;
  LaunchOpts o;
  o.pdl = pdl_enabled();
  CUDA_TRY(launch_shard_select(1, p, static_cast<cudaStream_t>(stream), o));
  return ADAKV_OK;
}

int adakv_shard_finish(const adakv_geometry* geo, const adakv_select_params* sp,
                       const void* records, size_t record_stride, const double* cc_all,
                       int32_t world, int32_t rank, int32_t block_lo, int32_t n_local,
                       int32_t* block_table, int32_t table_width, int32_t* sel_lens,
                       uint32_t* status, void* stream) {
  int rc;
  ShardGeo g;
  if ((rc = shard_geo(geo, sp, &g))) return rc;
  if (block_lo < 0 || n_local < 0 || (int64_t)block_lo + n_local > g.nb)
    return fail(ADAKV_ERR_INVALID, "shard [%d, %d + %d) outside the sequence's %d blocks", block_lo,
                block_lo, n_local, g.nb);
  if ((rc = shard_records_ok(g, records, record_stride, world))) return rc;
  if (rank < 0 || rank >= world) return fail(ADAKV_ERR_INVALID, "rank %d outside [0, %d)", rank, world);
  if (sp->policy == ADAKV_POLICY_ADAPTIVE && !cc_all)
    return fail(ADAKV_ERR_INVALID, "the adaptive policy needs every shard's clamp terms (cc_all)");
  if (!block_table || !sel_lens) return fail(ADAKV_ERR_INVALID, "block_table / sel_lens are NULL");
  if (table_width < g.table_width)
    return fail(ADAKV_ERR_INVALID, "table_width %d < required %d", table_width, g.table_width);
  DeviceState* ds = nullptr;
  if ((rc = device_state(&ds))) return rc;
  ShardSelParams p = shard_params(geo, g, nullptr, 0, block_lo, n_local);
  p.xall = static_cast<const unsigned char*>(records);
  p.xstride = record_stride;
  p.world = world;
  p.rank = rank;
  p.cc_all = cc_all;
  p.block_table = block_table;
  p.out_width = table_width;
  p.sel_lens = sel_lens;
  p.status = status;
  LaunchOpts o;
  o.pdl = pdl_enabled();
  CUDA_TRY(launch_shard_select(2, p, static_cast<cudaStream_t>(stream), o));
  return ADAKV_OK;
}

size_t adakv_peer_buffer_bytes(int32_t world, size_t slot_bytes) {
  if (world < 1 || world > kPeerMaxWorld || slot_bytes % 16) return 0;
  return peer_buffer_bytes(world, slot_bytes);
}

int adakv_peer_alloc(size_t bytes, void** ptr, void* handle) {
  if (!ptr || !handle || bytes == 0) return fail(ADAKV_ERR_INVALID, "ptr / handle NULL or bytes 0");
  *ptr = nullptr;
  void* p = nullptr;
  CUDA_TRY(cudaMalloc(&p, bytes));
  cudaError_t e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return fail(ADAKV_ERR_CUDA, "peer buffer set-up failed: %s", cudaGetErrorString(e));
  }
  *ptr = p;
  return ADAKV_OK;
}

int adakv_peer_free(void* ptr) {
  if (ptr) CUDA_TRY(cudaFree(ptr));
  return ADAKV_OK;
}

int adakv_peer_open(const void* handle, void** ptr) {
  if (!ptr || !handle) return fail(ADAKV_ERR_INVALID, "ptr / handle NULL");
  *ptr = nullptr;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  CUDA_TRY(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return ADAKV_OK;
}

int adakv_peer_close(void* ptr) {
  if (ptr) CUDA_TRY(cudaIpcCloseMemHandle(ptr));
  return ADAKV_OK;
}

int adakv_peer_exchange(const void* src, size_t bytes, void* const* dsts, int32_t world,
                        int32_t rank, size_t slot_bytes, void* local, uint32_t* status,
                        void* stream) {
  if (world < 1 || world > kPeerMaxWorld || rank < 0 || rank >= world)
    return fail(ADAKV_ERR_INVALID, "world %d / rank %d outside [1, %d] / [0, world)", world, rank,
                kPeerMaxWorld);
  if (!src || !dsts || !local || reinterpret_cast<uintptr_t>(src) % 16 ||
      reinterpret_cast<uintptr_t>(local) % 16)
    return fail(ADAKV_ERR_INVALID, "src, dsts and local are required; src and local 16-byte aligned");
  if (bytes % 16 || slot_bytes % 16 || bytes > slot_bytes)
    return fail(ADAKV_ERR_INVALID, "bytes (%zu) and slot_bytes (%zu) must be multiples of 16, "
                "bytes <= slot_bytes", bytes, slot_bytes);
  PeerParams p{};
  p.src = src;
  p.bytes = bytes;
  p.world = world;
  p.rank = rank;
  p.dsts = reinterpret_cast<unsigned char* const*>(dsts);
  p.slot_bytes = slot_bytes;
  p.local = static_cast<unsigned char*>(local);
  p.status = status;
  p.wait_ns = wait_limit_ns();
  LaunchOpts o;
  o.pdl = pdl_enabled();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  CUDA_TRY(launch_peer_put(p, st, o));
  CUDA_TRY(launch_peer_wait(p, st, o));
  return ADAKV_OK;
}

size_t adakv_importance_workspace_bytes(const adakv_geometry* geo, int32_t n_query) {
  if (!geo || n_query < 1 || geo->batch < 1 || geo->n_q_heads < 1) return 0;
  return 2 * sizeof(float) * (size_t)geo->batch * geo->n_q_heads * (size_t)n_query + 256;
}

int adakv_key_importance(const adakv_geometry* geo, const adakv_view* q, const adakv_view* k,
                         int32_t n_query, float sm_scale, float* importance, int32_t imp_stride,
                         void* workspace, size_t workspace_bytes, void* stream) {
  int rc;
  if ((rc = check_geometry(geo))) return rc;
  if ((rc = check_view(q, "q", geo->dtype, true))) return rc;
  if ((rc = check_view(k, "k", geo->dtype, true))) return rc;
  if (n_query < 1 || n_query > geo->max_seq_len)
    return fail(ADAKV_ERR_INVALID, "n_query must be in [1, max_seq_len] (got %d)", n_query);
  if (!importance || imp_stride < geo->max_seq_len)
    return fail(ADAKV_ERR_INVALID, "importance is NULL or imp_stride %d < max_seq_len %d", imp_stride,
                geo->max_seq_len);
  if (!(sm_scale > 0.f)) return fail(ADAKV_ERR_INVALID, "sm_scale must be > 0");
  if ((rc = check_workspace(workspace, workspace_bytes, adakv_importance_workspace_bytes(geo, n_query))))
    return rc;
  ImportanceParams p{};
  p.q = to_view(q);
  p.k = to_view(k);
  p.B = geo->batch;
  p.Hq = geo->n_q_heads;
  p.Hkv = geo->n_kv_heads;
  p.S = geo->max_seq_len;
  p.n_query = n_query;
  p.scale = sm_scale;
  p.row_m = static_cast<float*>(workspace);
  p.row_l = p.row_m + (size_t)geo->batch * geo->n_q_heads * n_query;
  p.imp = importance;
  p.imp_stride = imp_stride;
  CUDA_TRY(launch_importance(p, geo->dtype, geo->head_dim, static_cast<cudaStream_t>(stream)));
  return ADAKV_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// minmax (Quest) estimator: tables and scores; selection then runs through
// adakv_select and attention through adakv_attend
// ---------------------------------------------------------------------------
namespace {

int minmax_common(const adakv_geometry* geo, const float* kmin, const float* kmax) {
  int rc;
  if ((rc = check_geometry(geo))) return rc;
  if (!kmin || !kmax || reinterpret_cast<uintptr_t>(kmin) % 16 || reinterpret_cast<uintptr_t>(kmax) % 16)
    return fail(ADAKV_ERR_INVALID, "kmin / kmax must be 16-byte aligned device pointers");
  return ADAKV_OK;
}

MinmaxParams minmax_params(const adakv_geometry* geo, const int32_t* seq_lens, const float* kmin,
                           const float* kmax) {
  MinmaxParams p{};
  p.seq_lens = seq_lens;
  p.max_seq_len = geo->max_seq_len;
  p.B = geo->batch;
  p.Hq = geo->n_q_heads;
  p.Hkv = geo->n_kv_heads;
  p.g = geo->n_q_heads / geo->n_kv_heads;
  p.bs = geo->block_size;
  p.nb_cap = geo->nb_cap;
  p.kmin = const_cast<float*>(kmin);
  p.kmax = const_cast<float*>(kmax);
  return p;
}

}  // namespace

extern "C" {

int adakv_minmax_build(const adakv_geometry* geo, const adakv_view* k, const int32_t* seq_lens,
                       float* kmin, float* kmax, void* stream) {
  int rc;
  if ((rc = minmax_common(geo, kmin, kmax))) return rc;
  if ((rc = check_view(k, "k", geo->dtype, true))) return rc;
  MinmaxParams p = minmax_params(geo, seq_lens, kmin, kmax);
  p.k = to_view(k);
  CUDA_TRY(launch_minmax_build(p, geo->dtype, geo->head_dim, ceil_div(geo->max_seq_len, geo->block_size),
                               static_cast<cudaStream_t>(stream)));
  return ADAKV_OK;
}

int adakv_minmax_refresh(const adakv_geometry* geo, const adakv_view* k, int32_t n_new,
                         const int32_t* seq_lens, float* kmin, float* kmax, void* stream) {
  int rc;
  if ((rc = minmax_common(geo, kmin, kmax))) return rc;
  if ((rc = check_view(k, "k", geo->dtype, true))) return rc;
  if (n_new < 1 || n_new > geo->max_seq_len)
    return fail(ADAKV_ERR_INVALID, "n_new must be in [1, max_seq_len] (got %d)", n_new);
  MinmaxParams p = minmax_params(geo, seq_lens, kmin, kmax);
  p.k = to_view(k);
  p.n_new = n_new;
  CUDA_TRY(launch_minmax_build(p, geo->dtype, geo->head_dim, ceil_div(n_new, geo->block_size) + 1,
                               static_cast<cudaStream_t>(stream)));
  return ADAKV_OK;
}

int adakv_estimate_minmax(const adakv_geometry* geo, const adakv_view* q, const float* kmin,
                          const float* kmax, const int32_t* seq_lens, float* scores,
                          int32_t score_stride, void* stream) {
  int rc;
  if ((rc = minmax_common(geo, kmin, kmax))) return rc;
  if ((rc = check_view(q, "q", geo->dtype, false))) return rc;
  if (!scores) return fail(ADAKV_ERR_INVALID, "scores is NULL");
  if (score_stride < ceil_div(geo->max_seq_len, geo->block_size))
    return fail(ADAKV_ERR_INVALID, "score_stride %d < blocks of max_seq_len", score_stride);
  MinmaxParams p = minmax_params(geo, seq_lens, kmin, kmax);
  p.q = to_view(q);
  p.scores = scores;
  p.score_stride = score_stride;
  CUDA_TRY(launch_minmax_score(p, geo->dtype, geo->head_dim, ceil_div(geo->max_seq_len, geo->block_size),
                               static_cast<cudaStream_t>(stream)));
  return ADAKV_OK;
}

}  // extern "C"
