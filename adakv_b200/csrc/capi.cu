// extern "C" entry points declared in include/adakv_b200.h.
//
// Host-side responsibilities: validate every argument before anything is
// launched (the reference raises ValueError / asserts in the same places,
// adakv/attention.py:192,200,226, adakv/runtime.py:97), derive the workspace
// layout, size grids from host-known bounds (no device->host synchronisation
// anywhere on the decode path), and enqueue the kernels on the caller's stream.
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
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
};
constexpr int kMaxDevices = 64;
DeviceState g_dev[kMaxDevices];
std::mutex g_dev_mu;

int device_state(DeviceState** out) {
  int dev = 0;
  CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(ADAKV_ERR_UNSUPPORTED, "device index %d", dev);
  std::lock_guard<std::mutex> lock(g_dev_mu);
  DeviceState& s = g_dev[dev];
  if (!s.ready) {
    CUDA_TRY(cudaDeviceGetAttribute(&s.num_sms, cudaDevAttrMultiProcessorCount, dev));
    CUDA_TRY(select_kernels_init());
    CUDA_TRY(attend_kernels_init());
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
  if (sp->policy != ADAKV_POLICY_FIXED && sp->policy != ADAKV_POLICY_ADAPTIVE)
    return fail(ADAKV_ERR_INVALID, "unknown budget_policy %d", sp->policy);
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

// Blocks per attend work item: 4 keeps ~500 items per 128K-token batch-1 step
// (several per SM); bounded by the shared-memory budget of one CTA.
int item_blocks_for(const adakv_geometry* g) {
  const size_t per_block = (size_t)g->block_size * g->head_dim * elt_size(g->dtype) * 2;
  int c = 4;
  while (c > 1 && (size_t)c * per_block > kAttendSmemMax) --c;
  return c;
}

WsLayout plan_layout(const adakv_geometry* g, int table_width) {
  return make_layout(g->batch, g->n_q_heads, g->head_dim, g->nb_cap, table_width,
                     item_blocks_for(g), true);
}

WsLayout attend_layout(const adakv_geometry* g, int table_width) {
  return make_layout(g->batch, g->n_q_heads, g->head_dim, g->nb_cap, table_width,
                     item_blocks_for(g), false);
}

template <typename T>
T* ws_at(void* ws, size_t off) {
  return reinterpret_cast<T*>(static_cast<char*>(ws) + off);
}

// Grid of the persistent attend kernel: enough CTAs for every work item the
// selection can produce (a tight bound for the plan path, where the per-head
// counts of a sequence sum to at most Hq * target + Hq / 2 + 1), capped at the
// number of co-resident CTAs.
int attend_grid(const DeviceState* ds, const adakv_geometry* g, const WsLayout& L,
                const adakv_select_params* sp) {
  int64_t items = L.items_cap;
  if (sp && sp->policy == ADAKV_POLICY_ADAPTIVE) {
    const SeqBudget sb = seq_budget(g->nb_cap, to_cfg(sp));
    if (sb.hi >= sb.lo) {
      const double per_seq = g->n_q_heads * sb.target + g->n_q_heads / 2.0 + 1.0;
      const int64_t tight =
          (int64_t)g->batch * ((int64_t)std::ceil(per_seq / L.item_blocks) + g->n_q_heads);
      if (tight < items) items = tight;
    }
  }
  const int64_t resident =
      (int64_t)ds->num_sms *
      attend_ctas_per_sm(g->dtype, g->head_dim, g->block_size, L.item_blocks);
  int64_t grid = items < resident ? items : resident;
  if (grid < 1) grid = 1;
  return (int)grid;
}

int check_workspace(void* ws, size_t bytes, size_t need) {
  if (!ws) return fail(ADAKV_ERR_INVALID, "workspace is NULL");
  if (reinterpret_cast<uintptr_t>(ws) % 256)
    return fail(ADAKV_ERR_INVALID, "workspace must be 256-byte aligned");
  if (bytes < need)
    return fail(ADAKV_ERR_INVALID, "workspace too small: %zu < %zu bytes", bytes, need);
  return ADAKV_OK;
}

// plan = estimator + budget + select (shared by adakv_plan and adakv_decode_step)
int enqueue_plan(const adakv_geometry* g, const adakv_select_params* sp, const adakv_view* q,
                 const float* centroid, const int32_t* seq_lens, int32_t* block_table,
                 int32_t table_width, int32_t* sel_lens, void* ws, const WsLayout& L,
                 cudaStream_t st) {
  const int nb_max = ceil_div(g->max_seq_len, g->block_size);
  uint32_t* status = ws_at<uint32_t>(ws, L.status);
  const SelectCfg cfg = to_cfg(sp);

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
  ep.chunkmax = ws_at<float>(ws, L.chunkmax);
  ep.chunks_cap = L.chunks_cap;
  ep.status = status;
  CUDA_TRY(launch_estimate(ep, g->dtype, g->head_dim, nb_max, st));

  BudgetParams bp{};
  bp.seq_lens = seq_lens;
  bp.max_seq_len = g->max_seq_len;
  bp.B = g->batch;
  bp.Hq = g->n_q_heads;
  bp.bs = g->block_size;
  bp.cfg = cfg;
  bp.scores = ep.scores;
  bp.score_stride = L.score_stride;
  bp.chunkmax = ep.chunkmax;
  bp.chunks_cap = L.chunks_cap;
  bp.weights = ws_at<double>(ws, L.weights);
  bp.seq_counter = ws_at<int>(ws, L.seq_counter);
  bp.glob_counter = ws_at<int>(ws, L.glob_counter);
  bp.sel_lens = sel_lens;
  bp.head_item_off = ws_at<int>(ws, L.head_item_off);
  bp.seq_items = ws_at<int>(ws, L.seq_items);
  bp.head_item_base = ws_at<int>(ws, L.head_item_base);
  bp.total_items = ws_at<int>(ws, L.total_items);
  bp.item_blocks = L.item_blocks;
  bp.status = status;
  CUDA_TRY(launch_budget(bp, st));

  SelectParams sp2{};
  sp2.seq_lens = seq_lens;
  sp2.max_seq_len = g->max_seq_len;
  sp2.B = g->batch;
  sp2.Hq = g->n_q_heads;
  sp2.bs = g->block_size;
  sp2.n_sink = sp->n_sink_blocks;
  sp2.n_local = sp->n_local_blocks;
  sp2.scores = ep.scores;
  sp2.score_stride = L.score_stride;
  sp2.sel_lens = sel_lens;
  sp2.block_table = block_table;
  sp2.table_width = table_width;
  sp2.head_item_base = bp.head_item_base;
  sp2.work_hdr = ws_at<int4>(ws, L.work_hdr);
  sp2.work_blk = ws_at<int>(ws, L.work_blk);
  sp2.item_blocks = L.item_blocks;
  sp2.status = status;
  CUDA_TRY(launch_select(sp2, nb_max, st));
  return ADAKV_OK;
}

AttendParams attend_params(const adakv_geometry* g, const adakv_view* q, const adakv_view* k,
                           const adakv_view* v, const adakv_view* out, const int32_t* seq_lens,
                           float sm_scale, const int32_t* block_table, int32_t table_width,
                           const int32_t* sel_lens, void* ws, const WsLayout& L) {
  AttendParams ap{};
  ap.q = to_view(q);
  ap.k = to_view(k);
  ap.v = to_view(v);
  ap.out = to_view(out);
  ap.seq_lens = seq_lens;
  ap.max_seq_len = g->max_seq_len;
  ap.B = g->batch;
  ap.Hq = g->n_q_heads;
  ap.g = g->n_q_heads / g->n_kv_heads;
  ap.sm_scale = sm_scale;
  ap.block_table = block_table;
  ap.table_width = table_width;
  ap.sel_lens = sel_lens;
  ap.work_hdr = ws_at<int4>(ws, L.work_hdr);
  ap.work_blk = ws_at<int>(ws, L.work_blk);
  ap.total_items = ws_at<int>(ws, L.total_items);
  ap.item_blocks = L.item_blocks;
  ap.head_item_base = ws_at<int>(ws, L.head_item_base);
  ap.work_hdr_w = ws_at<int4>(ws, L.work_hdr);
  ap.work_blk_w = ws_at<int>(ws, L.work_blk);
  ap.total_items_w = ws_at<int>(ws, L.total_items);
  ap.head_counter = ws_at<int>(ws, L.head_counter);
  ap.part_ml = ws_at<float2>(ws, L.part_ml);
  ap.part_o = ws_at<float>(ws, L.part_o);
  ap.status = ws_at<uint32_t>(ws, L.status);
  return ap;
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
  return plan_layout(geo, table_width_for(geo->nb_cap, to_cfg(sp))).bytes;
}

size_t adakv_attend_workspace_bytes(const adakv_geometry* geo, int32_t table_width) {
  if (check_geometry(geo)) return 0;
  if (table_width < 1) {
    fail(ADAKV_ERR_INVALID, "table_width must be >= 1");
    return 0;
  }
  return attend_layout(geo, table_width).bytes;
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
  const WsLayout L = plan_layout(geo, table_width);
  if ((rc = check_workspace(workspace, workspace_bytes, L.bytes))) return rc;
  DeviceState* ds = nullptr;
  if ((rc = device_state(&ds))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((rc = enqueue_plan(geo, sp, q, centroid, seq_lens, block_table, table_width, sel_lens,
                         workspace, L, st)))
    return rc;
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
  const WsLayout L = attend_layout(geo, table_width);
  if ((rc = check_workspace(workspace, workspace_bytes, L.bytes))) return rc;
  DeviceState* ds = nullptr;
  if ((rc = device_state(&ds))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  AttendParams ap = attend_params(geo, q, k, v, out, seq_lens, sm_scale, block_table, table_width,
                                  sel_lens, workspace, L);
  CUDA_TRY(launch_items(ap, st));
  CUDA_TRY(launch_attend(ap, geo->dtype, geo->head_dim, geo->block_size,
                         attend_grid(ds, geo, L, nullptr), st));
  return ADAKV_OK;
}

int adakv_decode_step(const adakv_geometry* geo, const adakv_select_params* sp,
                      const adakv_view* q, const adakv_view* k, const adakv_view* v,
                      const float* centroid, const int32_t* seq_lens, float sm_scale,
                      int32_t* block_table, int32_t table_width, int32_t* sel_lens,
                      const adakv_view* out, void* workspace, size_t workspace_bytes,
                      void* stream) {
  int rc;
  if ((rc = check_geometry(geo))) return rc;
  if ((rc = check_params(sp))) return rc;
  if ((rc = check_attend_views(geo, q, k, v, out))) return rc;
  if (!centroid || reinterpret_cast<uintptr_t>(centroid) % 16)
    return fail(ADAKV_ERR_INVALID, "centroid must be a 16-byte aligned device pointer");
  if (!block_table || !sel_lens) return fail(ADAKV_ERR_INVALID, "block_table / sel_lens are NULL");
  if (!std::isfinite(sm_scale)) return fail(ADAKV_ERR_INVALID, "sm_scale must be finite");
  const int need_w = table_width_for(geo->nb_cap, to_cfg(sp));
  if (table_width < need_w)
    return fail(ADAKV_ERR_INVALID, "table_width %d < required %d", table_width, need_w);
  const WsLayout L = plan_layout(geo, table_width);
  if ((rc = check_workspace(workspace, workspace_bytes, L.bytes))) return rc;
  DeviceState* ds = nullptr;
  if ((rc = device_state(&ds))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((rc = enqueue_plan(geo, sp, q, centroid, seq_lens, block_table, table_width, sel_lens,
                         workspace, L, st)))
    return rc;
  AttendParams ap = attend_params(geo, q, k, v, out, seq_lens, sm_scale, block_table, table_width,
                                  sel_lens, workspace, L);
  CUDA_TRY(launch_attend(ap, geo->dtype, geo->head_dim, geo->block_size,
                         attend_grid(ds, geo, L, sp), st));
  return ADAKV_OK;
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
