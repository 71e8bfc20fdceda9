// Launch-parameter structs and launcher entry points shared by the kernel
// translation units and the C-ABI layer (capi.cu).
#pragma once

#include "common.cuh"

namespace adakv {

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

struct EstParams {
  View q;                 // [B, Hq, D]
  const float* cent;      // [B, Hkv, nb_cap, D]
  int nb_cap;
  const int* seq_lens;
  int max_seq_len;
  int B, Hq, Hkv, g, bs;
  float* scores;          // [B, Hq, score_stride]
  int score_stride;
  float* chunkmax;        // [B, Hq, chunks_cap]
  int chunks_cap;
  uint32_t* status;
};

struct BudgetParams {
  const int* seq_lens;
  int max_seq_len;
  int B, Hq, bs;
  SelectCfg cfg;
  const float* scores;
  int score_stride;
  const float* chunkmax;
  int chunks_cap;
  double* weights;          // [B*Hq]
  int* seq_counter;         // [B]   zero between calls
  int* glob_counter;        //       zero between calls
  int* sel_lens;            // [B*Hq] out: realised count per head
  int* head_item_off;       // [B*Hq] seq-local exclusive prefix of items
  int* seq_items;           // [B+1]  per-seq totals, then global bases
  int* head_item_base;      // [B*Hq] global index of the head's first item
  int* total_items;
  int item_blocks;
  uint32_t* status;
};

struct SelectParams {
  const int* seq_lens;
  int max_seq_len;
  int B, Hq, bs;
  int n_sink, n_local;
  const float* scores;
  int score_stride;
  const int* sel_lens;
  int* block_table;         // [B*Hq, table_width]
  int table_width;
  const int* head_item_base;
  int4* work_hdr;           // {b, h, head_item_base, count}
  int* work_blk;            // [items, item_blocks]
  int item_blocks;
  uint32_t* status;
};

struct AttendParams {
  View q, k, v, out;
  const int* seq_lens;
  int max_seq_len;
  int B, Hq, g;
  float sm_scale;
  const int* block_table;   // only for the stand-alone item builder
  int table_width;
  const int* sel_lens;
  const int4* work_hdr;
  const int* work_blk;
  const int* total_items;
  int item_blocks;
  int* head_item_base;      // item builder output
  int4* work_hdr_w;
  int* work_blk_w;
  int* total_items_w;
  int* head_counter;        // [B*Hq], zero between calls
  float2* part_ml;
  float* part_o;
  uint32_t* status;
};

// shared memory one select CTA may stage (keys); larger rows re-read L2
constexpr int kSelectSmemMaxKeys = 50 * 1024;
// shared memory budget of one attend CTA (K + V tiles of an item)
constexpr size_t kAttendSmemMax = 200 * 1024;

cudaError_t launch_centroid(const CentroidParams& p, int dtype, int D, int blocks_per_seq,
                            cudaStream_t stream);
cudaError_t launch_estimate(const EstParams& p, int dtype, int D, int nb_max, cudaStream_t stream);
cudaError_t launch_budget(const BudgetParams& p, cudaStream_t stream);
cudaError_t launch_select(const SelectParams& p, int nb_max, cudaStream_t stream);
cudaError_t launch_attend(const AttendParams& p, int dtype, int D, int bs, int grid,
                          cudaStream_t stream);
cudaError_t launch_items(const AttendParams& p, cudaStream_t stream);

// once per device (current device): opt-in shared memory sizes
cudaError_t select_kernels_init();
cudaError_t attend_kernels_init();
// attend CTAs resident per SM for this element type / head dim / block size / item size
int attend_ctas_per_sm(int dtype, int D, int bs, int item_blocks);

}  // namespace adakv
