// Device-resident model: weights, per-layer relative projections, workspace and the
// forward pass of GLiNERDecideClassifier (DeBERTa.swift:156-447).
#pragma once

#include <cstdint>
#include <mutex>
#include <string>
#include <vector>

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.h"

namespace gdc {

struct LayerWeights {
  __half* wqkv = nullptr;  // [3E, E] rows q | k | v (DeBERTa.swift:129-136)
  __half* bqkv = nullptr;  // [3E]
  __half* wo = nullptr;    // [E, E]
  __half* bo = nullptr;
  __half* ln1_g = nullptr;
  __half* ln1_b = nullptr;
  __half* w1 = nullptr;    // [F, E]
  __half* b1 = nullptr;
  __half* w2 = nullptr;    // [E, F]
  __half* b2 = nullptr;
  __half* ln2_g = nullptr;
  __half* ln2_b = nullptr;
  __half* pos_qk = nullptr;  // [512, 2E]: PQ | PK (DeBERTa.swift:218-227)
  __half* pos_exp = nullptr; // [1023, 2E]: pos_exp[r + 511] = pos_qk[i(r)] (attention's expanded table)
};

// Kernel groups recorded by the stage profiler.
enum ProfileClass : int {
  kProfEmbedding = 0,
  kProfQkvGemm,
  kProfAttention,
  kProfOutGemm,
  kProfLayerNorm,
  kProfFfnUpGemm,
  kProfFfnDownGemm,
  kProfClassifier,
  kProfCount
};

const char* profile_class_name(int c);

struct Workspace {
  int64_t tokens = 0;   // capacity in B*L rows
  int64_t markers = 0;  // capacity in B*Hm*O rows
  __half* x = nullptr;      // [T, E] hidden
  __half* x1 = nullptr;     // [T, E] hidden after the attention block
  __half* big = nullptr;    // [T, max(3E, F)] QKV projection, later FFN intermediate
  __half* ctx = nullptr;    // [T, E]
  __half* tmp = nullptr;    // [T, E] projection outputs before residual LN
  __half* mrows = nullptr;  // [R, E] gathered marker rows
  __half* mhid = nullptr;   // [R, dc] classifier hidden
  // input / output staging (device)
  int32_t* ids = nullptr;
  __half* mask = nullptr;
  // packed-row layout (kernels/pack.cu): seq_off [B + 1] (seq_off[B] = packed row count),
  // rowmap [T] packed row -> dense position b * L + t
  int32_t* seq_off = nullptr;
  int32_t* rowmap = nullptr;
  int32_t* row_order = nullptr;  // [B] attention work order (kernels/pack.cu)
  // [64] small control block: [0, 2) attention work counter (zero between launches),
  // [8, 13) attention work groups
  int32_t* ctrl = nullptr;
  int32_t* marker_idx = nullptr;
  float* marker_mask = nullptr;
  float* logits = nullptr;
  __half* logits16 = nullptr;
  // pinned host staging
  uint8_t* h_in = nullptr;
  size_t h_in_bytes = 0;
  uint8_t* h_out = nullptr;
  size_t h_out_bytes = 0;
  int generation = 0;  // bumped whenever a device buffer above is reallocated
};

// A captured forward for one input shape, replayed with cudaGraphLaunch. It reads the
// workspace staging buffers (ids, mask, marker_idx, marker_mask) and writes
// ws.logits / ws.logits16; valid while the workspace generation is unchanged.
struct ForwardGraph {
  int batch = 0, seq_len = 0, max_heads = 0, max_options = 0;
  bool packed = false;  // row layout the graph was captured with
  // profiled: the graph also records an event node after every kernel group (the stage
  // profiler's intervals, measured on the replayed graph instead of eager launches)
  bool profiled = false;
  int generation = -1;
  int calls = 0;                  // eager calls seen for this shape (captured on the second)
  cudaGraphExec_t exec = nullptr;
  uint64_t last_use = 0;
  std::vector<cudaEvent_t> events;  // profiled graphs: the event of every node, in order
  std::vector<int> event_class;     // class of the interval ending at events[i] (-1: none)
  size_t events_used = 0;
};

// Destroys a captured forward and its events, leaving an empty slot.
void release_graph(ForwardGraph& g);

}  // namespace gdc

struct gdc_model {
  int device = 0;
  gdc_config cfg{};
  int hidden = 1024;
  int heads = 16;
  int inter = 4096;
  int layers_n = 24;
  int64_t vocab = 128011;
  int classifier_hidden = 2048;
  float eps = 1e-7f;
  // Encoder rows: packed (only positions [0, ext_b) of each batch row, see
  // kernels/pack.cu) or the dense [B, L] grid. Both give bit-identical logits.
  bool pack_rows = true;

  cudaStream_t stream = nullptr;
  cudaEvent_t call_done = nullptr;  // end of the last gdc_classify_device on a caller's stream
  std::mutex mu;

  void* weight_pool = nullptr;
  __half* word_emb = nullptr;
  __half* emb_ln_g = nullptr;
  __half* emb_ln_b = nullptr;
  __half* rel_ln = nullptr;  // LN(rel_embeddings) [512, E]
  __half* cls_w0 = nullptr;
  __half* cls_b0 = nullptr;
  __half* cls_w2 = nullptr;
  __half* cls_b2 = nullptr;
  std::vector<gdc::LayerWeights> layers;
  int32_t* rel_table = nullptr;  // [1023]
  int* err = nullptr;            // device error word

  gdc::Workspace ws;

  // captured forwards (small LRU keyed by input shape); GDC_GRAPHS=0 disables them
  std::vector<gdc::ForwardGraph> graphs;
  uint64_t graph_clock = 0;

  // stage profiler (events bracket kernel groups)
  bool profiling = false;
  std::vector<cudaEvent_t> events;
  std::vector<int> event_class;  // class of the interval ending at events[i]
  size_t events_used = 0;
  double prof_ns[gdc::kProfCount] = {};
  int64_t prof_launches[gdc::kProfCount] = {};
  // named stage events for gdc_classify(collect_profile) (reference stage names)
  std::vector<std::string> stage_names;
};

namespace gdc {

gdc_status model_load(const char* path, const gdc_config* cfg, int device, gdc_model** out);
void model_free(gdc_model* m);

// Ensures workspace for `tokens` rows and `markers` marker rows.
gdc_status ensure_workspace(gdc_model* m, int64_t tokens, int64_t markers);

// Runs the forward on device-resident inputs (ws or caller buffers) on `stream`.
// named_stages: record the reference's stage events into m->stage_names / events.
// dense_hint: the caller knows this batch has no padding past any row's last valid position,
// so packed rows would save nothing; the call then runs on the dense grid.
gdc_status forward(gdc_model* m, int batch, int seq_len, int max_heads, int max_options, const int32_t* ids,
                   const __half* mask, const int32_t* markers, const float* marker_mask, float* logits,
                   __half* logits16, cudaStream_t stream, bool named_stages, bool dense_hint = false);

// Switches between packed and dense encoder rows; drops captured forwards when it changes.
void set_row_packing(gdc_model* m, bool on);

// Reads and clears the device error word (synchronises `stream`).
gdc_status read_device_errors(gdc_model* m, cudaStream_t stream);

// Host-side relative index table (DeBERTa.swift:521-551), 1023 entries.
void build_relative_table(int position_buckets, int max_relative_positions, int32_t* table);

}  // namespace gdc
