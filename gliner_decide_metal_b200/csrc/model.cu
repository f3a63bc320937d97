// Model load and forward orchestration.
//
// Load follows GLiNERDecideClassifier.init (DeBERTa.swift:188-242): every tensor is read
// from one safetensors file with the reference's key names, the QKV weights are
// concatenated q | k | v (DeBERTa.swift:129-136), LN(rel_embeddings) and the per-layer
// relative projections [PQ | PK] = LN(rel) [Wq; Wk]^T + [bq; bk] are computed once on the
// device with the same GEMM kernel the forward uses (DeBERTa.swift:204-227).
//
// The forward (DeBERTa.swift:274-447) runs on one CUDA stream with no host
// synchronisation: embedding -> 24 x (QKV GEMM, attention, out-proj GEMM, residual LN,
// FFN-up GEMM + GELU, FFN-down GEMM, residual LN) -> marker gather -> classifier GEMM +
// ReLU -> classifier dot + mask.
#include "model.h"

#include <algorithm>
#include <cstdlib>
#include <cmath>
#include <cstring>

#include "kernels/kernels.h"
#include "safetensors.h"

namespace gdc {

gdc_status launch_attention_simt(const __half* qkv, const __half* pos_qk, const __half* key_mask,
                                 const int32_t* rel_table, __half* ctx, int batch, int seq_len, int heads,
                                 cudaStream_t stream);

const char* profile_class_name(int c) {
  static const char* names[kProfCount] = {"embedding",  "qkv_gemm",      "attention",       "out_gemm",
                                          "layer_norm", "ffn_up_gemm",   "ffn_down_gemm",   "classifier"};
  return (c >= 0 && c < kProfCount) ? names[c] : "?";
}

void build_relative_table(int position_buckets, int max_relative_positions, int32_t* table) {
  // DeBERTa.swift:526-547 in double precision, then clip(bucket + 256, 0, 511)
  // (DeBERTa.swift:507-515). Index r + 511 for r = q - k in [-511, 511].
  const int mid = position_buckets / 2;
  const int span = position_buckets;
  for (int r = -511; r <= 511; ++r) {
    int abs_pos = (r > -mid && r < mid) ? mid - 1 : (r < 0 ? -r : r);
    const double lp = std::ceil(std::log(double(abs_pos) / double(mid)) /
                                std::log(double(max_relative_positions - 1) / double(mid)) * double(mid - 1));
    const int log_pos = int(lp) + mid;
    const int bucket = abs_pos <= mid ? r : log_pos * (r < 0 ? -1 : 1);
    int idx = bucket + span;
    if (idx < 0) idx = 0;
    if (idx > 2 * span - 1) idx = 2 * span - 1;
    table[r + 511] = idx;
  }
}

namespace {

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct PendingUpload {
  __half** dst;
  std::vector<uint16_t> host;
};

}  // namespace

gdc_status model_load(const char* path, const gdc_config* cfg_in, int device, gdc_model** out) {
  if (!path || !out) return set_error(GDC_ERR_NULL_POINTER, "gdc_model_load: null argument");
  *out = nullptr;
  gdc_config cfg;
  gdc_config_default(&cfg);
  if (cfg_in) cfg = *cfg_in;
  if (cfg.num_attention_heads <= 0 || cfg.hidden_size != cfg.num_attention_heads * 64)
    return set_error(GDC_ERR_UNSUPPORTED, "hidden_size must equal 64 * num_attention_heads (got %d, %d)",
                     cfg.hidden_size, cfg.num_attention_heads);
  if (cfg.hidden_size % 256 != 0 || cfg.hidden_size > 4096 || cfg.intermediate_size % 256 != 0 ||
      cfg.intermediate_size <= 0)
    return set_error(GDC_ERR_UNSUPPORTED, "hidden/intermediate sizes must be multiples of 256 (hidden <= 4096)");
  if (cfg.num_hidden_layers <= 0) return set_error(GDC_ERR_UNSUPPORTED, "num_hidden_layers must be positive");
  if (cfg.position_buckets != 256)
    return set_error(GDC_ERR_UNSUPPORTED, "position_buckets must be 256 (512-row relative table)");
  if (cfg.vocab_size <= 0) return set_error(GDC_ERR_UNSUPPORTED, "vocab_size must be positive");

  // Parse and validate the whole file on the host first: key / shape / dtype errors are
  // reported without touching the device.
  SafetensorsFile file;
  GDC_TRY(file.open(path));

  const int64_t E = cfg.hidden_size, F = cfg.intermediate_size;
  auto m = new gdc_model();
  m->device = device;
  m->cfg = cfg;
  m->hidden = int(E);
  m->heads = cfg.num_attention_heads;
  m->inter = int(F);
  m->layers_n = cfg.num_hidden_layers;
  m->vocab = cfg.vocab_size;
  m->eps = cfg.layer_norm_eps;
  {
    const char* v = std::getenv("GDC_PACK_ROWS");  // "0": dense rows by default
    m->pack_rows = !(v && v[0] == '0');
  }
  m->layers.resize(size_t(cfg.num_hidden_layers));

  std::vector<PendingUpload> ups;
  gdc_status st = GDC_OK;
  auto get = [&](const std::string& key, std::vector<int64_t> shape, __half** dst) -> gdc_status {
    PendingUpload u;
    u.dst = dst;
    gdc_status s = file.get_f16(key, &shape, &u.host);
    if (s != GDC_OK) return s;
    ups.push_back(std::move(u));
    return GDC_OK;
  };

  // classifier width from the file (DeBERTa.swift:228-229 does not constrain it)
  const TensorInfo* c0 = file.info("classifier.0.weight");
  if (!c0) {
    delete m;
    return set_error(GDC_ERR_MISSING_WEIGHT, "Missing model weight: classifier.0.weight");
  }
  if (c0->shape.size() != 2 || c0->shape[1] != E || c0->shape[0] <= 0 || c0->shape[0] % 256 != 0) {
    delete m;
    return set_error(GDC_ERR_INVALID_SHAPE, "Weight classifier.0.weight must be [d_c, %lld] with d_c %% 256 == 0",
                     (long long)E);
  }
  const int64_t DC = c0->shape[0];
  m->classifier_hidden = int(DC);

  do {
    if ((st = get("encoder.embeddings.word_embeddings.weight", {cfg.vocab_size, E}, &m->word_emb)) != GDC_OK) break;
    if ((st = get("encoder.embeddings.LayerNorm.weight", {E}, &m->emb_ln_g)) != GDC_OK) break;
    if ((st = get("encoder.embeddings.LayerNorm.bias", {E}, &m->emb_ln_b)) != GDC_OK) break;
    if ((st = get("encoder.encoder.rel_embeddings.weight", {512, E}, &m->rel_ln)) != GDC_OK) break;
    for (int i = 0; i < cfg.num_hidden_layers && st == GDC_OK; ++i) {
      const std::string p = "encoder.encoder.layer." + std::to_string(i);
      LayerWeights& L = m->layers[size_t(i)];
      // q, k, v are concatenated into one [3E, E] matrix below.
      std::vector<uint16_t> wq, wk, wv, bq, bk, bv;
      std::vector<int64_t> sw = {E, E}, sb = {E};
      if ((st = file.get_f16(p + ".attention.self.query_proj.weight", &sw, &wq)) != GDC_OK) break;
      if ((st = file.get_f16(p + ".attention.self.key_proj.weight", &sw, &wk)) != GDC_OK) break;
      if ((st = file.get_f16(p + ".attention.self.value_proj.weight", &sw, &wv)) != GDC_OK) break;
      if ((st = file.get_f16(p + ".attention.self.query_proj.bias", &sb, &bq)) != GDC_OK) break;
      if ((st = file.get_f16(p + ".attention.self.key_proj.bias", &sb, &bk)) != GDC_OK) break;
      if ((st = file.get_f16(p + ".attention.self.value_proj.bias", &sb, &bv)) != GDC_OK) break;
      PendingUpload uw, ub;
      uw.dst = &L.wqkv;
      uw.host.reserve(wq.size() * 3);
      uw.host.insert(uw.host.end(), wq.begin(), wq.end());
      uw.host.insert(uw.host.end(), wk.begin(), wk.end());
      uw.host.insert(uw.host.end(), wv.begin(), wv.end());
      ub.dst = &L.bqkv;
      ub.host.insert(ub.host.end(), bq.begin(), bq.end());
      ub.host.insert(ub.host.end(), bk.begin(), bk.end());
      ub.host.insert(ub.host.end(), bv.begin(), bv.end());
      ups.push_back(std::move(uw));
      ups.push_back(std::move(ub));
      if ((st = get(p + ".attention.output.dense.weight", {E, E}, &L.wo)) != GDC_OK) break;
      if ((st = get(p + ".attention.output.dense.bias", {E}, &L.bo)) != GDC_OK) break;
      if ((st = get(p + ".attention.output.LayerNorm.weight", {E}, &L.ln1_g)) != GDC_OK) break;
      if ((st = get(p + ".attention.output.LayerNorm.bias", {E}, &L.ln1_b)) != GDC_OK) break;
      if ((st = get(p + ".intermediate.dense.weight", {F, E}, &L.w1)) != GDC_OK) break;
      if ((st = get(p + ".intermediate.dense.bias", {F}, &L.b1)) != GDC_OK) break;
      if ((st = get(p + ".output.dense.weight", {E, F}, &L.w2)) != GDC_OK) break;
      if ((st = get(p + ".output.dense.bias", {E}, &L.b2)) != GDC_OK) break;
      if ((st = get(p + ".output.LayerNorm.weight", {E}, &L.ln2_g)) != GDC_OK) break;
      if ((st = get(p + ".output.LayerNorm.bias", {E}, &L.ln2_b)) != GDC_OK) break;
    }
    if (st) break;
    if ((st = get("classifier.0.weight", {DC, E}, &m->cls_w0)) != GDC_OK) break;
    if ((st = get("classifier.0.bias", {DC}, &m->cls_b0)) != GDC_OK) break;
    if ((st = get("classifier.2.weight", {1, DC}, &m->cls_w2)) != GDC_OK) break;
    if ((st = get("classifier.2.bias", {1}, &m->cls_b2)) != GDC_OK) break;
  } while (false);
  // LN(rel) scratch: the encoder LN params are needed only at load.
  std::vector<uint16_t> rel_g, rel_b;
  if (st == GDC_OK) {
    std::vector<int64_t> sb = {E};
    st = file.get_f16("encoder.encoder.LayerNorm.weight", &sb, &rel_g);
    if (st == GDC_OK) st = file.get_f16("encoder.encoder.LayerNorm.bias", &sb, &rel_b);
  }
  if (st != GDC_OK) {
    delete m;
    return st;
  }

  int ndev = 0;
  cudaError_t dc = cudaGetDeviceCount(&ndev);
  if (dc != cudaSuccess || device < 0 || device >= ndev) {
    delete m;
    return set_error(GDC_ERR_CUDA, "CUDA device %d not available (%s, %d devices)", device,
                     dc == cudaSuccess ? "ok" : cudaGetErrorString(dc), ndev);
  }

  // One pool: uploaded tensors, per-layer [512, 2E] relative projections, LN(rel) params,
  // relative table and the error word.
  size_t total = 0;
  for (auto& u : ups) total += align256(u.host.size() * 2);
  const size_t pos_bytes = align256(size_t(512) * 2 * E * 2);
  const size_t exp_bytes = align256(size_t(1023) * 2 * E * 2);
  total += (pos_bytes + exp_bytes) * size_t(cfg.num_hidden_layers);
  total += align256(E * 2) * 2 + align256(size_t(512) * E * 2) + align256(1023 * 4) + 256;

  auto fail = [&](gdc_status s) {
    model_free(m);
    return s;
  };
  cudaError_t ce = cudaSetDevice(device);
  if (ce != cudaSuccess) {
    delete m;
    return set_error(GDC_ERR_CUDA, "cudaSetDevice(%d): %s", device, cudaGetErrorString(ce));
  }
  ce = cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking);
  if (ce != cudaSuccess) {
    delete m;
    return set_error(GDC_ERR_CUDA, "cudaStreamCreate: %s", cudaGetErrorString(ce));
  }
  ce = cudaMalloc(&m->weight_pool, total);
  if (ce != cudaSuccess) {
    m->weight_pool = nullptr;
    return fail(set_error(GDC_ERR_OUT_OF_MEMORY, "cudaMalloc(%zu) for weights: %s", total, cudaGetErrorString(ce)));
  }
  uint8_t* cur = static_cast<uint8_t*>(m->weight_pool);
  for (auto& u : ups) {
    *u.dst = reinterpret_cast<__half*>(cur);
    ce = cudaMemcpy(cur, u.host.data(), u.host.size() * 2, cudaMemcpyHostToDevice);
    if (ce != cudaSuccess) return fail(set_error(GDC_ERR_CUDA, "weight upload: %s", cudaGetErrorString(ce)));
    cur += align256(u.host.size() * 2);
  }
  for (auto& L : m->layers) {
    L.pos_qk = reinterpret_cast<__half*>(cur);
    cur += pos_bytes;
    L.pos_exp = reinterpret_cast<__half*>(cur);
    cur += exp_bytes;
  }
  __half* rel_g_d = reinterpret_cast<__half*>(cur);
  cur += align256(E * 2);
  __half* rel_b_d = reinterpret_cast<__half*>(cur);
  cur += align256(E * 2);
  __half* rel_norm = reinterpret_cast<__half*>(cur);
  cur += align256(size_t(512) * E * 2);
  m->rel_table = reinterpret_cast<int32_t*>(cur);
  cur += align256(1023 * 4);
  m->err = reinterpret_cast<int*>(cur);

  int32_t table[1023];
  build_relative_table(cfg.position_buckets, 512, table);
  if ((ce = cudaMemcpy(m->rel_table, table, sizeof(table), cudaMemcpyHostToDevice)) != cudaSuccess ||
      (ce = cudaMemcpy(rel_g_d, rel_g.data(), E * 2, cudaMemcpyHostToDevice)) != cudaSuccess ||
      (ce = cudaMemcpy(rel_b_d, rel_b.data(), E * 2, cudaMemcpyHostToDevice)) != cudaSuccess ||
      (ce = cudaMemset(m->err, 0, 256)) != cudaSuccess)
    return fail(set_error(GDC_ERR_CUDA, "model upload: %s", cudaGetErrorString(ce)));

  // LN(rel_embeddings) (DeBERTa.swift:209-213) -> rel_norm; then per layer
  // [PQ | PK] = rel_norm . Wqkv[0:2E]^T + bqkv[0:2E] (DeBERTa.swift:218-227).
  st = launch_residual_layer_norm(m->rel_ln, nullptr, rel_g_d, rel_b_d, rel_norm, 512, int(E), m->eps, m->stream);
  if (st != GDC_OK) return fail(st);
  for (auto& L : m->layers) {
    st = launch_linear(rel_norm, E, L.wqkv, L.bqkv, L.pos_qk, 2 * E, 512, int(2 * E), int(E), kActNone, m->stream,
                       m->err);
    if (st != GDC_OK) return fail(st);
    st = launch_expand_positions(L.pos_qk, m->rel_table, L.pos_exp, int(2 * E), m->stream);
    if (st != GDC_OK) return fail(st);
  }
  // keep LN(rel) as the model's relative table copy (rel_ln aliases the raw upload slot)
  ce = cudaMemcpyAsync(m->rel_ln, rel_norm, size_t(512) * E * 2, cudaMemcpyDeviceToDevice, m->stream);
  if (ce != cudaSuccess) return fail(set_error(GDC_ERR_CUDA, "copy: %s", cudaGetErrorString(ce)));
  st = read_device_errors(m, m->stream);
  if (st != GDC_OK) return fail(st);
  *out = m;
  return GDC_OK;
}

void model_free(gdc_model* m) {
  if (!m) return;
  cudaSetDevice(m->device);
  if (m->stream) cudaStreamSynchronize(m->stream);
  Workspace& w = m->ws;
  for (void* p : {(void*)w.x, (void*)w.x1, (void*)w.big, (void*)w.ctx, (void*)w.tmp, (void*)w.mrows,
                  (void*)w.mhid, (void*)w.ids, (void*)w.mask, (void*)w.seq_off, (void*)w.rowmap,
                  (void*)w.row_order, (void*)w.ctrl,
                  (void*)w.marker_idx, (void*)w.marker_mask, (void*)w.logits, (void*)w.logits16})
    if (p) cudaFree(p);
  if (w.h_in) cudaFreeHost(w.h_in);
  if (w.h_out) cudaFreeHost(w.h_out);
  for (auto e : m->events) cudaEventDestroy(e);
  if (m->call_done) cudaEventDestroy(m->call_done);
  for (auto& g : m->graphs) release_graph(g);
  if (m->weight_pool) cudaFree(m->weight_pool);
  if (m->stream) cudaStreamDestroy(m->stream);
  delete m;
}

gdc_status ensure_workspace(gdc_model* m, int64_t tokens, int64_t markers) {
  Workspace& w = m->ws;
  const int64_t E = m->hidden;
  const int64_t big_cols = std::max<int64_t>(3 * E, m->inter);
  auto grow = [](void** p, size_t bytes) -> gdc_status {
    if (*p) cudaFree(*p);
    *p = nullptr;
    cudaError_t e = cudaMalloc(p, bytes);
    if (e != cudaSuccess) {
      *p = nullptr;
      return set_error(GDC_ERR_OUT_OF_MEMORY, "workspace cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
    }
    return GDC_OK;
  };
  if (tokens > w.tokens) {
    // grow geometrically to avoid reallocation churn across buckets
    int64_t cap = std::max<int64_t>(tokens, w.tokens * 2);
    cudaStreamSynchronize(m->stream);
    GDC_TRY(grow((void**)&w.x, size_t(cap) * E * 2));
    GDC_TRY(grow((void**)&w.x1, size_t(cap) * E * 2));
    GDC_TRY(grow((void**)&w.big, size_t(cap) * big_cols * 2));
    GDC_TRY(grow((void**)&w.ctx, size_t(cap) * E * 2));
    GDC_TRY(grow((void**)&w.tmp, size_t(cap) * E * 2));
    GDC_TRY(grow((void**)&w.ids, size_t(cap) * 4));
    GDC_TRY(grow((void**)&w.mask, size_t(cap) * 2));
    GDC_TRY(grow((void**)&w.seq_off, size_t(cap + 1) * 4));
    GDC_TRY(grow((void**)&w.rowmap, size_t(cap) * 4));
    GDC_TRY(grow((void**)&w.row_order, size_t(cap) * 4));
    if (!w.ctrl) GDC_TRY(grow((void**)&w.ctrl, 64 * 4));
    GDC_CUDA_TRY(cudaMemsetAsync(w.ctrl, 0, 64 * 4, m->stream));
    // With packed rows, GEMM tiles also read rows past the packed count that no kernel of the
    // call writes (their outputs are never read). Starting every activation buffer at zero
    // keeps them finite; the rows attention reads past the count are zeroed by the embedding
    // kernel on every call.
    for (void* p : {(void*)w.x, (void*)w.x1, (void*)w.ctx, (void*)w.tmp})
      GDC_CUDA_TRY(cudaMemsetAsync(p, 0, size_t(cap) * E * 2, m->stream));
    GDC_CUDA_TRY(cudaMemsetAsync(w.big, 0, size_t(cap) * big_cols * 2, m->stream));
    GDC_CUDA_TRY(cudaStreamSynchronize(m->stream));  // the forward may run on another stream
    w.tokens = cap;
    ++w.generation;
  }
  if (markers > w.markers) {
    int64_t cap = std::max<int64_t>(markers, w.markers * 2);
    cudaStreamSynchronize(m->stream);
    GDC_TRY(grow((void**)&w.mrows, size_t(cap) * E * 2));
    GDC_TRY(grow((void**)&w.mhid, size_t(cap) * m->classifier_hidden * 2));
    GDC_TRY(grow((void**)&w.marker_idx, size_t(cap) * 4));
    GDC_TRY(grow((void**)&w.marker_mask, size_t(cap) * 4));
    GDC_TRY(grow((void**)&w.logits, size_t(cap) * 4));
    GDC_TRY(grow((void**)&w.logits16, size_t(cap) * 2));
    w.markers = cap;
    ++w.generation;
  }
  return GDC_OK;
}

namespace {

// Records an event after the kernels of `cls` when profiling: on the stream (eager
// forwards, m->events), or as an event node of the graph being captured (graph->events).
struct StageRecorder {
  gdc_model* m;
  cudaStream_t s;
  bool on;
  bool named;
  ForwardGraph* graph = nullptr;
  void record(int cls) {
    if (graph != nullptr) {
      if (graph->events_used < graph->events.size()) {
        cudaEventRecordWithFlags(graph->events[graph->events_used], s, cudaEventRecordExternal);
        graph->event_class[graph->events_used] = cls;
        ++graph->events_used;
      }
      return;
    }
    if (m->events_used < m->events.size()) {
      cudaEventRecord(m->events[m->events_used], s);
      m->event_class[m->events_used] = cls;
      ++m->events_used;
    }
  }
  void begin() {
    if (on) record(-1);
  }
  void end(int cls, const std::string& name) {
    if (!on) return;
    record(cls);
    if (named && graph == nullptr) m->stage_names.push_back(name);
  }
};

}  // namespace

namespace {

// The kernel sequence of the forward (DeBERTa.swift:274-447) on stream s.
gdc_status enqueue_forward(gdc_model* m, int B, int L, int Hm, int O, const int32_t* ids, const __half* mask,
                           const int32_t* markers, const float* marker_mask, float* logits, __half* logits16,
                           cudaStream_t s, StageRecorder& rec, bool pack) {
  const int64_t T = int64_t(B) * L;
  const int64_t R = int64_t(B) * Hm * O;
  const int E = m->hidden, F = m->inter;
  Workspace& w = m->ws;
  // Packed rows: seq_off / rowmap from the mask and markers on the device; every encoder
  // kernel then reads the packed row count seq_off[B] (m_dev), the buffers keep their
  // B * L capacity and the launch shapes stay those of the dense grid.
  const int32_t* seq_off = nullptr;
  const int32_t* rowmap = nullptr;
  const int32_t* m_dev = nullptr;
  // attention CTAs take work items from the workspace counter (heaviest first when packed)
  AttentionWork work;
  work.counter = w.ctrl;
  rec.begin();
  if (pack) {
    GDC_TRY(launch_row_pack(mask, markers, marker_mask, B, L, Hm * O, w.seq_off, w.rowmap, w.row_order, w.ctrl + 8,
                            s));
    seq_off = w.seq_off;
    rowmap = w.rowmap;
    m_dev = w.seq_off + B;
    work.seq_off = w.seq_off;
    work.row_order = w.row_order;
    work.groups = w.ctrl + 8;
  }
  GDC_TRY(launch_embedding(ids, mask, m->word_emb, m->vocab, m->emb_ln_g, m->emb_ln_b, w.x, T, E, m->eps, s, m->err,
                           rowmap, m_dev, pack ? w.big : nullptr, 3 * E));
  rec.end(kProfEmbedding, "embedding");
  for (int i = 0; i < m->layers_n; ++i) {
    const LayerWeights& Lw = m->layers[size_t(i)];
    const std::string p = rec.named ? "layer_" + std::to_string(i) + "_" : std::string();
    GDC_TRY(launch_linear(w.x, E, Lw.wqkv, Lw.bqkv, w.big, 3 * E, T, 3 * E, E, kActNone, s, m->err, m_dev));
    rec.end(kProfQkvGemm, p + "attention_projection");
    GDC_TRY(launch_attention(w.big, Lw.pos_exp, mask, w.ctx, B, L, m->heads, s, m->err, work));
    rec.end(kProfAttention, p + "attention");
    GDC_TRY(launch_linear(w.ctx, E, Lw.wo, Lw.bo, w.tmp, E, T, E, E, kActNone, s, m->err, m_dev));
    rec.end(kProfOutGemm, "");
    GDC_TRY(launch_residual_layer_norm(w.tmp, w.x, Lw.ln1_g, Lw.ln1_b, w.x1, T, E, m->eps, s, m_dev));
    rec.end(kProfLayerNorm, p + "attention_output");
    GDC_TRY(launch_linear(w.x1, E, Lw.w1, Lw.b1, w.big, F, T, F, E, kActGelu, s, m->err, m_dev));
    rec.end(kProfFfnUpGemm, "");
    GDC_TRY(launch_linear(w.big, F, Lw.w2, Lw.b2, w.tmp, E, T, E, F, kActNone, s, m->err, m_dev));
    rec.end(kProfFfnDownGemm, "");
    GDC_TRY(launch_residual_layer_norm(w.tmp, w.x1, Lw.ln2_g, Lw.ln2_b, w.x, T, E, m->eps, s, m_dev));
    rec.end(kProfLayerNorm, p + "feed_forward");
  }
  GDC_TRY(launch_marker_gather(w.x, markers, w.mrows, int(R), Hm * O, L, E, s, m->err, seq_off));
  GDC_TRY(launch_linear(w.mrows, E, m->cls_w0, m->cls_b0, w.mhid, m->classifier_hidden, R, m->classifier_hidden, E,
                        kActRelu, s, m->err));
  GDC_TRY(launch_classifier_out(w.mhid, m->cls_w2, m->cls_b2, marker_mask, logits, logits16, int(R),
                                m->classifier_hidden, s));
  rec.end(kProfClassifier, "classifier");
  return GDC_OK;
}

bool graphs_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("GDC_GRAPHS");
    return !(v && v[0] == '0');
  }();
  return on;
}

// The graph slot of a shape (created on first use; the least recently used slot is
// recycled beyond 8 shapes).
ForwardGraph& graph_slot(gdc_model* m, int B, int L, int Hm, int O, bool packed, bool profiled) {
  for (auto& g : m->graphs)
    if (g.batch == B && g.seq_len == L && g.max_heads == Hm && g.max_options == O && g.packed == packed &&
        g.profiled == profiled)
      return g;
  ForwardGraph* slot = nullptr;
  if (m->graphs.size() >= 8) {
    auto it = std::min_element(m->graphs.begin(), m->graphs.end(),
                               [](const ForwardGraph& x, const ForwardGraph& y) { return x.last_use < y.last_use; });
    release_graph(*it);
    slot = &*it;
  } else {
    m->graphs.emplace_back();
    slot = &m->graphs.back();
  }
  slot->batch = B, slot->seq_len = L, slot->max_heads = Hm, slot->max_options = O, slot->packed = packed;
  slot->profiled = profiled;
  return *slot;
}

// Captures the forward of `g`'s shape on the workspace staging buffers (with one event node
// after every kernel group when g.profiled).
gdc_status capture_graph(gdc_model* m, ForwardGraph& g, cudaStream_t s) {
  Workspace& w = m->ws;
  if (g.exec) {
    cudaGraphExecDestroy(g.exec);
    g.exec = nullptr;
  }
  StageRecorder off{m, s, g.profiled, false};
  if (g.profiled) {
    const size_t need = size_t(7 * m->layers_n + 4);
    while (g.events.size() < need) {
      cudaEvent_t e;
      GDC_CUDA_TRY(cudaEventCreate(&e));
      g.events.push_back(e);
      g.event_class.push_back(-1);
    }
    g.events_used = 0;
    off.graph = &g;
  }
  GDC_CUDA_TRY(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
  const gdc_status st = enqueue_forward(m, g.batch, g.seq_len, g.max_heads, g.max_options, w.ids, w.mask,
                                        w.marker_idx, w.marker_mask, w.logits, w.logits16, s, off, g.packed);
  cudaGraph_t graph = nullptr;
  const cudaError_t ce = cudaStreamEndCapture(s, &graph);
  if (st != GDC_OK) {
    if (graph) cudaGraphDestroy(graph);
    return st;
  }
  if (ce != cudaSuccess) return set_error(GDC_ERR_CUDA, "forward graph capture: %s", cudaGetErrorString(ce));
  const cudaError_t ie = cudaGraphInstantiate(&g.exec, graph, 0);
  cudaGraphDestroy(graph);
  if (ie != cudaSuccess) {
    g.exec = nullptr;
    return set_error(GDC_ERR_CUDA, "forward graph instantiate: %s", cudaGetErrorString(ie));
  }
  g.generation = w.generation;
  return GDC_OK;
}

gdc_status copy_if_needed(void* dst, const void* src, size_t bytes, cudaStream_t s) {
  if (dst == src || bytes == 0) return GDC_OK;
  GDC_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, s));
  return GDC_OK;
}

}  // namespace

gdc_status forward(gdc_model* m, int B, int L, int Hm, int O, const int32_t* ids, const __half* mask,
                   const int32_t* markers, const float* marker_mask, float* logits, __half* logits16,
                   cudaStream_t s, bool named_stages, bool dense_hint) {
  const int64_t T = int64_t(B) * L;
  const bool pack = m->pack_rows && !dense_hint;
  const int64_t R = int64_t(B) * Hm * O;
  GDC_TRY(ensure_workspace(m, T, R));
  Workspace& w = m->ws;
  StageRecorder rec{m, s, m->profiling || named_stages, named_stages};
  if (rec.on && (named_stages || !graphs_enabled())) {
    // one event after every kernel group; make sure the pool is large enough
    const size_t need = m->events_used + size_t(7 * m->layers_n + 4);
    while (m->events.size() < need) {
      cudaEvent_t e;
      GDC_CUDA_TRY(cudaEventCreate(&e));
      m->events.push_back(e);
      m->event_class.push_back(-1);
    }
    return enqueue_forward(m, B, L, Hm, O, ids, mask, markers, marker_mask, logits, logits16, s, rec, pack);
  }
  if (!graphs_enabled())
    return enqueue_forward(m, B, L, Hm, O, ids, mask, markers, marker_mask, logits, logits16, s, rec, pack);
  // Replay path: the graph reads the workspace staging buffers and writes ws.logits /
  // ws.logits16, so caller buffers elsewhere are copied in and out around it. The first
  // call of a shape runs eagerly (one-time kernel attribute set-up happens outside any
  // capture); the second captures the graph.
  // With the stage profiler on (rec.on), a separate graph of the shape carries an event node
  // after every kernel group; each replay is synchronised and its intervals added to the
  // profiler's totals, so they measure the replayed kernels without eager launch gaps.
  const bool profiled = rec.on;
  if (profiled) {
    const size_t need = m->events_used + size_t(7 * m->layers_n + 4);
    while (m->events.size() < need) {
      cudaEvent_t e;
      GDC_CUDA_TRY(cudaEventCreate(&e));
      m->events.push_back(e);
      m->event_class.push_back(-1);
    }
  }
  ForwardGraph& g = graph_slot(m, B, L, Hm, O, pack, profiled);
  g.last_use = ++m->graph_clock;
  if (g.calls++ == 0)
    return enqueue_forward(m, B, L, Hm, O, ids, mask, markers, marker_mask, logits, logits16, s, rec, pack);
  if (g.exec == nullptr || g.generation != w.generation) GDC_TRY(capture_graph(m, g, s));
  GDC_TRY(copy_if_needed(w.ids, ids, size_t(T) * 4, s));
  GDC_TRY(copy_if_needed(w.mask, mask, size_t(T) * 2, s));
  GDC_TRY(copy_if_needed(w.marker_idx, markers, size_t(R) * 4, s));
  GDC_TRY(copy_if_needed(w.marker_mask, marker_mask, size_t(R) * 4, s));
  GDC_CUDA_TRY(cudaGraphLaunch(g.exec, s));
  GDC_TRY(copy_if_needed(logits, w.logits, size_t(R) * 4, s));
  if (logits16) GDC_TRY(copy_if_needed(logits16, w.logits16, size_t(R) * 2, s));
  if (profiled) {
    GDC_CUDA_TRY(cudaStreamSynchronize(s));
    for (size_t e = 1; e < g.events_used; ++e) {
      const int c = g.event_class[e];
      if (c < 0) continue;
      float ms = 0.f;
      GDC_CUDA_TRY(cudaEventElapsedTime(&ms, g.events[e - 1], g.events[e]));
      m->prof_ns[c] += double(ms) * 1e6;
      m->prof_launches[c] += 1;
    }
  }
  return GDC_OK;
}

void release_graph(ForwardGraph& g) {
  if (g.exec) cudaGraphExecDestroy(g.exec);
  for (auto e : g.events) cudaEventDestroy(e);
  g = ForwardGraph{};
}

void set_row_packing(gdc_model* m, bool on) {
  if (m->pack_rows == on) return;
  m->pack_rows = on;
  if (m->stream) cudaStreamSynchronize(m->stream);
  for (auto& g : m->graphs) release_graph(g);
  m->graphs.clear();
}

gdc_status read_device_errors(gdc_model* m, cudaStream_t s) {
  int h = 0;
  GDC_CUDA_TRY(cudaMemcpyAsync(&h, m->err, sizeof(int), cudaMemcpyDeviceToHost, s));
  GDC_CUDA_TRY(cudaStreamSynchronize(s));
  if (h != 0) {
    GDC_CUDA_TRY(cudaMemsetAsync(m->err, 0, sizeof(int), s));
    GDC_CUDA_TRY(cudaStreamSynchronize(s));
    if (h & kErrTimeout)
      return set_error(GDC_ERR_TIMEOUT, "a device-side wait exceeded its time limit (error word 0x%x)", h);
    if (h & kErrBadTokenId) return set_error(GDC_ERR_INVALID_INPUT, "input id outside [0, vocab) (device check)");
    if (h & kErrBadMarkerIndex)
      return set_error(GDC_ERR_INVALID_INPUT, "marker index outside [0, seq_len) (device check)");
    return set_error(GDC_ERR_CUDA, "device error word 0x%x", h);
  }
  return GDC_OK;
}

}  // namespace gdc
