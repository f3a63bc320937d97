// C ABI implementation (include/gdc.h): argument checking, host staging, the host-side
// layout / decode logic of the reference, and dispatch to the device runtime.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <mutex>
#include <set>
#include <thread>
#include <vector>

#include <cuda_fp16.h>

#include "common.h"
#include "kernels/kernels.h"
#include "model.h"

namespace gdc {

gdc_status launch_attention_simt(const __half* qkv, const __half* pos_qk, const __half* key_mask,
                                 const int32_t* rel_table, __half* ctx, int batch, int seq_len, int heads,
                                 cudaStream_t stream);

namespace {
thread_local std::string g_last_error;

// Per-device error word for the kernel-level entry points (no model handle).
std::mutex g_err_mu;
int* g_err_words[64] = {};

gdc_status device_error_word(int** out) {
  int dev = 0;
  GDC_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return set_error(GDC_ERR_CUDA, "device ordinal out of range");
  std::lock_guard<std::mutex> lk(g_err_mu);
  if (!g_err_words[dev]) {
    int* p = nullptr;
    GDC_CUDA_TRY(cudaMalloc(&p, 256));
    GDC_CUDA_TRY(cudaMemset(p, 0, 256));
    g_err_words[dev] = p;
  }
  *out = g_err_words[dev];
  return GDC_OK;
}

size_t dtype_bytes(gdc_dtype d) {
  switch (d) {
    case GDC_INT32:
    case GDC_FLOAT32:
      return 4;
    case GDC_INT64:
      return 8;
    case GDC_FLOAT16:
      return 2;
    case GDC_UINT8:
      return 1;
  }
  return 0;
}

// Reads element i of a host array of dtype d as double.
double read_value(const void* p, gdc_dtype d, int64_t i) {
  switch (d) {
    case GDC_INT32:
      return double(static_cast<const int32_t*>(p)[i]);
    case GDC_INT64:
      return double(static_cast<const int64_t*>(p)[i]);
    case GDC_FLOAT16:
      return double(__half2float(__ushort_as_half(static_cast<const uint16_t*>(p)[i])));
    case GDC_FLOAT32:
      return double(static_cast<const float*>(p)[i]);
    case GDC_UINT8:
      return double(static_cast<const uint8_t*>(p)[i]);
  }
  return 0.0;
}

bool read_int(const void* p, gdc_dtype d, int64_t i, int64_t* out) {
  if (d == GDC_INT32) {
    *out = static_cast<const int32_t*>(p)[i];
    return true;
  }
  if (d == GDC_INT64) {
    *out = static_cast<const int64_t*>(p)[i];
    return true;
  }
  return false;
}

gdc_status check_input_shape(const gdc_input* in) {
  if (!in) return set_error(GDC_ERR_NULL_POINTER, "input is null");
  if (!in->input_ids || !in->attention_mask || !in->marker_indices || !in->marker_mask)
    return set_error(GDC_ERR_NULL_POINTER, "input arrays must be non-null");
  if (in->batch <= 0 || in->seq_len <= 0 || in->max_heads <= 0 || in->max_options <= 0)
    return set_error(GDC_ERR_INVALID_INPUT, "input dimensions must be positive (B=%d L=%d Hm=%d O=%d)", in->batch,
                     in->seq_len, in->max_heads, in->max_options);
  if (in->ids_dtype != GDC_INT32 && in->ids_dtype != GDC_INT64)
    return set_error(GDC_ERR_INVALID_INPUT, "input_ids must be int32 or int64");
  if (in->marker_dtype != GDC_INT32 && in->marker_dtype != GDC_INT64)
    return set_error(GDC_ERR_INVALID_INPUT, "marker_indices must be int32 or int64");
  if (dtype_bytes(in->mask_dtype) == 0 || dtype_bytes(in->marker_mask_dtype) == 0)
    return set_error(GDC_ERR_INVALID_INPUT, "unknown mask dtype");
  if (in->seq_len > 512)
    return set_error(GDC_ERR_UNSUPPORTED, "seq_len %d exceeds 512 (the relative-position table size)", in->seq_len);
  return GDC_OK;
}

// Converts a host gdc_input into the device staging layout (int32 ids, fp16 mask,
// int32 markers, fp32 marker mask rounded through fp16 as the reference compares it).
// Copies n integer ids of type S into dst as int32 and reports whether all lie in [0, hi).
template <typename S>
bool copy_ids_in_range(const void* src, int64_t n, int64_t hi, int32_t* dst) {
  const S* s = static_cast<const S*>(src);
  bool ok = true;
  for (int64_t i = 0; i < n; ++i) {
    const S v = s[i];
    ok &= v >= 0 && int64_t(v) < hi;
    dst[i] = int32_t(v);
  }
  return ok;
}

// Typed staging for the common dtypes: int32 / int64 ids and markers are range-checked and
// narrowed in one pass, an fp16 mask is copied as is (fp16 -> float -> fp16 is the identity)
// and a u8 mask goes through a 256-entry fp16 table; marker-mask values 0 and 1 are exact in
// fp16. Returns false (nothing reported) when a value is out of range or a dtype has no fast
// path; the element-wise pass below then stages the input and names the first bad value.
bool stage_input_fast(gdc_model* m, const gdc_input* in, int64_t T, int64_t R, int32_t* ids, uint16_t* mask,
                      int32_t* mk, float* mm) {
  bool ok;
  if (in->ids_dtype == GDC_INT32)
    ok = copy_ids_in_range<int32_t>(in->input_ids, T, m->vocab, ids);
  else if (in->ids_dtype == GDC_INT64)
    ok = copy_ids_in_range<int64_t>(in->input_ids, T, m->vocab, ids);
  else
    return false;
  if (!ok) return false;
  if (in->marker_dtype == GDC_INT32)
    ok = copy_ids_in_range<int32_t>(in->marker_indices, R, in->seq_len, mk);
  else if (in->marker_dtype == GDC_INT64)
    ok = copy_ids_in_range<int64_t>(in->marker_indices, R, in->seq_len, mk);
  else
    return false;
  if (!ok) return false;
  if (in->mask_dtype == GDC_FLOAT16) {
    std::memcpy(mask, in->attention_mask, size_t(T) * 2);
  } else if (in->mask_dtype == GDC_UINT8) {
    static const std::vector<uint16_t> table = [] {
      std::vector<uint16_t> t(256);
      for (int v = 0; v < 256; ++v) t[size_t(v)] = __half_as_ushort(__float2half_rn(float(v)));
      return t;
    }();
    const uint8_t* s = static_cast<const uint8_t*>(in->attention_mask);
    for (int64_t i = 0; i < T; ++i) mask[i] = table[s[i]];
  } else {
    return false;
  }
  if (in->marker_mask_dtype != GDC_FLOAT32) return false;
  const float* s = static_cast<const float*>(in->marker_mask);
  for (int64_t i = 0; i < R; ++i) {
    const float v = s[i];
    mm[i] = (v == 0.f || v == 1.f) ? v : __half2float(__float2half_rn(v));
  }
  return true;
}

gdc_status stage_input(gdc_model* m, const gdc_input* in, uint8_t* dst) {
  const int64_t T = int64_t(in->batch) * in->seq_len;
  const int64_t R = int64_t(in->batch) * in->max_heads * in->max_options;
  int32_t* ids = reinterpret_cast<int32_t*>(dst);
  uint16_t* mask = reinterpret_cast<uint16_t*>(dst + T * 4);
  int32_t* mk = reinterpret_cast<int32_t*>(dst + T * 6);
  float* mm = reinterpret_cast<float*>(dst + T * 6 + R * 4);
  if (stage_input_fast(m, in, T, R, ids, mask, mk, mm)) return GDC_OK;
  for (int64_t i = 0; i < T; ++i) {
    int64_t v = 0;
    read_int(in->input_ids, in->ids_dtype, i, &v);
    if (v < 0 || v >= m->vocab)
      return set_error(GDC_ERR_INVALID_INPUT, "input_ids[%lld] = %lld is outside [0, %lld)", (long long)i,
                       (long long)v, (long long)m->vocab);
    ids[i] = int32_t(v);
    mask[i] = __half_as_ushort(__float2half_rn(float(read_value(in->attention_mask, in->mask_dtype, i))));
  }
  for (int64_t i = 0; i < R; ++i) {
    int64_t v = 0;
    read_int(in->marker_indices, in->marker_dtype, i, &v);
    if (v < 0 || v >= in->seq_len)
      return set_error(GDC_ERR_INVALID_INPUT, "marker_indices[%lld] = %lld is outside [0, %d)", (long long)i,
                       (long long)v, in->seq_len);
    mk[i] = int32_t(v);
    mm[i] = __half2float(__float2half_rn(float(read_value(in->marker_mask, in->marker_mask_dtype, i))));
  }
  return GDC_OK;
}

gdc_status ensure_pinned(uint8_t** p, size_t* cap, size_t bytes) {
  if (*cap >= bytes) return GDC_OK;
  if (*p) cudaFreeHost(*p);
  *p = nullptr;
  *cap = 0;
  size_t want = std::max(bytes, size_t(1) << 16);
  GDC_CUDA_TRY(cudaMallocHost(reinterpret_cast<void**>(p), want));
  *cap = want;
  return GDC_OK;
}

}  // namespace

gdc_status set_error(gdc_status st, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return st;
}

void clear_error() { g_last_error.clear(); }

uint16_t f32_to_f16_bits(float f) { return __half_as_ushort(__float2half_rn(f)); }
float f16_bits_to_f32(uint16_t h) { return __half2float(__ushort_as_half(h)); }

}  // namespace gdc

using namespace gdc;

extern "C" {

void gdc_config_default(gdc_config* c) {
  if (!c) return;
  std::memset(c, 0, sizeof(*c));
  c->hidden_size = 1024;
  c->intermediate_size = 4096;
  c->num_hidden_layers = 24;
  c->num_attention_heads = 16;
  c->layer_norm_eps = 1e-7f;
  c->position_buckets = 256;
  c->max_relative_positions = -1;
  c->pad_token_id = 0;
  c->vocab_size = 128011;
  c->use_fast_attention = 1;
}

const char* gdc_last_error(void) { return g_last_error.c_str(); }

int gdc_abi_version(void) { return GDC_ABI_VERSION; }

const char* gdc_build_info(void) {
  return "gliner-decide-metal B200 backend; sm_100a tcgen05/TMA kernels; nvcc " __DATE__;
}

gdc_status gdc_model_load(const char* path, const gdc_config* cfg, int device, gdc_model** out) {
  clear_error();
  return model_load(path, cfg, device, out);
}

void gdc_model_free(gdc_model* m) { model_free(m); }

int gdc_model_device(const gdc_model* m) { return m ? m->device : -1; }

int gdc_model_classifier_hidden(const gdc_model* m) { return m ? m->classifier_hidden : -1; }

void* gdc_model_stream(gdc_model* m) { return m ? static_cast<void*>(m->stream) : nullptr; }

gdc_status gdc_classify(gdc_model* m, const gdc_input* in, int collect_profile, gdc_output* out) {
  clear_error();
  const auto t0 = std::chrono::steady_clock::now();
  if (!m || !out) return set_error(GDC_ERR_NULL_POINTER, "gdc_classify: null model or output");
  if (!out->logits) return set_error(GDC_ERR_NULL_POINTER, "output->logits must be non-null");
  GDC_TRY(check_input_shape(in));
  std::lock_guard<std::mutex> lk(m->mu);
  GDC_CUDA_TRY(cudaSetDevice(m->device));
  const int64_t T = int64_t(in->batch) * in->seq_len;
  const int64_t R = int64_t(in->batch) * in->max_heads * in->max_options;
  Workspace& w = m->ws;
  const size_t in_bytes = size_t(T) * 6 + size_t(R) * 8;
  GDC_TRY(ensure_pinned(&w.h_in, &w.h_in_bytes, in_bytes));
  GDC_TRY(ensure_pinned(&w.h_out, &w.h_out_bytes, size_t(R) * 6 + 64));
  GDC_TRY(stage_input(m, in, w.h_in));
  GDC_TRY(ensure_workspace(m, T, R));
  cudaStream_t s = m->stream;
  GDC_CUDA_TRY(cudaMemcpyAsync(w.ids, w.h_in, size_t(T) * 4, cudaMemcpyHostToDevice, s));
  GDC_CUDA_TRY(cudaMemcpyAsync(w.mask, w.h_in + T * 4, size_t(T) * 2, cudaMemcpyHostToDevice, s));
  GDC_CUDA_TRY(cudaMemcpyAsync(w.marker_idx, w.h_in + T * 6, size_t(R) * 4, cudaMemcpyHostToDevice, s));
  GDC_CUDA_TRY(cudaMemcpyAsync(w.marker_mask, w.h_in + T * 6 + R * 4, size_t(R) * 4, cudaMemcpyHostToDevice, s));
  const size_t ev0 = m->events_used;
  if (collect_profile) m->stage_names.clear();
  const bool prev_prof = m->profiling;
  if (collect_profile) m->profiling = false;  // named stages only
  // Packed rows only pay off when some row ends in padding; the staged fp16 mask says so.
  bool dense_hint = true;
  const uint16_t* mask16 = reinterpret_cast<const uint16_t*>(w.h_in + T * 4);
  for (int32_t b = 0; b < in->batch && dense_hint; ++b)
    dense_hint = f16_bits_to_f32(mask16[int64_t(b) * in->seq_len + in->seq_len - 1]) > 0.f;
  gdc_status st = forward(m, in->batch, in->seq_len, in->max_heads, in->max_options, w.ids, w.mask, w.marker_idx,
                          w.marker_mask, w.logits, w.logits16, s, collect_profile != 0, dense_hint);
  m->profiling = prev_prof;
  if (st != GDC_OK) return st;
  GDC_CUDA_TRY(cudaMemcpyAsync(w.h_out, w.logits, size_t(R) * 4, cudaMemcpyDeviceToHost, s));
  GDC_CUDA_TRY(cudaMemcpyAsync(w.h_out + R * 4, w.logits16, size_t(R) * 2, cudaMemcpyDeviceToHost, s));
  // the error word rides along into the pinned buffer (one synchronisation for both); a
  // nonzero word is read again, cleared and reported by read_device_errors
  const int* h_err = reinterpret_cast<const int*>(w.h_out + ((size_t(R) * 6 + 3) & ~size_t(3)));
  GDC_CUDA_TRY(cudaMemcpyAsync(const_cast<int*>(h_err), m->err, sizeof(int), cudaMemcpyDeviceToHost, s));
  GDC_CUDA_TRY(cudaStreamSynchronize(s));
  if (*h_err != 0) GDC_TRY(read_device_errors(m, s));
  std::memcpy(out->logits, w.h_out, size_t(R) * 4);
  if (out->logits_f16) std::memcpy(out->logits_f16, w.h_out + R * 4, size_t(R) * 2);
  out->events_count = 0;
  if (collect_profile) {
    // Merge kernel-group intervals into the reference's named stages.
    double acc = 0.0;
    size_t name_i = 0;
    for (size_t e = ev0 + 1; e < m->events_used; ++e) {
      float ms = 0.f;
      cudaEventElapsedTime(&ms, m->events[e - 1], m->events[e]);
      acc += double(ms) * 1e6;
      const std::string& nm = name_i < m->stage_names.size() ? m->stage_names[name_i] : std::string();
      ++name_i;
      if (nm.empty()) continue;
      if (out->events && out->events_count < out->events_capacity) {
        gdc_profile_event& ev = out->events[out->events_count++];
        std::snprintf(ev.name, sizeof(ev.name), "%s", nm.c_str());
        ev.nanoseconds = uint64_t(acc);
      }
      acc = 0.0;
    }
    m->events_used = ev0;
  }
  out->wall_ns = uint64_t(std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0)
                              .count());
  return GDC_OK;
}

gdc_status gdc_classify_device(gdc_model* m, int32_t B, int32_t L, int32_t Hm, int32_t O, const int32_t* ids,
                               const uint16_t* mask, const int32_t* markers, const float* marker_mask, float* logits,
                               uint16_t* logits16, void* stream) {
  clear_error();
  if (!m || !ids || !mask || !markers || !marker_mask || !logits)
    return set_error(GDC_ERR_NULL_POINTER, "gdc_classify_device: null argument");
  if (B <= 0 || L <= 0 || Hm <= 0 || O <= 0) return set_error(GDC_ERR_INVALID_INPUT, "dimensions must be positive");
  if (L > 512) return set_error(GDC_ERR_UNSUPPORTED, "seq_len %d exceeds 512", L);
  std::lock_guard<std::mutex> lk(m->mu);
  GDC_CUDA_TRY(cudaSetDevice(m->device));
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : m->stream;
  GDC_TRY(forward(m, B, L, Hm, O, ids, reinterpret_cast<const __half*>(mask), markers, marker_mask, logits,
                  reinterpret_cast<__half*>(logits16), s, false));
  if (s != m->stream) {
    // order the model's stream after this forward, so gdc_check_errors (which synchronises
    // the model's stream) reads the error word only once this forward has finished with it
    if (m->call_done == nullptr) GDC_CUDA_TRY(cudaEventCreateWithFlags(&m->call_done, cudaEventDisableTiming));
    GDC_CUDA_TRY(cudaEventRecord(m->call_done, s));
    GDC_CUDA_TRY(cudaStreamWaitEvent(m->stream, m->call_done, 0));
  }
  return GDC_OK;
}

gdc_status gdc_check_errors(gdc_model* m) {
  clear_error();
  if (!m) return set_error(GDC_ERR_NULL_POINTER, "null model");
  std::lock_guard<std::mutex> lk(m->mu);
  GDC_CUDA_TRY(cudaSetDevice(m->device));
  GDC_CUDA_TRY(cudaStreamSynchronize(m->stream));
  return read_device_errors(m, m->stream);
}

gdc_status gdc_model_set_row_packing(gdc_model* m, int enabled) {
  if (!m) return set_error(GDC_ERR_NULL_POINTER, "null model");
  std::lock_guard<std::mutex> lk(m->mu);
  cudaSetDevice(m->device);
  set_row_packing(m, enabled != 0);
  return GDC_OK;
}

int gdc_model_row_packing(const gdc_model* m) { return m && m->pack_rows ? 1 : 0; }

gdc_status gdc_profile_enable(gdc_model* m, int enabled) {
  if (!m) return set_error(GDC_ERR_NULL_POINTER, "null model");
  std::lock_guard<std::mutex> lk(m->mu);
  m->profiling = enabled != 0;
  return GDC_OK;
}

gdc_status gdc_profile_reset(gdc_model* m) {
  if (!m) return set_error(GDC_ERR_NULL_POINTER, "null model");
  std::lock_guard<std::mutex> lk(m->mu);
  m->events_used = 0;
  for (int c = 0; c < kProfCount; ++c) {
    m->prof_ns[c] = 0.0;
    m->prof_launches[c] = 0;
  }
  return GDC_OK;
}

int gdc_profile_read(gdc_model* m, gdc_profile_event* events, int capacity, int32_t* launches) {
  if (!m) return 0;
  std::lock_guard<std::mutex> lk(m->mu);
  cudaSetDevice(m->device);
  for (size_t e = 1; e < m->events_used; ++e) {
    const int c = m->event_class[e];
    if (c < 0) continue;
    if (cudaEventSynchronize(m->events[e]) != cudaSuccess) break;
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, m->events[e - 1], m->events[e]) != cudaSuccess) continue;
    m->prof_ns[c] += double(ms) * 1e6;
    m->prof_launches[c] += (c == kProfLayerNorm || c == kProfClassifier) ? 1 : 1;
  }
  m->events_used = 0;
  int n = 0;
  for (int c = 0; c < kProfCount && n < capacity; ++c) {
    if (events) {
      std::snprintf(events[n].name, sizeof(events[n].name), "%s", profile_class_name(c));
      events[n].nanoseconds = uint64_t(m->prof_ns[c]);
    }
    if (launches) launches[n] = int32_t(m->prof_launches[c]);
    ++n;
  }
  return n;
}

gdc_status gdc_classify_sharded(gdc_model* const* models, int n, const gdc_input* in, gdc_output* out,
                                gdc_status* per_device) {
  clear_error();
  if (!models || n <= 0 || !out || !out->logits) return set_error(GDC_ERR_NULL_POINTER, "gdc_classify_sharded: null");
  GDC_TRY(check_input_shape(in));
  for (int i = 0; i < n; ++i)
    if (!models[i]) return set_error(GDC_ERR_NULL_POINTER, "model %d is null", i);
  const int B = in->batch;
  const int per_row_ids = in->seq_len;
  const int per_row_mk = in->max_heads * in->max_options;
  std::vector<gdc_status> st(size_t(n), GDC_OK);
  std::vector<std::string> msg(static_cast<size_t>(n));
  std::vector<std::thread> th;
  const auto t0 = std::chrono::steady_clock::now();
  int start = 0;
  for (int i = 0; i < n; ++i) {
    const int rows = B / n + (i < B % n ? 1 : 0);
    const int s0 = start;
    start += rows;
    if (rows == 0) continue;
    th.emplace_back([&, i, s0, rows] {
      gdc_input sub = *in;
      sub.batch = rows;
      sub.input_ids = static_cast<const uint8_t*>(in->input_ids) + size_t(s0) * per_row_ids * dtype_bytes(in->ids_dtype);
      sub.attention_mask =
          static_cast<const uint8_t*>(in->attention_mask) + size_t(s0) * per_row_ids * dtype_bytes(in->mask_dtype);
      sub.marker_indices =
          static_cast<const uint8_t*>(in->marker_indices) + size_t(s0) * per_row_mk * dtype_bytes(in->marker_dtype);
      sub.marker_mask =
          static_cast<const uint8_t*>(in->marker_mask) + size_t(s0) * per_row_mk * dtype_bytes(in->marker_mask_dtype);
      gdc_output o{};
      o.logits = out->logits + size_t(s0) * per_row_mk;
      o.logits_f16 = out->logits_f16 ? out->logits_f16 + size_t(s0) * per_row_mk : nullptr;
      st[size_t(i)] = gdc_classify(models[i], &sub, 0, &o);
      if (st[size_t(i)] != GDC_OK) msg[size_t(i)] = gdc_last_error();
    });
  }
  for (auto& t : th) t.join();
  out->wall_ns = uint64_t(
      std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0).count());
  out->events_count = 0;
  int failed = 0;
  std::string all;
  for (int i = 0; i < n; ++i) {
    if (per_device) per_device[i] = st[size_t(i)];
    if (st[size_t(i)] != GDC_OK) {
      ++failed;
      all += "device " + std::to_string(models[i]->device) + ": " + msg[size_t(i)] + "; ";
    }
  }
  if (failed == 0) return GDC_OK;
  if (failed == n) {
    gdc_status first = st[0];
    for (int i = 0; i < n; ++i)
      if (st[size_t(i)] != GDC_OK) {
        first = st[size_t(i)];
        break;
      }
    set_error(first, "%s", all.c_str());
    return first;
  }
  return set_error(GDC_ERR_PARTIAL, "%d of %d devices failed: %s", failed, n, all.c_str());
}

gdc_status gdc_decode(const float* logits, int32_t B, int32_t Hm, int32_t O, const int32_t* n_labels,
                      const uint8_t* multi_label, double* probs, uint8_t* selected) {
  clear_error();
  if (!logits || !n_labels || !multi_label || !probs || !selected)
    return set_error(GDC_ERR_NULL_POINTER, "gdc_decode: null argument");
  if (B <= 0 || Hm <= 0 || O <= 0) return set_error(GDC_ERR_INVALID_INPUT, "gdc_decode: bad dimensions");
  for (int64_t t = 0; t < int64_t(B) * Hm; ++t) {
    const float* x = logits + t * O;
    double* p = probs + t * O;
    uint8_t* s = selected + t * O;
    for (int o = 0; o < O; ++o) {
      p[o] = 0.0;
      s[o] = 0;
    }
    int n = n_labels[t];
    if (n <= 0) continue;
    if (n > O) return set_error(GDC_ERR_INVALID_INPUT, "n_labels[%lld] = %d exceeds max_options %d", (long long)t, n, O);
    if (multi_label[t]) {
      bool any = false;
      int best = 0;
      for (int o = 0; o < n; ++o) {
        p[o] = 1.0 / (1.0 + std::exp(-double(x[o])));
        if (p[o] >= 0.5) {
          s[o] = 1;
          any = true;
        }
        if (p[o] > p[best]) best = o;
      }
      if (!any) s[best] = 1;
    } else {
      double mx = double(x[0]);
      for (int o = 1; o < n; ++o) mx = std::max(mx, double(x[o]));
      double sum = 0.0;
      for (int o = 0; o < n; ++o) {
        p[o] = std::exp(double(x[o]) - mx);
        sum += p[o];
      }
      int best = 0;
      for (int o = 0; o < n; ++o) {
        p[o] /= sum;
        if (p[o] > p[best]) best = o;
      }
      s[best] = 1;
    }
  }
  return GDC_OK;
}

gdc_status gdc_decode_device(gdc_model* m, const float* logits, int32_t B, int32_t Hm, int32_t O,
                             const int32_t* n_labels, const uint8_t* multi_label, float* probs, uint8_t* selected,
                             void* stream) {
  clear_error();
  if (!m || !logits || !n_labels || !multi_label || !probs || !selected)
    return set_error(GDC_ERR_NULL_POINTER, "gdc_decode_device: null argument");
  if (B <= 0 || Hm <= 0 || O <= 0) return set_error(GDC_ERR_INVALID_INPUT, "gdc_decode_device: bad dimensions");
  GDC_CUDA_TRY(cudaSetDevice(m->device));
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : m->stream;
  return launch_decode(logits, B, Hm, O, n_labels, multi_label, probs, selected, s);
}

gdc_status gdc_select_bucket(int32_t len, const int32_t* buckets, int32_t n, int32_t* selected) {
  clear_error();
  if (!selected || (n > 0 && !buckets)) return set_error(GDC_ERR_NULL_POINTER, "gdc_select_bucket: null argument");
  std::set<int32_t> ordered;
  for (int i = 0; i < n; ++i) ordered.insert(buckets[i]);
  if (ordered.empty()) return set_error(GDC_ERR_INPUT_DOES_NOT_FIT, "Encoded schema/text does not fit any requested bucket: []");
  for (int32_t b : ordered)
    if (b >= len) {
      *selected = b;
      return GDC_OK;
    }
  std::string list = "[";
  for (int32_t b : ordered) list += (list.size() > 1 ? ", " : "") + std::to_string(b);
  list += "]";
  return set_error(GDC_ERR_INPUT_DOES_NOT_FIT, "Encoded schema/text does not fit any requested bucket: %s",
                   list.c_str());
}

gdc_status gdc_layout_row(const int32_t* token_ids, int32_t n_tokens, const int32_t* marker_positions,
                          const int32_t* marker_offsets, int32_t n_tasks, const int32_t* buckets, int32_t n_buckets,
                          int32_t pad_id, int32_t* bucket_len, int32_t* max_heads, int32_t* max_options,
                          int32_t* ids_out, int32_t ids_capacity, float* mask_out, int32_t* marker_out,
                          float* marker_mask_out, int32_t marker_capacity) {
  clear_error();
  if (!bucket_len || !max_heads || !max_options || (n_tokens > 0 && !token_ids))
    return set_error(GDC_ERR_NULL_POINTER, "gdc_layout_row: null argument");
  // NativeTokenizer.swift:81-84: at least one task, every task with at least one label.
  if (n_tasks <= 0 || !marker_offsets) return set_error(GDC_ERR_NO_TASK_LABELS, "Every decision task must contain at least one label");
  for (int t = 0; t < n_tasks; ++t)
    if (marker_offsets[t + 1] - marker_offsets[t] <= 0)
      return set_error(GDC_ERR_NO_TASK_LABELS, "Every decision task must contain at least one label");
  if (!marker_positions) return set_error(GDC_ERR_NULL_POINTER, "gdc_layout_row: null marker positions");
  int32_t L = 0;
  GDC_TRY(gdc_select_bucket(n_tokens, buckets, n_buckets, &L));
  int32_t O = 1;
  for (int t = 0; t < n_tasks; ++t) O = std::max(O, marker_offsets[t + 1] - marker_offsets[t]);
  const int32_t Hm = std::max(n_tasks, 1);
  *bucket_len = L;
  *max_heads = Hm;
  *max_options = O;
  if (!ids_out || !mask_out || !marker_out || !marker_mask_out || ids_capacity < L || marker_capacity < Hm * O)
    return set_error(GDC_ERR_INVALID_INPUT, "gdc_layout_row: output buffers too small (need %d ids, %d markers)", L,
                     Hm * O);
  for (int i = 0; i < L; ++i) {
    ids_out[i] = i < n_tokens ? token_ids[i] : pad_id;
    mask_out[i] = i < n_tokens ? 1.0f : 0.0f;
  }
  for (int i = 0; i < Hm * O; ++i) {
    marker_out[i] = 0;
    marker_mask_out[i] = 0.0f;
  }
  for (int t = 0; t < n_tasks; ++t)
    for (int j = marker_offsets[t]; j < marker_offsets[t + 1]; ++j) {
      const int o = j - marker_offsets[t];
      if (o < O) {
        marker_out[t * O + o] = marker_positions[j];
        marker_mask_out[t * O + o] = 1.0f;
      }
    }
  return GDC_OK;
}

gdc_status gdc_relative_index_table(int32_t position_buckets, int32_t max_relative_positions, int32_t* table_out) {
  clear_error();
  if (!table_out) return set_error(GDC_ERR_NULL_POINTER, "null table");
  if (position_buckets != 256 || max_relative_positions != 512)
    return set_error(GDC_ERR_UNSUPPORTED, "only position_buckets=256, max_relative_positions=512 are used");
  build_relative_table(position_buckets, max_relative_positions, table_out);
  return GDC_OK;
}

gdc_status gdc_residual_layer_norm(const uint16_t* x, const uint16_t* residual, const uint16_t* weight,
                                   const uint16_t* bias, uint16_t* out, int64_t rows, int32_t cols, float eps,
                                   void* stream) {
  clear_error();
  if (!x || !weight || !bias || !out) return set_error(GDC_ERR_NULL_POINTER, "gdc_residual_layer_norm: null argument");
  return launch_residual_layer_norm(reinterpret_cast<const __half*>(x), reinterpret_cast<const __half*>(residual),
                                    reinterpret_cast<const __half*>(weight), reinterpret_cast<const __half*>(bias),
                                    reinterpret_cast<__half*>(out), rows, cols, eps, static_cast<cudaStream_t>(stream));
}

namespace {

// Relative index table on the current device for the kernel-level entry points.
gdc_status device_rel_table(int32_t** out) {
  static std::mutex mu;
  static int32_t* tables[64] = {};
  int dev = 0;
  GDC_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return set_error(GDC_ERR_CUDA, "device ordinal out of range");
  std::lock_guard<std::mutex> lk(mu);
  if (!tables[dev]) {
    int32_t host[1023];
    build_relative_table(256, 512, host);
    int32_t* d = nullptr;
    GDC_CUDA_TRY(cudaMalloc(&d, sizeof(host)));
    GDC_CUDA_TRY(cudaMemcpy(d, host, sizeof(host), cudaMemcpyHostToDevice));
    tables[dev] = d;
  }
  *out = tables[dev];
  return GDC_OK;
}

gdc_status check_attention_args(const uint16_t* qkv, const uint16_t* pos_qk, const uint16_t* key_mask,
                                 const uint16_t* ctx, int32_t batch, int32_t seq_len, int32_t heads) {
  if (!qkv || !pos_qk || !key_mask || !ctx) return set_error(GDC_ERR_NULL_POINTER, "attention: null argument");
  if (heads != 16) return set_error(GDC_ERR_UNSUPPORTED, "heads must be 16 (hidden 1024)");
  if (batch <= 0 || seq_len <= 0 || seq_len > 512)
    return set_error(GDC_ERR_INVALID_INPUT, "attention: batch > 0 and seq_len in [1, 512] required");
  return GDC_OK;
}

}  // namespace

gdc_status gdc_disentangled_attention(const uint16_t* qkv, const uint16_t* pos_qk, const uint16_t* key_mask,
                                      uint16_t* ctx, int32_t batch, int32_t seq_len, int32_t heads, void* stream) {
  clear_error();
  GDC_TRY(check_attention_args(qkv, pos_qk, key_mask, ctx, batch, seq_len, heads));
  int* err = nullptr;
  int32_t* table = nullptr;
  GDC_TRY(device_error_word(&err));
  GDC_TRY(device_rel_table(&table));
  // the expanded position table of this call, from the stream-ordered allocator
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  __half* pos_exp = nullptr;
  GDC_CUDA_TRY(cudaMallocAsync(reinterpret_cast<void**>(&pos_exp), expanded_position_bytes(heads), s));
  gdc_status st = launch_expand_positions(reinterpret_cast<const __half*>(pos_qk), table, pos_exp, 2 * heads * 64, s);
  if (st == GDC_OK)
    st = launch_attention(reinterpret_cast<const __half*>(qkv), pos_exp, reinterpret_cast<const __half*>(key_mask),
                          reinterpret_cast<__half*>(ctx), batch, seq_len, heads, s, err);
  const cudaError_t fe = cudaFreeAsync(pos_exp, s);
  if (st != GDC_OK) return st;
  if (fe != cudaSuccess) return set_error(GDC_ERR_CUDA, "cudaFreeAsync: %s", cudaGetErrorString(fe));
  return GDC_OK;
}

gdc_status gdc_disentangled_attention_scalar(const uint16_t* qkv, const uint16_t* pos_qk, const uint16_t* key_mask,
                                             uint16_t* ctx, int32_t batch, int32_t seq_len, int32_t heads,
                                             void* stream) {
  clear_error();
  GDC_TRY(check_attention_args(qkv, pos_qk, key_mask, ctx, batch, seq_len, heads));
  int32_t* table = nullptr;
  GDC_TRY(device_rel_table(&table));
  return launch_attention_simt(reinterpret_cast<const __half*>(qkv), reinterpret_cast<const __half*>(pos_qk),
                               reinterpret_cast<const __half*>(key_mask), table, reinterpret_cast<__half*>(ctx), batch,
                               seq_len, heads, static_cast<cudaStream_t>(stream));
}

gdc_status gdc_linear(const uint16_t* a, const uint16_t* w, const uint16_t* bias, uint16_t* out, int64_t M, int32_t N,
                      int32_t K, int64_t ldo, int32_t act, void* stream) {
  clear_error();
  if (!a || !w || !bias || !out) return set_error(GDC_ERR_NULL_POINTER, "gdc_linear: null argument");
  int* err = nullptr;
  GDC_TRY(device_error_word(&err));
  return launch_linear(reinterpret_cast<const __half*>(a), K, reinterpret_cast<const __half*>(w),
                       reinterpret_cast<const __half*>(bias), reinterpret_cast<__half*>(out), ldo, M, N, K, act,
                       static_cast<cudaStream_t>(stream), err);
}

gdc_status gdc_selftest_wait_timeout(int32_t limit_us, void* stream) {
  clear_error();
  int* err = nullptr;
  GDC_TRY(device_error_word(&err));
  return launch_wait_timeout_probe(err, limit_us, static_cast<cudaStream_t>(stream));
}

gdc_status gdc_kernels_check_errors(void) {
  clear_error();
  int* err = nullptr;
  GDC_TRY(device_error_word(&err));
  GDC_CUDA_TRY(cudaDeviceSynchronize());
  int h = 0;
  GDC_CUDA_TRY(cudaMemcpy(&h, err, sizeof(int), cudaMemcpyDeviceToHost));
  if (h != 0) {
    GDC_CUDA_TRY(cudaMemset(err, 0, sizeof(int)));
    if (h & kErrTimeout) return set_error(GDC_ERR_TIMEOUT, "a device-side wait exceeded its time limit");
    return set_error(GDC_ERR_CUDA, "device error word 0x%x", h);
  }
  return GDC_OK;
}

}  // extern "C"
