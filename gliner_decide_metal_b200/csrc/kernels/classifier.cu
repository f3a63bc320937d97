// Classifier head kernels (DeBERTa.swift:430-444) and the per-task decode
// (RawCLI.swift:182-223).
//
//   marker_gather    rows[r] = hidden[markerIdx[r] + b * L]  (b = r / (Hm * O))
//   (tcgen05 GEMM)   h = relu(rows . W0^T + b0)               (classifier.0 + ReLU)
//   classifier_out   logit[r] = fp16(h[r] . w2 + b2), -10000 where markerMask <= 0
//   decode           per (row, task): sigmoid / threshold 0.5 / argmax fallback, or
//                    max-subtracted softmax / argmax over the task's labels.
#include "kernels.h"
#include "ptx.cuh"

namespace gdc {
namespace {

__global__ void marker_gather_kernel(const __half* __restrict__ hidden, const int32_t* __restrict__ markers,
                                     __half* __restrict__ rows, int n_rows, int per_batch, int seq_len, int cols,
                                     int* err, const int32_t* __restrict__ seq_off) {
  const int r = blockIdx.x;
  if (r >= n_rows) return;
  const int b = r / per_batch;
  int idx = markers[r];
  if (idx < 0 || idx >= seq_len) {
    if (threadIdx.x == 0) atomicOr(err, kErrBadMarkerIndex);
    idx = 0;
  }
  long long row = (long long)b * seq_len + idx;
  if (seq_off != nullptr) {
    const int off = seq_off[b];
    row = off + (idx < seq_off[b + 1] - off ? idx : 0);  // an inactive marker past the extent
  }
  const uint4* src = reinterpret_cast<const uint4*>(hidden + row * cols);
  uint4* dst = reinterpret_cast<uint4*>(rows + (long long)r * cols);
  for (int i = threadIdx.x; i < cols / 8; i += blockDim.x) dst[i] = src[i];
}

// One warp per marker row.
__global__ void classifier_out_kernel(const __half* __restrict__ h, const __half* __restrict__ w2,
                                      const __half* __restrict__ b2, const float* __restrict__ marker_mask,
                                      float* __restrict__ logits, __half* __restrict__ logits16, int n_rows, int dc) {
  const int lane = threadIdx.x & 31;
  const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= n_rows) return;
  const __half* hr = h + (long long)r * dc;
  float acc = 0.f;
  for (int i = lane * 8; i < dc; i += 256) {
    const uint4 hv = *reinterpret_cast<const uint4*>(hr + i);
    const uint4 wv = __ldg(reinterpret_cast<const uint4*>(w2 + i));
    const __half2* hh = reinterpret_cast<const __half2*>(&hv);
    const __half2* wh = reinterpret_cast<const __half2*>(&wv);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 a = __half22float2(hh[j]);
      const float2 w = __half22float2(wh[j]);
      acc = fmaf(a.x, w.x, acc);
      acc = fmaf(a.y, w.y, acc);
    }
  }
  acc = ptx::warp_sum(acc);
  if (lane == 0) {
    // classifier.2 output is an fp16 array in the reference; the -10000 fill is fp16 too.
    const __half v = __float2half_rn(acc + __half2float(b2[0]));
    const __half out = marker_mask[r] > 0.f ? v : __float2half_rn(-10000.0f);
    logits[r] = __half2float(out);
    if (logits16) logits16[r] = out;
  }
}

// One thread per (row, task). RawCLI.swift:182-223 decodes in Swift Double, so the
// arithmetic here is float64 as well (probabilities are stored as float32): the
// selections then equal the host decode's, including first-argmax ties and logits whose
// sigmoid or shifted exponential underflows to 0.
__global__ void decode_kernel(const float* __restrict__ logits, int batch, int max_heads, int max_options,
                              const int32_t* __restrict__ n_labels, const uint8_t* __restrict__ multi_label,
                              float* __restrict__ probs, uint8_t* __restrict__ selected) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= batch * max_heads) return;
  const float* x = logits + (long long)t * max_options;
  float* p = probs + (long long)t * max_options;
  uint8_t* s = selected + (long long)t * max_options;
  int n = n_labels[t];
  if (n > max_options) n = max_options;
  for (int o = 0; o < max_options; ++o) {
    p[o] = 0.f;
    s[o] = 0;
  }
  if (n <= 0) return;
  if (multi_label[t]) {
    // unshifted sigmoid; select p >= 0.5, else the first argmax
    int best = 0;
    double best_p = -1.0;
    bool any = false;
    for (int o = 0; o < n; ++o) {
      const double q = 1.0 / (1.0 + exp(-double(x[o])));
      p[o] = float(q);
      if (q >= 0.5) {
        s[o] = 1;
        any = true;
      }
      if (q > best_p) {
        best_p = q;
        best = o;
      }
    }
    if (!any) s[best] = 1;
  } else {
    // max-subtracted softmax, first argmax
    double m = double(x[0]);
    for (int o = 1; o < n; ++o) m = fmax(m, double(x[o]));
    double sum = 0.0;
    for (int o = 0; o < n; ++o) sum += exp(double(x[o]) - m);
    int best = 0;
    double best_p = -1.0;
    for (int o = 0; o < n; ++o) {
      const double q = exp(double(x[o]) - m) / sum;
      p[o] = float(q);
      if (q > best_p) {
        best_p = q;
        best = o;
      }
    }
    s[best] = 1;
  }
}

}  // namespace

gdc_status launch_marker_gather(const __half* hidden, const int32_t* markers, __half* rows, int n_rows, int per_batch,
                                int seq_len, int cols, cudaStream_t stream, int* err, const int32_t* seq_off) {
  if (n_rows <= 0) return GDC_OK;
  if (cols % 8 != 0 || per_batch <= 0) return set_error(GDC_ERR_UNSUPPORTED, "marker gather: bad shape");
  marker_gather_kernel<<<n_rows, 128, 0, stream>>>(hidden, markers, rows, n_rows, per_batch, seq_len, cols, err,
                                                   seq_off);
  return check_launch("marker_gather_kernel");
}

gdc_status launch_classifier_out(const __half* h, const __half* w2, const __half* b2, const float* marker_mask,
                                 float* logits, __half* logits_f16, int n_rows, int dc, cudaStream_t stream) {
  if (n_rows <= 0) return GDC_OK;
  if (dc % 256 != 0) return set_error(GDC_ERR_UNSUPPORTED, "classifier: hidden width %d not a multiple of 256", dc);
  const int per_block = 8;
  classifier_out_kernel<<<(n_rows + per_block - 1) / per_block, per_block * 32, 0, stream>>>(
      h, w2, b2, marker_mask, logits, logits_f16, n_rows, dc);
  return check_launch("classifier_out_kernel");
}

gdc_status launch_decode(const float* logits, int batch, int max_heads, int max_options, const int32_t* n_labels,
                         const uint8_t* multi_label, float* probs, uint8_t* selected, cudaStream_t stream) {
  const int n = batch * max_heads;
  if (n <= 0) return GDC_OK;
  decode_kernel<<<(n + 127) / 128, 128, 0, stream>>>(logits, batch, max_heads, max_options, n_labels, multi_label,
                                                     probs, selected);
  return check_launch("decode_kernel");
}

}  // namespace gdc
