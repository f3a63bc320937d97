// Disentangled attention launchers (DeBERTa.swift:322-395).
//
// launch_attention runs the tcgen05 kernel (attention_tc.cuh). The scalar kernel
// (attention_simt.cuh) is kept as an on-device cross-check at sizes the CPU oracle
// cannot reach; the forward never calls it.
#include <cuda.h>

#include <mutex>

#include "../model.h"
#include "attention_simt.cuh"
#include "attention_tc.cuh"
#include "kernels.h"

namespace gdc {

gdc_status launch_attention_simt(const __half* qkv, const __half* pos_qk, const __half* key_mask,
                                 const int32_t* rel_table, __half* ctx, int batch, int seq_len, int heads,
                                 cudaStream_t stream) {
  if (batch <= 0 || seq_len <= 0) return GDC_OK;
  if (seq_len > 512) return set_error(GDC_ERR_UNSUPPORTED, "attention: seq_len %d > 512", seq_len);
  dim3 grid((seq_len + 7) / 8, heads, batch);
  attention_simt_kernel<<<grid, 256, 0, stream>>>(qkv, pos_qk, key_mask, rel_table, ctx, seq_len, heads);
  return check_launch("attention_simt_kernel");
}

gdc_status launch_expand_positions(const __half* pos_qk, const int32_t* rel_table, __half* pos_exp, int cols,
                                   cudaStream_t stream) {
  if (cols <= 0 || cols % 8 != 0) return set_error(GDC_ERR_UNSUPPORTED, "expand positions: %d columns", cols);
  if ((reinterpret_cast<uintptr_t>(pos_qk) & 15) || (reinterpret_cast<uintptr_t>(pos_exp) & 15))
    return set_error(GDC_ERR_INVALID_INPUT, "expand positions: buffers must be 16-byte aligned");
  attn::expand_positions_kernel<<<attn::kExpRows, 256, 0, stream>>>(pos_qk, rel_table, pos_exp, cols);
  return check_launch("expand_positions_kernel");
}

gdc_status launch_attention(const __half* qkv, const __half* pos_exp, const __half* key_mask, __half* ctx,
                            int batch, int seq_len, int heads, cudaStream_t stream, int* err,
                            const AttentionWork& work) {
  if (batch <= 0 || seq_len <= 0) return GDC_OK;
  if (seq_len > 512) return set_error(GDC_ERR_UNSUPPORTED, "attention: seq_len %d > 512", seq_len);
  if (heads <= 0 || heads > 64) return set_error(GDC_ERR_UNSUPPORTED, "attention: heads %d", heads);
  if (work.row_order != nullptr && (work.groups == nullptr || work.counter == nullptr || work.seq_off == nullptr))
    return set_error(GDC_ERR_INVALID_INPUT, "attention: a row order needs groups, packed rows and a counter");
  if ((reinterpret_cast<uintptr_t>(qkv) & 15) || (reinterpret_cast<uintptr_t>(pos_exp) & 15) ||
      (reinterpret_cast<uintptr_t>(ctx) & 15))
    return set_error(GDC_ERR_INVALID_INPUT, "attention: buffers must be 16-byte aligned");
  const int E = heads * 64;
  CUtensorMap tm_qkv, tm_pos;
  GDC_TRY(make_tmap_2d(&tm_qkv, qkv, uint64_t(batch) * uint64_t(seq_len), uint64_t(3 * E), uint64_t(3 * E),
                       attn::kTile));
  GDC_TRY(make_tmap_2d(&tm_pos, pos_exp, attn::kExpRows, uint64_t(2 * E), uint64_t(2 * E), attn::kWin));
  static PerDeviceOnce configured;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return set_error(GDC_ERR_CUDA, "device ordinal out of range");
  const cudaError_t ce = cudaError_t(per_device_once(configured, dev, [] {
    return cudaFuncSetAttribute(attn::attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                attn::kSmemBytes);
  }));
  if (ce != cudaSuccess) return set_error(GDC_ERR_CUDA, "attention smem attribute: %s", cudaGetErrorString(ce));
  const long long items = (long long)((seq_len + attn::kTile - 1) / attn::kTile) * heads * batch;
  if (items > (1ll << 30)) return set_error(GDC_ERR_UNSUPPORTED, "attention: too many work items");
  const int sms = device_sm_count(dev);
  const int grid = items < sms ? int(items) : sms;  // persistent: one CTA per SM
  AttentionWork w = work;
  if (items <= grid) {
    // one item per CTA at most: the static split is already balanced and needs no atomics
    w.counter = nullptr;
    w.row_order = nullptr;
    w.groups = nullptr;
  }
  attn::attention_tc_kernel<<<grid, attn::kThreads, attn::kSmemBytes, stream>>>(tm_qkv, tm_pos, key_mask, ctx, batch,
                                                                                seq_len, heads, err, w);
  return check_launch("attention_tc_kernel");
}

namespace {

// Allocation-free attention: the scratch that gdc_disentangled_attention takes from the
// stream-ordered allocator (the expanded position table) or keeps in cudaMalloc'd memory
// (the relative index table and the device-side status word) lives in this file-scope array
// instead. It is 4,194,560 bytes (heads = 16, seq_len <= 512) and every device that loads
// the library holds it until the process exits.
//   [0, 4190208)        expanded position table, 1023 rows x 2048 fp16 (rebuilt by every call)
//   [4190208, +4092)    relative index table i(r), index r + 511 (written once per device)
//   [4194304]           status word; bounded-wait timeouts set bits in it (cleared by every call)
constexpr int kStaticHeads = 16;
constexpr size_t kStaticExpBytes = size_t(1023) * 2 * kStaticHeads * 64 * 2;
constexpr size_t kStaticTableOffset = kStaticExpBytes;
constexpr int kStaticTableEntries = 1023;
constexpr size_t kStaticStatusOffset = kStaticTableOffset + 4096;
constexpr size_t kStaticBytes = kStaticStatusOffset + 256;
static __device__ __align__(256) uint8_t g_attention_scratch[kStaticBytes];

std::mutex g_static_mu;
uint8_t* g_static_scratch[64] = {};  // device address of g_attention_scratch, per device

// Once per device, with that device current: resolve the array's device address and write
// the relative index table into it (a synchronous copy from host memory).
gdc_status static_scratch(uint8_t** out) {
  int dev = 0;
  GDC_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return set_error(GDC_ERR_CUDA, "device ordinal out of range");
  std::lock_guard<std::mutex> lk(g_static_mu);
  if (!g_static_scratch[dev]) {
    uint8_t* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&ptr), g_attention_scratch);
    if (e != cudaSuccess)
      return set_error(GDC_ERR_CUDA, "cudaGetSymbolAddress(attention scratch): %s", cudaGetErrorString(e));
    int32_t table[kStaticTableEntries];
    build_relative_table(256, 512, table);
    GDC_CUDA_TRY(cudaMemcpy(ptr + kStaticTableOffset, table, sizeof(table), cudaMemcpyHostToDevice));
    GDC_CUDA_TRY(cudaMemset(ptr + kStaticStatusOffset, 0, sizeof(int32_t)));
    g_static_scratch[dev] = ptr;
  }
  *out = g_static_scratch[dev];
  return GDC_OK;
}

}  // namespace

}  // namespace gdc

extern "C" gdc_status gdc_disentangled_attention_noalloc(const uint16_t* qkv, const uint16_t* pos_qk,
                                                         const uint16_t* key_mask, uint16_t* ctx, int32_t batch,
                                                         int32_t seq_len, int32_t heads, void* stream) {
  using namespace gdc;
  clear_error();
  if (!qkv || !pos_qk || !key_mask || !ctx)
    return set_error(GDC_ERR_NULL_POINTER, "gdc_disentangled_attention_noalloc: null argument");
  if (heads != 16) return set_error(GDC_ERR_UNSUPPORTED, "gdc_disentangled_attention_noalloc: heads must be 16");
  if (batch <= 0 || seq_len <= 0)
    return set_error(GDC_ERR_INVALID_INPUT, "gdc_disentangled_attention_noalloc: batch and seq_len must be > 0");
  if (seq_len > 512)
    return set_error(GDC_ERR_UNSUPPORTED,
                     "gdc_disentangled_attention_noalloc: seq_len %d exceeds the static scratch limit of 512 "
                     "(its expanded position table covers distances up to %d)",
                     seq_len, kStaticTableEntries / 2);
  uint8_t* scratch = nullptr;
  GDC_TRY(static_scratch(&scratch));
  __half* pos_exp = reinterpret_cast<__half*>(scratch);
  const int32_t* table = reinterpret_cast<const int32_t*>(scratch + kStaticTableOffset);
  int32_t* status = reinterpret_cast<int32_t*>(scratch + kStaticStatusOffset);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  GDC_CUDA_TRY(cudaMemsetAsync(status, 0, sizeof(int32_t), s));
  GDC_TRY(launch_expand_positions(reinterpret_cast<const __half*>(pos_qk), table, pos_exp, 2 * kStaticHeads * 64, s));
  GDC_TRY(launch_attention(reinterpret_cast<const __half*>(qkv), pos_exp, reinterpret_cast<const __half*>(key_mask),
                           reinterpret_cast<__half*>(ctx), batch, seq_len, heads, s, status));
  int32_t h = 0;
  GDC_CUDA_TRY(cudaMemcpyAsync(&h, status, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
  GDC_CUDA_TRY(cudaStreamSynchronize(s));
  if (h != 0) {
    if (h & kErrTimeout)
      return set_error(GDC_ERR_TIMEOUT, "gdc_disentangled_attention_noalloc: a device-side wait exceeded its limit");
    return set_error(GDC_ERR_CUDA, "gdc_disentangled_attention_noalloc: device status word 0x%x", h);
  }
  return GDC_OK;
}
