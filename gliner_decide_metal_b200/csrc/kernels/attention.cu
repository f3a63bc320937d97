// Disentangled attention launchers (DeBERTa.swift:322-395).
//
// launch_attention runs the tcgen05 kernel (attention_tc.cuh). The scalar kernel
// (attention_simt.cuh) is kept as an on-device cross-check at sizes the CPU oracle
// cannot reach; the forward never calls it.
#include <cuda.h>

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

gdc_status launch_attention(const __half* qkv, const __half* pos_qk, const __half* key_mask,
                            const int32_t* rel_table, __half* ctx, int batch, int seq_len, int heads,
                            cudaStream_t stream, int* err) {
  if (batch <= 0 || seq_len <= 0) return GDC_OK;
  if (seq_len > 512) return set_error(GDC_ERR_UNSUPPORTED, "attention: seq_len %d > 512", seq_len);
  if (heads <= 0 || heads > 64) return set_error(GDC_ERR_UNSUPPORTED, "attention: heads %d", heads);
  if ((reinterpret_cast<uintptr_t>(qkv) & 15) || (reinterpret_cast<uintptr_t>(pos_qk) & 15) ||
      (reinterpret_cast<uintptr_t>(ctx) & 15))
    return set_error(GDC_ERR_INVALID_INPUT, "attention: buffers must be 16-byte aligned");
  const int E = heads * 64;
  CUtensorMap tm_qkv, tm_pos;
  GDC_TRY(make_tmap_2d(&tm_qkv, qkv, uint64_t(batch) * uint64_t(seq_len), uint64_t(3 * E), uint64_t(3 * E),
                       attn::kTile));
  GDC_TRY(make_tmap_2d(&tm_pos, pos_qk, 512, uint64_t(2 * E), uint64_t(2 * E), attn::kWin));
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(attn::attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         attn::kSmemBytes);
    if (e != cudaSuccess) return set_error(GDC_ERR_CUDA, "attention smem attribute: %s", cudaGetErrorString(e));
    configured[dev] = true;
  }
  const long long items = (long long)((seq_len + attn::kTile - 1) / attn::kTile) * heads * batch;
  if (items > (1ll << 30)) return set_error(GDC_ERR_UNSUPPORTED, "attention: too many work items");
  const int sms = device_sm_count(dev);
  const int grid = items < sms ? int(items) : sms;  // persistent: one CTA per SM
  attn::attention_tc_kernel<<<grid, attn::kThreads, attn::kSmemBytes, stream>>>(tm_qkv, tm_pos, key_mask, rel_table,
                                                                                ctx, batch, seq_len, heads, err);
  return check_launch("attention_tc_kernel");
}

}  // namespace gdc
