// Disentangled attention launchers (DeBERTa.swift:322-395).
#include "attention_simt.cuh"
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
  (void)err;
  return launch_attention_simt(qkv, pos_qk, key_mask, rel_table, ctx, batch, seq_len, heads, stream);
}

}  // namespace gdc
