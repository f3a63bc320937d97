// Host-side launchers for the sm_100a kernels of the forward.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "../common.h"

namespace gdc {

// Activation fused into the GEMM epilogue.
enum Act : int { kActNone = 0, kActGelu = 1, kActRelu = 2 };

// out[M, N] = act(a[M, K] . w[N, K]^T + bias[N]), fp16 in/out, fp32 accumulate, on
// tcgen05 tensor cores (persistent warp-specialised kernel, TMA-fed).
// Requirements: N % 128 == 0, K % 64 == 0, lda/ldo multiples of 8 elements,
// 16-byte aligned pointers. err: device error word (timeouts). m_dev (nullable): a device
// int read at kernel start; when given, only rows [0, min(M, *m_dev)) are computed (M is
// then the buffers' row capacity and fixes the launch shape).
gdc_status launch_linear(const __half* a, int64_t lda, const __half* w, const __half* bias, __half* out,
                         int64_t ldo, int64_t M, int N, int K, int act, cudaStream_t stream, int* err,
                         const int32_t* m_dev = nullptr);

// Same contract on CTA pairs (cta_group::2, 256-row tiles); launch_linear dispatches here
// for M > 128.
gdc_status launch_linear_pair(const __half* a, int64_t lda, const __half* w, const __half* bias, __half* out,
                              int64_t ldo, int64_t M, int N, int K, int act, cudaStream_t stream, int* err,
                              const int32_t* m_dev = nullptr);

// out = LN(x + residual) * gamma + beta (rows x cols, fp16; fp32 statistics). The
// sum x + residual is rounded to fp16 first, as the reference's fp16 add does.
// residual may be null. cols % 256 == 0, cols <= 4096. m_dev (nullable): device row count
// limiting the rows normalised, as for launch_linear.
gdc_status launch_residual_layer_norm(const __half* x, const __half* residual, const __half* gamma,
                                      const __half* beta, __half* out, int64_t rows, int cols, float eps,
                                      cudaStream_t stream, const int32_t* m_dev = nullptr);

// hidden[t] = LN(E[ids[t]]) * mask[t] for t < rows (DeBERTa.swift:285-292). Ids outside
// [0, vocab) set kErrBadTokenId and read row 0. Packed rows (rowmap and m_dev non-null):
// hidden[r] = LN(E[ids[rowmap[r]]]) * mask[rowmap[r]] for r < *m_dev, and the 256 rows after
// *m_dev (below `rows`) of hidden and of tail_buf (rows of tail_cols columns, nullable) are
// zeroed.
gdc_status launch_embedding(const int32_t* ids, const __half* mask, const __half* table, int64_t vocab,
                            const __half* gamma, const __half* beta, __half* out, int64_t rows, int cols,
                            float eps, cudaStream_t stream, int* err, const int32_t* rowmap = nullptr,
                            const int32_t* m_dev = nullptr, __half* tail_buf = nullptr, int tail_cols = 0);

// Packed-row layout of a batch (pack.cu): seq_off[0..B] (exclusive prefix sum of the
// per-row extents; seq_off[B] = packed row count), rowmap[r] = b * L + t for packed row
// r = seq_off[b] + t, and the attention work order: groups[c] = rows whose extent spans c
// 128-position tiles (c = 1..4, groups[0] = 0), row_order = the batch rows by descending c.
// One CTA; mask [B, L], markers / marker_mask [B, per_batch]; seq_len <= 512.
gdc_status launch_row_pack(const __half* mask, const int32_t* markers, const float* marker_mask, int batch,
                           int seq_len, int per_batch, int32_t* seq_off, int32_t* rowmap, int32_t* row_order,
                           int32_t* groups, cudaStream_t stream);

// Row layout and work distribution of one attention launch (all fields nullable).
//   seq_off    packed rows: position t of batch row b at qkv / ctx row seq_off[b] + t for
//              t < seq_off[b+1] - seq_off[b] (the key mask stays [batch, seq_len])
//   row_order  [batch] batch rows by descending key-tile count, groups[c] (c = 1..4) rows
//              with c key tiles (both from launch_row_pack; need seq_off and counter)
//   counter    2 device ints, zero before the launch and left zero after it: CTAs take
//              items from it one at a time (heaviest first with row_order); null: every
//              CTA takes every gridDim-th item. One launch at a time per counter.
struct AttentionWork {
  const int32_t* seq_off = nullptr;
  const int32_t* row_order = nullptr;
  const int32_t* groups = nullptr;
  int* counter = nullptr;
};

// Disentangled attention over the fused QKV projection output (see gdc.h). pos_exp: the
// expanded position table of launch_expand_positions ([1023, 2 * heads * 64] fp16, device).
gdc_status launch_attention(const __half* qkv, const __half* pos_exp, const __half* key_mask, __half* ctx,
                            int batch, int seq_len, int heads, cudaStream_t stream, int* err,
                            const AttentionWork& work = AttentionWork{});

// Expanded position table: pos_exp[x] = pos_qk[rel_table[x]] for x in [0, 1023), rows of
// `cols` fp16 (cols = 2 * heads * 64: PQ | PK). rel_table: the 1023 gather indices i(r),
// index r + 511 (device). Row x holds the relative projections of distance r = x - 511.
gdc_status launch_expand_positions(const __half* pos_qk, const int32_t* rel_table, __half* pos_exp, int cols,
                                   cudaStream_t stream);

// Bytes of an expanded position table for `heads` heads.
inline size_t expanded_position_bytes(int heads) { return size_t(1023) * size_t(2 * heads * 64) * 2; }

// rows[r] = hidden[marker[r] + (r / per_batch) * seq_len] (DeBERTa.swift:430-436).
// Marker indices outside [0, seq_len) set kErrBadMarkerIndex and read row 0 of the batch.
// Packed rows (seq_off non-null): hidden row seq_off[b] + marker; a marker at or beyond the
// row's extent (only inactive ones can be) reads row 0 of the batch row.
gdc_status launch_marker_gather(const __half* hidden, const int32_t* markers, __half* rows, int n_rows,
                                int per_batch, int seq_len, int cols, cudaStream_t stream, int* err,
                                const int32_t* seq_off = nullptr);

// logits[r] = where(marker_mask[r] > 0, fp16(h[r] . w2 + b2), -10000) (DeBERTa.swift:437-443).
gdc_status launch_classifier_out(const __half* h, const __half* w2, const __half* b2, const float* marker_mask,
                                 float* logits, __half* logits_f16, int n_rows, int dc, cudaStream_t stream);

// Per-task softmax / sigmoid decode in fp32 (RawCLI.swift:182-223).
gdc_status launch_decode(const float* logits, int batch, int max_heads, int max_options, const int32_t* n_labels,
                         const uint8_t* multi_label, float* probs, uint8_t* selected, cudaStream_t stream);

int device_sm_count(int device);

// Failure-detection self-test: a kernel whose bounded wait on an mbarrier that never
// completes runs out after limit_us microseconds and sets kErrTimeout in *err.
gdc_status launch_wait_timeout_probe(int* err, int limit_us, cudaStream_t stream);

// 2-D fp16 TMA descriptor: `rows` x `cols` (cols contiguous), row pitch `ld` elements,
// box = box_rows x 64 columns, 128-byte swizzle, out-of-bounds rows read as zero.
// (CUtensorMap is passed as void* to keep <cuda.h> out of this header.)
gdc_status make_tmap_2d(void* map, const __half* base, uint64_t rows, uint64_t cols, uint64_t ld,
                        uint32_t box_rows);

// K-atom fp16 TMA descriptor of a row-major `rows` x `cols` matrix (cols a multiple of 64,
// row pitch `ld` elements): dimensions {64 columns, rows, cols / 64 atoms} with strides
// {ld, 64 columns}, box {64, box_rows, atoms}, 128-byte swizzle. One load at {0, row, a}
// writes `atoms` swizzle atoms of box_rows x 64 columns each back to back in shared
// memory ([atom][row][64], atoms box_rows * 128 bytes apart): the K-major layout the MMA
// reads, in one box instead of one per atom. Out-of-range rows and atoms read as zero.
gdc_status make_tmap_katoms(void* map, const __half* base, uint64_t rows, uint64_t cols, uint64_t ld,
                            uint32_t box_rows, uint32_t atoms);

// 2-D fp16 TMA descriptor for 32 x 32 output boxes (64-byte rows, 64-byte swizzle), used by
// the GEMM epilogue's tensor stores; rows / columns beyond the extent are not written.
gdc_status make_tmap_2d_out32(void* map, const __half* base, uint64_t rows, uint64_t cols, uint64_t ld);

}  // namespace gdc
