// Row packing (padding removal) for the encoder.
//
// The reference runs every layer on the dense [B, L] grid (DeBERTa.swift:274-447), padding
// positions included. The logits depend only on the rows the classifier gathers
// (DeBERTa.swift:430-436) and on the keys the attention mask admits: a position p of batch
// row b influences another position only as a key, and keys with mask 0 get weight exactly
// zero whenever the row has one valid key. So the encoder may compute, per batch row, only
// the positions [0, ext_b), where
//   ext_b = max(last position with mask > 0, last active marker index) + 1,
//   ext_b = L when the row has no position with mask > 0 (the softmax then spreads over
//           all L masked keys, as in the dense grid).
// Rows of a batch are stored back to back ("packed"): packed row seq_off[b] + t holds
// position t of batch row b, seq_off is the exclusive prefix sum of the extents and
// seq_off[B] is the packed row count. Every kernel computes each packed row exactly as the
// dense grid computes that position (same tiles along K, same key tiles), so the logits are
// bit-identical to the dense forward.
//
// The same pass orders the attention work: a row whose extent spans c 128-position tiles
// has c live query tiles per head, each costing up to c (query tile, key tile) pairs.
// groups[c] counts those rows and row_order lists the rows by descending c (order inside
// a group is arbitrary), so attention CTAs that take items from a shared counter take the
// expensive ones first.
#include "kernels.h"
#include "ptx.cuh"

namespace gdc {
namespace {

constexpr int kPackThreads = 1024;
constexpr int kMaxTiles = 4;  // 128-position tiles of seq_len <= 512

__device__ __forceinline__ int warp_max_i(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// One CTA: extents (warp per batch row), work groups, block-wide exclusive scan, row map.
__global__ void __launch_bounds__(kPackThreads)
    row_pack_kernel(const __half* __restrict__ mask, const int32_t* __restrict__ markers,
                    const float* __restrict__ marker_mask, int B, int L, int per_batch, int32_t* __restrict__ seq_off,
                    int32_t* __restrict__ rowmap, int32_t* __restrict__ row_order, int32_t* __restrict__ groups) {
  __shared__ int32_t s_warp[32];
  __shared__ int32_t s_count[kMaxTiles + 1];
  __shared__ int32_t s_cursor[kMaxTiles + 1];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  constexpr int kWarps = kPackThreads / 32;

  for (int b = warp; b < B; b += kWarps) {
    const __half* mr = mask + (long long)b * L;
    int last = -1;
    for (int t = lane; t < L; t += 32)
      if (__half2float(mr[t]) > 0.f) last = t;
    last = warp_max_i(last);
    int mk = 0;
    const long long m0 = (long long)b * per_batch;
    for (int j = lane; j < per_batch; j += 32) {
      const int idx = markers[m0 + j];
      if (marker_mask[m0 + j] > 0.f && idx >= 0 && idx < L) mk = max(mk, idx + 1);
    }
    mk = warp_max_i(mk);
    if (lane == 0) seq_off[b + 1] = last < 0 ? L : max(last + 1, mk);
  }
  if (threadIdx.x <= kMaxTiles) s_count[threadIdx.x] = 0;
  __syncthreads();

  // work groups: rows by number of 128-position tiles c, groups and row order by descending c
  for (int b = int(threadIdx.x); b < B; b += kPackThreads) atomicAdd(&s_count[(seq_off[b + 1] + 127) >> 7], 1);
  __syncthreads();
  if (threadIdx.x == 0) {
    int start = 0;
    for (int c = kMaxTiles; c >= 0; --c) {
      s_cursor[c] = start;
      start += s_count[c];
      groups[c] = s_count[c];
    }
    seq_off[0] = 0;
  }
  __syncthreads();
  for (int b = int(threadIdx.x); b < B; b += kPackThreads)
    row_order[atomicAdd(&s_cursor[(seq_off[b + 1] + 127) >> 7], 1)] = b;
  __syncthreads();

  int carry = 0;
  for (int base = 0; base < B; base += kPackThreads) {
    const int b = base + int(threadIdx.x);
    const int v = b < B ? seq_off[b + 1] : 0;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) s_warp[warp] = x;
    __syncthreads();
    if (warp == 0) {
      int w = s_warp[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      s_warp[lane] = w;
    }
    __syncthreads();
    const int incl = x + (warp > 0 ? s_warp[warp - 1] : 0) + carry;
    carry += s_warp[kWarps - 1];
    if (b < B) seq_off[b + 1] = incl;
    __syncthreads();  // s_warp is rewritten by the next chunk
  }

  for (int b = warp; b < B; b += kWarps) {
    const int off = seq_off[b];
    const int ext = seq_off[b + 1] - off;
    for (int t = lane; t < ext; t += 32) rowmap[off + t] = b * L + t;
  }
}

}  // namespace

gdc_status launch_row_pack(const __half* mask, const int32_t* markers, const float* marker_mask, int batch,
                           int seq_len, int per_batch, int32_t* seq_off, int32_t* rowmap, int32_t* row_order,
                           int32_t* groups, cudaStream_t stream) {
  if (batch <= 0 || seq_len <= 0) return GDC_OK;
  if (seq_len > kMaxTiles * 128) return set_error(GDC_ERR_UNSUPPORTED, "row packing: seq_len %d > 512", seq_len);
  if (int64_t(batch) * seq_len > (int64_t(1) << 30))
    return set_error(GDC_ERR_UNSUPPORTED, "row packing: batch * seq_len too large");
  row_pack_kernel<<<1, kPackThreads, 0, stream>>>(mask, markers, marker_mask, batch, seq_len, per_batch, seq_off,
                                                  rowmap, row_order, groups);
  return check_launch("row_pack_kernel");
}

}  // namespace gdc
