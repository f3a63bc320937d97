// Row LayerNorm kernels: residual-add LayerNorm and the fused embedding stage.
//
// residual LN replaces `norm(x + residual)` (DeBERTa.swift:449-464, MLXFast.layerNorm)
// and FusedKernels.residualLayerNorm (FusedKernels.swift:125-155): one warp per row,
// 16-byte loads (8 fp16 per lane per chunk), the row held in registers, two-pass
// mean / biased variance in fp32, rsqrt(var + eps), affine, fp16 store.
//
// The embedding kernel replaces DeBERTa.swift:285-292: gather the word-embedding row of
// each token id, LayerNorm it, multiply by the attention-mask value.
//
// Both are HBM-bound: per row they move cols * 2 bytes per input and output once.
#include "kernels.h"
#include "ptx.cuh"

namespace gdc {
namespace {

constexpr int kRowsPerBlock = 8;  // 8 warps, one row each
constexpr int kPackedTailRows = 256;  // a GEMM tile (256 rows) covers every row a key tile reaches

// gamma / beta of this lane's columns. Rows of up to 1024 columns load them before the row,
// so their round trip overlaps the row's instead of following the statistics; wider rows
// (more registers per lane) load them where they are used.
template <int CH>
struct AffineRegs {
  static constexpr bool kEarly = CH <= 4;
  static constexpr int kN = kEarly ? CH : 1;
  uint4 g[kN], b[kN];
  const __half* gamma;
  const __half* beta;
  __device__ __forceinline__ void load(const __half* __restrict__ gm, const __half* __restrict__ bt, int lane) {
    gamma = gm;
    beta = bt;
    if (kEarly) {
#pragma unroll
      for (int c = 0; c < kN; ++c) {
        const int col = (c * 32 + lane) * 8;
        g[c] = __ldg(reinterpret_cast<const uint4*>(gamma + col));
        b[c] = __ldg(reinterpret_cast<const uint4*>(beta + col));
      }
    }
  }
  __device__ __forceinline__ uint4 gv(int c, int col) const {
    return kEarly ? g[c < kN ? c : 0] : __ldg(reinterpret_cast<const uint4*>(gamma + col));
  }
  __device__ __forceinline__ uint4 bv(int c, int col) const {
    return kEarly ? b[c < kN ? c : 0] : __ldg(reinterpret_cast<const uint4*>(beta + col));
  }
};

template <int CH>
__device__ __forceinline__ void ln_row_store(float (&v)[CH * 8], const AffineRegs<CH>& aff, __half* __restrict__ dst,
                                             int lane, float eps, float scale_after) {
  constexpr int cols = CH * 256;
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < CH * 8; ++i) s += v[i];
  const float mean = ptx::warp_sum(s) * (1.0f / cols);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < CH * 8; ++i) {
    const float d = v[i] - mean;
    q += d * d;
  }
  const float var = ptx::warp_sum(q) * (1.0f / cols);
  const float inv = rsqrtf(var + eps);
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int col = (c * 32 + lane) * 8;
    const uint4 gw = aff.gv(c, col);
    const uint4 bw = aff.bv(c, col);
    const __half2* gh = reinterpret_cast<const __half2*>(&gw);
    const __half2* bh = reinterpret_cast<const __half2*>(&bw);
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 g = __half22float2(gh[j]);
      const float2 b = __half22float2(bh[j]);
      float y0 = (v[c * 8 + 2 * j] - mean) * inv * g.x + b.x;
      float y1 = (v[c * 8 + 2 * j + 1] - mean) * inv * g.y + b.y;
      if (scale_after != 1.0f) {
        // LN output is rounded to fp16 before the mask multiply (two fp16 ops).
        y0 = __half2float(__float2half_rn(y0)) * scale_after;
        y1 = __half2float(__float2half_rn(y1)) * scale_after;
      }
      o[j] = ptx::pack_half2(y0, y1);
    }
    *reinterpret_cast<uint4*>(dst + col) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

template <int CH>
__global__ void __launch_bounds__(kRowsPerBlock * 32)
    residual_ln_kernel(const __half* __restrict__ x, const __half* __restrict__ res, const __half* __restrict__ gamma,
                       const __half* __restrict__ beta, __half* __restrict__ out, long long rows, float eps,
                       const int32_t* __restrict__ m_dev) {
  constexpr int cols = CH * 256;
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * kRowsPerBlock + (threadIdx.x >> 5);
  if (row >= rows || (m_dev != nullptr && row >= *m_dev)) return;
  AffineRegs<CH> aff;
  aff.load(gamma, beta, lane);
  const __half* xr = x + row * cols;
  float v[CH * 8];
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int col = (c * 32 + lane) * 8;
    const uint4 xv = *reinterpret_cast<const uint4*>(xr + col);
    const __half2* xh = reinterpret_cast<const __half2*>(&xv);
    if (res != nullptr) {
      const uint4 rv = *reinterpret_cast<const uint4*>(res + row * cols + col);
      const __half2* rh = reinterpret_cast<const __half2*>(&rv);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 s = __half22float2(__hadd2(xh[j], rh[j]));  // fp16 add, as the reference
        v[c * 8 + 2 * j] = s.x;
        v[c * 8 + 2 * j + 1] = s.y;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 s = __half22float2(xh[j]);
        v[c * 8 + 2 * j] = s.x;
        v[c * 8 + 2 * j + 1] = s.y;
      }
    }
  }
  ln_row_store<CH>(v, aff, out + row * cols, lane, eps, 1.0f);
}

template <int CH>
__global__ void __launch_bounds__(kRowsPerBlock * 32)
    embedding_kernel(const int32_t* __restrict__ ids, const __half* __restrict__ mask, const __half* __restrict__ table,
                     long long vocab, const __half* __restrict__ gamma, const __half* __restrict__ beta,
                     __half* __restrict__ out, long long rows, float eps, int* err,
                     const int32_t* __restrict__ rowmap, const int32_t* __restrict__ m_dev,
                     __half* __restrict__ tail_buf, int tail_cols) {
  constexpr int cols = CH * 256;
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * kRowsPerBlock + (threadIdx.x >> 5);
  if (row >= rows) return;
  if (m_dev != nullptr && row >= *m_dev) {
    // Rows just past the packed count: GEMM tiles and attention key tiles read them. Zero
    // hidden rows make every layer's QKV rows there its bias, and zero QKV rows beyond the
    // last GEMM tile stay zero, so nothing left by an earlier call can reach this one.
    if (row < (long long)*m_dev + kPackedTailRows) {
      const uint4 z = make_uint4(0u, 0u, 0u, 0u);
      for (int c = lane; c < cols / 8; c += 32) reinterpret_cast<uint4*>(out + row * cols)[c] = z;
      if (tail_buf != nullptr)
        for (int c = lane; c < tail_cols / 8; c += 32)
          reinterpret_cast<uint4*>(tail_buf + row * (long long)tail_cols)[c] = z;
    }
    return;
  }
  AffineRegs<CH> aff;
  aff.load(gamma, beta, lane);
  const long long src = rowmap != nullptr ? (long long)rowmap[row] : row;  // dense position of the row
  long long id = ids[src];
  if (id < 0 || id >= vocab) {
    if (lane == 0) atomicOr(err, kErrBadTokenId);
    id = 0;
  }
  const __half* er = table + id * cols;
  float v[CH * 8];
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    const int col = (c * 32 + lane) * 8;
    const uint4 ev = __ldg(reinterpret_cast<const uint4*>(er + col));
    const __half2* eh = reinterpret_cast<const __half2*>(&ev);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 s = __half22float2(eh[j]);
      v[c * 8 + 2 * j] = s.x;
      v[c * 8 + 2 * j + 1] = s.y;
    }
  }
  const float m = __half2float(mask[src]);
  // scale_after == 1 would skip the rounding; a mask of exactly 1 changes nothing anyway.
  ln_row_store<CH>(v, aff, out + row * cols, lane, eps, m);
}

}  // namespace

#define GDC_LN_DISPATCH(CH_EXPR, KERNEL, ...)                                                 \
  switch (CH_EXPR) {                                                                          \
    case 1: KERNEL<1><<<grid, kRowsPerBlock * 32, 0, stream>>>(__VA_ARGS__); break;          \
    case 2: KERNEL<2><<<grid, kRowsPerBlock * 32, 0, stream>>>(__VA_ARGS__); break;          \
    case 3: KERNEL<3><<<grid, kRowsPerBlock * 32, 0, stream>>>(__VA_ARGS__); break;          \
    case 4: KERNEL<4><<<grid, kRowsPerBlock * 32, 0, stream>>>(__VA_ARGS__); break;          \
    case 8: KERNEL<8><<<grid, kRowsPerBlock * 32, 0, stream>>>(__VA_ARGS__); break;          \
    case 16: KERNEL<16><<<grid, kRowsPerBlock * 32, 0, stream>>>(__VA_ARGS__); break;        \
    default: return set_error(GDC_ERR_UNSUPPORTED, "layer norm: cols=%d unsupported", cols); \
  }

gdc_status launch_residual_layer_norm(const __half* x, const __half* residual, const __half* gamma,
                                      const __half* beta, __half* out, int64_t rows, int cols, float eps,
                                      cudaStream_t stream, const int32_t* m_dev) {
  if (rows <= 0) return GDC_OK;
  if (cols <= 0 || cols % 256 != 0 || cols > 4096)
    return set_error(GDC_ERR_UNSUPPORTED, "layer norm: cols=%d must be a multiple of 256 and <= 4096", cols);
  const unsigned grid = unsigned((rows + kRowsPerBlock - 1) / kRowsPerBlock);
  GDC_LN_DISPATCH(cols / 256, residual_ln_kernel, x, residual, gamma, beta, out, (long long)rows, eps, m_dev);
  return check_launch("residual_ln_kernel");
}

gdc_status launch_embedding(const int32_t* ids, const __half* mask, const __half* table, int64_t vocab,
                            const __half* gamma, const __half* beta, __half* out, int64_t rows, int cols,
                            float eps, cudaStream_t stream, int* err, const int32_t* rowmap,
                            const int32_t* m_dev, __half* tail_buf, int tail_cols) {
  if (rows <= 0) return GDC_OK;
  if (cols <= 0 || cols % 256 != 0 || cols > 4096)
    return set_error(GDC_ERR_UNSUPPORTED, "embedding: cols=%d unsupported", cols);
  if ((rowmap == nullptr) != (m_dev == nullptr))
    return set_error(GDC_ERR_INVALID_INPUT, "embedding: rowmap and row count go together");
  if (tail_buf != nullptr && (tail_cols <= 0 || tail_cols % 8 != 0 || (reinterpret_cast<uintptr_t>(tail_buf) & 15)))
    return set_error(GDC_ERR_INVALID_INPUT, "embedding: tail buffer must be 16-byte aligned rows of 8k columns");
  const unsigned grid = unsigned((rows + kRowsPerBlock - 1) / kRowsPerBlock);
  GDC_LN_DISPATCH(cols / 256, embedding_kernel, ids, mask, table, (long long)vocab, gamma, beta, out,
                  (long long)rows, eps, err, rowmap, m_dev, tail_buf, tail_cols);
  return check_launch("embedding_kernel");
}

}  // namespace gdc
