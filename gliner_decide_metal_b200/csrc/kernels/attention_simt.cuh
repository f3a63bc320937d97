// Scalar (CUDA-core) disentangled attention: one warp per query row.
//
// Follows the reference's fused Metal kernel structure (FusedKernels.swift:13-81): each
// lane scores keys k = lane, lane + 32, ...: content q.k, c2p q.PK[idx(q-k)] and p2c
// k.PQ[idx(q-k)], with the default path's fp16 rounding of the relative bias
// (DeBERTa.swift:374-379), additive -65504 key mask, fp32 softmax, then P.V with lanes
// over head dimensions. It is the correctness baseline that the tensor-core kernel is
// tested against at sizes the CPU oracle cannot reach; the forward does not use it.
#pragma once

#include <cuda_fp16.h>

#include "ptx.cuh"

namespace gdc {

constexpr float kInvSqrt192 = 0.07216878364870322f;  // 1 / sqrt(3 * 64), fp32
constexpr float kScale16 = 13.859375f;               // fp16(sqrt(192))

// fp16 relative bias of the reference: fp16(fp16(fp16(c2p) + fp16(p2c)) / fp16(sqrt(192)))
__device__ __forceinline__ float rel_bias_f16(float c2p, float p2c) {
  const __half c = __float2half_rn(c2p);
  const __half p = __float2half_rn(p2c);
  const float sum = __half2float(__hadd(c, p));
  return __half2float(__float2half_rn(sum / kScale16));
}

__device__ __forceinline__ void load_row64(const __half* src, float (&dst)[64]) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(src) + i);
    const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __half22float2(h[j]);
      dst[i * 8 + 2 * j] = f.x;
      dst[i * 8 + 2 * j + 1] = f.y;
    }
  }
}

__device__ __forceinline__ float dot_row64(const float (&a)[64], const __half* b) {
  float acc = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(b) + i);
    const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __half22float2(h[j]);
      acc = fmaf(a[i * 8 + 2 * j], f.x, acc);
      acc = fmaf(a[i * 8 + 2 * j + 1], f.y, acc);
    }
  }
  return acc;
}

// grid (ceil(L/8), heads, batch), 256 threads. qkv [B*L, 3*E], pos_qk [512, 2*E] (PQ|PK),
// ctx [B*L, E] with E = heads * 64.
__global__ void __launch_bounds__(256) attention_simt_kernel(const __half* __restrict__ qkv,
                                                             const __half* __restrict__ pos_qk,
                                                             const __half* __restrict__ key_mask,
                                                             const int32_t* __restrict__ rel_table,
                                                             __half* __restrict__ ctx, int L, int heads) {
  __shared__ float probs[8][512];
  __shared__ int table[1024];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < 1023; i += blockDim.x) table[i] = rel_table[i];
  __syncthreads();
  const int q = blockIdx.x * 8 + warp;
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  if (q >= L) return;
  const int E = heads * 64;
  const long long row0 = (long long)b * L;
  float qv[64];
  load_row64(qkv + (row0 + q) * 3 * E + h * 64, qv);
  float lmax = -INFINITY;
  for (int k = lane; k < L; k += 32) {
    const __half* krow = qkv + (row0 + k) * 3 * E + E + h * 64;
    const int idx = table[q - k + 511];
    const __half* pq = pos_qk + (long long)idx * 2 * E + h * 64;
    const __half* pk = pos_qk + (long long)idx * 2 * E + E + h * 64;
    float kv[64];
    load_row64(krow, kv);
    float qk = 0.f;
#pragma unroll
    for (int d = 0; d < 64; ++d) qk = fmaf(qv[d], kv[d], qk);
    const float c2p = dot_row64(qv, pk);
    const float p2c = dot_row64(kv, pq);
    float s = qk * kInvSqrt192;
    if (__half2float(key_mask[row0 + k]) > 0.f)
      s += rel_bias_f16(c2p, p2c);
    else
      s += -65504.0f;
    probs[warp][k] = s;
    lmax = fmaxf(lmax, s);
  }
  const float m = ptx::warp_max(lmax);
  float lsum = 0.f;
  for (int k = lane; k < L; k += 32) {
    const float e = __expf(probs[warp][k] - m);
    probs[warp][k] = e;
    lsum += e;
  }
  const float inv = 1.0f / ptx::warp_sum(lsum);
  __syncwarp();
  float2 acc = make_float2(0.f, 0.f);
  const __half* vbase = qkv + row0 * 3 * E + 2 * E + h * 64 + 2 * lane;
  for (int k = 0; k < L; ++k) {
    const float p = probs[warp][k];
    const float2 v = __half22float2(*reinterpret_cast<const __half2*>(vbase + (long long)k * 3 * E));
    acc.x = fmaf(p, v.x, acc.x);
    acc.y = fmaf(p, v.y, acc.y);
  }
  *reinterpret_cast<__half2*>(ctx + (row0 + q) * E + h * 64 + 2 * lane) = __floats2half2_rn(acc.x * inv, acc.y * inv);
}

}  // namespace gdc
