// Disentangled attention on tcgen05 tensor cores (sm_100a).
//
// Computes, per (batch b, head h), exactly the reference's default path
// (DeBERTa.swift:322-395):
//   c2p[q,k] = fp16(q . PK[i(q-k)]),  p2c[q,k] = fp16(k . PQ[i(q-k)])
//   rb[q,k]  = fp16(fp16(c2p + p2c) / fp16(sqrt 192))
//   s[q,k]   = (q . k) / sqrt(192) + (key valid ? rb : -65504)
//   ctx[q]   = softmax_k(s) . V
// with i(r) = clip(bucket(r) + 256, 0, 511) from the 1023-entry table.
//
// One CTA per (128-query tile, h, b); it walks the 128-key tiles of the row (tiles
// whose keys are all padding are skipped: their softmax weight is exactly zero). For a
// (query tile, key tile) pair the relative distances q-k span 255 values, so the needed
// position rows form one window [lo, lo+256) of PQ / PK. Per pair:
//   TMA   K, V tiles [128 x 64] and the PK / PQ windows [256 x 64] (128B swizzle)
//   MMA   S = Q K^T (TMEM cols 0-127), C = Q PKw^T (cols 128-383)
//   rows  drain C -> fp16 in SMEM (row q, 128B-chunk XOR swizzle)
//   MMA   P = K PQw^T into cols 128-383
//   rows  drain P -> fp16 in SMEM (row k); gather c2p from the own row and p2c across
//         rows, add the fp16 relative bias to S, online softmax (fp32), write the fp16
//         probabilities as a K-major SW128 operand
//   MMA   O_j = Prob . V (cols 384-447, V as an MN-major operand)
//   rows  O = O * exp(m_old - m_new) + O_j in registers
// Threads: warps 0-3 own TMEM lanes / query rows (one thread per row); warp 4 lane 0
// issues TMA and MMA. All waits are bounded mbarrier waits.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>

#include "ptx.cuh"

namespace gdc {
namespace attn {

constexpr int kTile = 128;      // query rows per CTA and keys per tile
constexpr int kWin = 256;       // relative-position window rows per pair
constexpr int kThreads = 160;   // 4 row warps + 1 control warp
constexpr int kTmemCols = 512;
constexpr uint32_t kColS = 0, kColCP = 128, kColO = 384;

// shared memory map (offsets from the 1024-aligned base)
constexpr int kOffQ = 0;                       // Q tile       16 KB
constexpr int kOffK = kOffQ + 16384;           // K tile       16 KB
constexpr int kOffV = kOffK + 16384;           // V tile       16 KB
constexpr int kOffW = kOffV + 16384;           // PK | PQ windows 2 x 32 KB, then P rows (64 KB)
constexpr int kOffC = kOffW + 65536;           // C rows 64 KB, then probabilities (32 KB)
constexpr int kOffTab = kOffC + 65536;         // relative index table, 1024 x int16
constexpr int kOffMask = kOffTab + 2048;       // key-mask values of the tile, 128 x f32
constexpr int kOffFlags = kOffMask + 512;      // per key tile: any valid key (4 x int)
constexpr int kOffBar = kOffFlags + 64;        // mbarriers
constexpr int kNumBars = 10;
constexpr int kOffTmemSlot = kOffBar + kNumBars * 8;
constexpr int kSmemBytes = kOffTmemSlot + 16 + 1024;  // + alignment slack

enum Bar { kBarQ = 0, kBarKV, kBarSC, kBarCDone, kBarP, kBarProbs, kBarO, kBarODone, kBarRow, kBarDrain };

constexpr float kInvSqrt192f = 0.07216878364870322f;
constexpr float kInvScale16 = 1.0f / 13.859375f;  // 1 / fp16(sqrt(192))
constexpr float kLog2e = 1.4426950408889634f;

// byte offset of fp16 element (row, col) in a [rows x 256] fp16 block whose 16-byte
// chunks are XOR-swizzled by (row & 7) inside each row of 512 bytes.
__device__ __forceinline__ uint32_t rowblk_off(int row, int col) {
  return uint32_t(row) * 512u + ((uint32_t(col >> 3) ^ uint32_t(row & 7)) << 4) + (uint32_t(col & 7) << 1);
}

// Bounded wait on a CTA-local barrier used as a rendezvous of the 128 row threads.
struct RowSync {
  uint64_t* bar;
  uint32_t phase = 0;
  __device__ __forceinline__ bool sync(int* err) {
    ptx::mbar_arrive(bar);
    const bool ok = ptx::mbar_wait(bar, phase, err);
    phase ^= 1u;
    return ok;
  }
};

__global__ void __launch_bounds__(kThreads, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ CUtensorMap tm_pos,
                        const __half* __restrict__ key_mask, const int32_t* __restrict__ rel_table,
                        __half* __restrict__ ctx, int L, int heads, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  int16_t* s_tab = reinterpret_cast<int16_t*>(sm + kOffTab);
  float* s_mask = reinterpret_cast<float*>(sm + kOffMask);
  int* s_flags = reinterpret_cast<int*>(sm + kOffFlags);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + kOffTmemSlot);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int qt = blockIdx.x;
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int q0 = qt * kTile;
  const int E = heads * 64;
  const int n_kt = (L + kTile - 1) / kTile;
  const long long row0 = (long long)b * L;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNumBars; ++i) ptx::mbar_init(&bars[i], 1);
    ptx::mbar_init(&bars[kBarCDone], 4);
    ptx::mbar_init(&bars[kBarProbs], 4);
    ptx::mbar_init(&bars[kBarODone], 4);
    ptx::mbar_init(&bars[kBarRow], 128);
    ptx::fence_barrier_init();
  }
  if (threadIdx.x < 4) s_flags[threadIdx.x] = 0;
  for (int i = threadIdx.x; i < 1023; i += kThreads) s_tab[i] = int16_t(rel_table[i]);
  if (warp == 4) {
    ptx::tmem_alloc(tmem_slot, kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  // which key tiles hold at least one valid key
  for (int k = threadIdx.x; k < L; k += kThreads)
    if (__half2float(key_mask[row0 + k]) > 0.f) s_flags[k / kTile] = 1;  // benign same-value race
  __syncthreads();
  int any_valid = 0;
  for (int t = 0; t < n_kt; ++t) any_valid |= s_flags[t];
  const uint32_t tbase = *tmem_slot;

  // tile kt is processed unless every key in it is padding (and the row has a valid key)
  auto process = [&](int kt) { return !any_valid || s_flags[kt] != 0; };
  auto window_lo = [&](int k0) {
    int lo = s_tab[q0 - (k0 + kTile - 1) + 511];
    return lo < 512 - kWin ? lo : 512 - kWin;
  };

  if (warp == 4) {
    if (lane == 0) {
      uint8_t* sQ = sm + kOffQ;
      uint8_t* sK = sm + kOffK;
      uint8_t* sV = sm + kOffV;
      uint8_t* sPK = sm + kOffW;
      uint8_t* sPQ = sm + kOffW + 32768;
      uint8_t* sProb = sm + kOffC;
      const uint32_t id_s = ptx::idesc_f16_f32(128, 128);
      const uint32_t id_cp = ptx::idesc_f16_f32(128, 256);
      const uint32_t id_pv = ptx::idesc_f16_f32(128, 64, 1);
      ptx::prefetch_tensor_map(&tm_qkv);
      ptx::prefetch_tensor_map(&tm_pos);
      ptx::mbar_arrive_expect_tx(&bars[kBarQ], 16384);
      ptx::tma_load_2d(sQ, &tm_qkv, h * 64, int(row0 + q0), &bars[kBarQ]);
      bool ok = true;
      int np = 0;
      bool kv_pending = false;
      for (int kt = 0; kt < n_kt && ok; ++kt) {
        if (!process(kt)) continue;
        const int k0 = kt * kTile;
        const int lo = window_lo(k0);
        const uint32_t par = uint32_t(np & 1);
        if (np > 0 && !ptx::mbar_wait(&bars[kBarODone], par ^ 1u, err)) break;
        ptx::mbar_arrive_expect_tx(&bars[kBarKV], 2 * 16384 + 2 * 32768);
        ptx::tma_load_2d(sK, &tm_qkv, E + h * 64, int(row0 + k0), &bars[kBarKV]);
        ptx::tma_load_2d(sV, &tm_qkv, 2 * E + h * 64, int(row0 + k0), &bars[kBarKV]);
        ptx::tma_load_2d(sPK, &tm_pos, E + h * 64, lo, &bars[kBarKV]);
        ptx::tma_load_2d(sPQ, &tm_pos, h * 64, lo, &bars[kBarKV]);
        kv_pending = true;
        if (np == 0 && !ptx::mbar_wait(&bars[kBarQ], 0, err)) break;
        if (!ptx::mbar_wait(&bars[kBarKV], par, err)) break;
        kv_pending = false;
        ptx::tc_fence_after();
        const uint32_t aQ = ptx::smem_u32(sQ), aK = ptx::smem_u32(sK), aV = ptx::smem_u32(sV);
        const uint32_t aPK = ptx::smem_u32(sPK), aPQ = ptx::smem_u32(sPQ), aP = ptx::smem_u32(sProb);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          ptx::umma_f16_ss(tbase + kColS, ptx::desc_kmajor_sw128(aQ + k * 32), ptx::desc_kmajor_sw128(aK + k * 32),
                           id_s, k > 0);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          ptx::umma_f16_ss(tbase + kColCP, ptx::desc_kmajor_sw128(aQ + k * 32),
                           ptx::desc_kmajor_sw128(aPK + k * 32), id_cp, k > 0);
        ptx::umma_commit(&bars[kBarSC]);
        if (!ptx::mbar_wait(&bars[kBarCDone], par, err)) break;
        ptx::tc_fence_after();
#pragma unroll
        for (int k = 0; k < 4; ++k)
          ptx::umma_f16_ss(tbase + kColCP, ptx::desc_kmajor_sw128(aK + k * 32),
                           ptx::desc_kmajor_sw128(aPQ + k * 32), id_cp, k > 0);
        ptx::umma_commit(&bars[kBarP]);
        if (!ptx::mbar_wait(&bars[kBarProbs], par, err)) break;
        ptx::tc_fence_after();
#pragma unroll
        for (int s = 0; s < 8; ++s)
          ptx::umma_f16_ss(tbase + kColO, ptx::desc_kmajor_sw128(aP + (s >> 2) * 16384 + (s & 3) * 32),
                           ptx::desc_mnmajor_sw128(aV + s * 2048), id_pv, s > 0);
        ptx::umma_commit(&bars[kBarO]);
        ++np;
      }
      // drain outstanding tensor-core work and TMA loads before TMEM is released
      ptx::umma_commit(&bars[kBarDrain]);
      const unsigned long long t0 = ptx::globaltimer();
      while (!ptx::mbar_try_wait(&bars[kBarDrain], 0) && ptx::globaltimer() - t0 < ptx::kTimeoutNs) {
      }
      if (kv_pending) {
        const uint32_t par = uint32_t(np & 1);
        const unsigned long long t1 = ptx::globaltimer();
        while (!ptx::mbar_try_wait(&bars[kBarKV], par) && ptx::globaltimer() - t1 < ptx::kTimeoutNs) {
        }
      }
      if (np == 0) {
        const unsigned long long t2 = ptx::globaltimer();
        while (!ptx::mbar_try_wait(&bars[kBarQ], 0) && ptx::globaltimer() - t2 < ptx::kTimeoutNs) {
        }
      }
    }
  } else {
    // ---------------------------------------------------------------- row threads
    const int t = threadIdx.x;  // 0..127: TMEM lane, query row q0 + t, key row k0 + t
    const int q = q0 + t;
    const uint32_t lane_base = tbase + (uint32_t(warp * 32) << 16);
    uint8_t* sC = sm + kOffC;
    uint8_t* sPst = sm + kOffW;
    RowSync rs{&bars[kBarRow]};
    float o[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) o[i] = 0.f;
    float m_run = -INFINITY, l_run = 0.f;
    int np = 0;
    bool ok = true;
    for (int kt = 0; kt < n_kt && ok; ++kt) {
      if (!process(kt)) continue;
      const int k0 = kt * kTile;
      const int lo = window_lo(k0);
      const uint32_t par = uint32_t(np & 1);
      // key-mask values of this tile (thread t loads key k0 + t)
      {
        const int k = k0 + t;
        s_mask[t] = k < L ? __half2float(key_mask[row0 + k]) : 0.f;
      }
      // ---- drain C (own query row) into fp16 rows
      if (!ptx::mbar_wait(&bars[kBarSC], par, err)) {
        ok = false;
        break;
      }
      ptx::tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < 8; ++c) {
        uint32_t r[32];
        ptx::tmem_ld_32x32b_x32(lane_base + kColCP + c * 32, r);
        ptx::tmem_wait_ld();
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          uint4 v;
          v.x = ptx::pack_half2(__uint_as_float(r[u * 8 + 0]), __uint_as_float(r[u * 8 + 1]));
          v.y = ptx::pack_half2(__uint_as_float(r[u * 8 + 2]), __uint_as_float(r[u * 8 + 3]));
          v.z = ptx::pack_half2(__uint_as_float(r[u * 8 + 4]), __uint_as_float(r[u * 8 + 5]));
          v.w = ptx::pack_half2(__uint_as_float(r[u * 8 + 6]), __uint_as_float(r[u * 8 + 7]));
          *reinterpret_cast<uint4*>(sC + rowblk_off(t, c * 32 + u * 8)) = v;
        }
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&bars[kBarCDone]);
      // ---- drain P (own key row) into fp16 rows (over the consumed PK / PQ windows)
      if (!ptx::mbar_wait(&bars[kBarP], par, err)) {
        ok = false;
        break;
      }
      ptx::tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < 8; ++c) {
        uint32_t r[32];
        ptx::tmem_ld_32x32b_x32(lane_base + kColCP + c * 32, r);
        ptx::tmem_wait_ld();
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          uint4 v;
          v.x = ptx::pack_half2(__uint_as_float(r[u * 8 + 0]), __uint_as_float(r[u * 8 + 1]));
          v.y = ptx::pack_half2(__uint_as_float(r[u * 8 + 2]), __uint_as_float(r[u * 8 + 3]));
          v.z = ptx::pack_half2(__uint_as_float(r[u * 8 + 4]), __uint_as_float(r[u * 8 + 5]));
          v.w = ptx::pack_half2(__uint_as_float(r[u * 8 + 6]), __uint_as_float(r[u * 8 + 7]));
          *reinterpret_cast<uint4*>(sPst + rowblk_off(t, c * 32 + u * 8)) = v;
        }
      }
      ptx::tc_fence_before();
      if (!rs.sync(err)) {
        ok = false;
        break;
      }
      // ---- scores with the gathered relative bias
      float sc[kTile];
      float tile_max = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        ptx::tmem_ld_32x32b_x32(lane_base + kColS + c * 32, r);
        ptx::tmem_wait_ld();
#pragma unroll
        for (int u = 0; u < 32; ++u) {
          const int kk = c * 32 + u;
          const int k = k0 + kk;
          const int w = int(s_tab[q - k + 511]) - lo;
          const __half cv = *reinterpret_cast<const __half*>(sC + rowblk_off(t, w));
          const __half pv = *reinterpret_cast<const __half*>(sPst + rowblk_off(kk, w));
          const float sum16 = __half2float(__hadd(cv, pv));
          const float rb = __half2float(__float2half_rn(sum16 * kInvScale16));
          const float mk = s_mask[kk];
          float s = __uint_as_float(r[u]) * kInvSqrt192f + (mk > 0.f ? rb : -65504.0f);
          s = (k < L) ? s : -INFINITY;
          sc[kk] = s;
          tile_max = fmaxf(tile_max, s);
        }
      }
      // all rows done reading C / P rows: the probability operand overwrites the C rows
      if (!rs.sync(err)) {
        ok = false;
        break;
      }
      const float m_new = fmaxf(m_run, tile_max);
      const float alpha = exp2f((m_run - m_new) * kLog2e);
      float psum = 0.f;
#pragma unroll
      for (int a = 0; a < 2; ++a) {
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint32_t pk[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int kk = a * 64 + c * 8 + 2 * j;
            const __half2 p2 = __floats2half2_rn(exp2f((sc[kk] - m_new) * kLog2e),
                                                 exp2f((sc[kk + 1] - m_new) * kLog2e));
            const float2 pf = __half22float2(p2);
            psum += pf.x + pf.y;
            pk[j] = *reinterpret_cast<const uint32_t*>(&p2);
          }
          const uint32_t off = uint32_t(a) * 16384u + uint32_t(t >> 3) * 1024u + uint32_t(t & 7) * 128u +
                               ((uint32_t(c) ^ uint32_t(t & 7)) << 4);
          *reinterpret_cast<uint4*>(sC + off) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        }
      }
      ptx::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&bars[kBarProbs]);
      l_run = l_run * alpha + psum;
      m_run = m_new;
      // ---- accumulate O_j
      if (!ptx::mbar_wait(&bars[kBarO], par, err)) {
        ok = false;
        break;
      }
      ptx::tc_fence_after();
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t r[32];
        ptx::tmem_ld_32x32b_x32(lane_base + kColO + c * 32, r);
        ptx::tmem_wait_ld();
#pragma unroll
        for (int u = 0; u < 32; ++u) o[c * 32 + u] = o[c * 32 + u] * alpha + __uint_as_float(r[u]);
      }
      ptx::tc_fence_before();
      ptx::fence_proxy_async_smem();  // generic P-row writes precede the next TMA into that region
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&bars[kBarODone]);
      ++np;
    }
    if (ok && q < L && np > 0) {
      const float inv = 1.0f / l_run;
      __half* dst = ctx + (row0 + q) * (long long)E + h * 64;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint4 v;
        v.x = ptx::pack_half2(o[c * 8 + 0] * inv, o[c * 8 + 1] * inv);
        v.y = ptx::pack_half2(o[c * 8 + 2] * inv, o[c * 8 + 3] * inv);
        v.z = ptx::pack_half2(o[c * 8 + 4] * inv, o[c * 8 + 5] * inv);
        v.w = ptx::pack_half2(o[c * 8 + 6] * inv, o[c * 8 + 7] * inv);
        reinterpret_cast<uint4*>(dst)[c] = v;
      }
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tbase, kTmemCols);
  }
}

}  // namespace attn
}  // namespace gdc
