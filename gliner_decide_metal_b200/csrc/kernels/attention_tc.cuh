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
//   TMA   K, V tiles [128 x 64] (double-buffered) and the PK / PQ windows [256 x 64]
//   MMA   S = Q K^T (TMEM cols 0-127), C = Q PKw^T (cols 128-383)
//   rows  drain C -> fp16 in SMEM (row q, 16-byte chunks XOR-swizzled by row)
//   MMA   P = K PQw^T into cols 128-383
//   rows  drain P -> fp16 in SMEM (row k) over the consumed windows; gather c2p from the
//         own row and p2c across rows, add the fp16 relative bias to S, online softmax
//         (fp32), write fp16 probabilities as a K-major SW128 operand
//   MMA   O_j = Prob . V (cols 384-447, V as an MN-major operand); the next pair's TMA is
//         issued here, overlapping the rest of this pair
//   rows  O = O * exp(m_old - m_new) + O_j in registers
// Threads: 8 row warps; warp w owns TMEM lane quarter w % 4 (query rows / key rows
// 32*(w%4)..+32) and half w / 4 of the columns / keys of every phase; warp 8 lane 0 issues
// TMA and MMA. Every wait is a bounded mbarrier wait.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>

#include "ptx.cuh"

namespace gdc {
namespace attn {

constexpr int kTile = 128;      // query rows per CTA and keys per tile
constexpr int kWin = 256;       // relative-position window rows per pair
constexpr int kRowWarps = 8;
constexpr int kRowThreads = kRowWarps * 32;
constexpr int kThreads = kRowThreads + 32;
constexpr int kTmemCols = 512;
constexpr uint32_t kColS = 0, kColCP = 128, kColO = 384;

// shared memory map (offsets from the 1024-aligned base)
constexpr int kOffQ = 0;                       // Q tile                16 KB
constexpr int kOffK = kOffQ + 16384;           // K tiles (2 buffers)   32 KB
constexpr int kOffV = kOffK + 32768;           // V tiles (2 buffers)   32 KB
constexpr int kOffW = kOffV + 32768;           // PK | PQ windows 2 x 32 KB, then P rows (64 KB)
constexpr int kOffC = kOffW + 65536;           // C rows 64 KB, then probabilities (32 KB)
constexpr int kOffTab = kOffC + 65536;         // relative index table, 1024 x int16
constexpr int kOffAdd = kOffTab + 2048;        // per key of the tile: 0 valid, -65504 masked, -inf beyond L
constexpr int kOffRed = kOffAdd + 512;         // cross-half max exchange, 2 x 128 f32
constexpr int kOffRedL = kOffRed + 1024;       // cross-half denominator exchange, 2 x 128 f32
constexpr int kOffFlags = kOffRedL + 1024;     // per key tile: any valid key (4 x int)
constexpr int kOffBar = kOffFlags + 64;        // mbarriers
constexpr int kNumBars = 12;
constexpr int kOffTmemSlot = kOffBar + kNumBars * 8;
constexpr int kSmemBytes = kOffTmemSlot + 16 + 1024;  // + alignment slack

enum Bar {
  kBarQ = 0, kBarKV0, kBarKV1, kBarSC, kBarCDone, kBarP, kBarProbs, kBarO, kBarODone, kBarRow, kBarDrain, kBarSpare
};

constexpr float kInvSqrt192f = 0.07216878364870322f;
constexpr float kInvScale16 = 1.0f / 13.859375f;  // 1 / fp16(sqrt(192))

// Byte offset of fp16 element (row, col) in a [rows x 256] fp16 block: rows of 512 bytes,
// 16-byte chunks XOR-swizzled by (row & 7). (col >> 3) << 4 == (2 col) & ~15, and the XOR
// touches only bits 4-6, so the offset inside a row is (2 col) ^ ((row & 7) << 4).
__device__ __forceinline__ uint32_t rowblk_off(int row, int col) {
  return uint32_t(row) * 512u + ((uint32_t(col) << 1) ^ (uint32_t(row & 7) << 4));
}

// Bounded rendezvous of the 256 row threads.
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

__device__ __forceinline__ void drain_rows_f16(uint32_t taddr, uint8_t* base, int row, int col0) {
  // four chunks of 32 fp32 TMEM columns -> fp16, 16-byte stores into the swizzled row
#pragma unroll 1
  for (int c = 0; c < 4; ++c) {
    uint32_t r[32];
    ptx::tmem_ld_32x32b_x32(taddr + uint32_t(c * 32), r);
    ptx::tmem_wait_ld();
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      uint4 v;
      v.x = ptx::pack_half2(__uint_as_float(r[u * 8 + 0]), __uint_as_float(r[u * 8 + 1]));
      v.y = ptx::pack_half2(__uint_as_float(r[u * 8 + 2]), __uint_as_float(r[u * 8 + 3]));
      v.z = ptx::pack_half2(__uint_as_float(r[u * 8 + 4]), __uint_as_float(r[u * 8 + 5]));
      v.w = ptx::pack_half2(__uint_as_float(r[u * 8 + 6]), __uint_as_float(r[u * 8 + 7]));
      *reinterpret_cast<uint4*>(base + rowblk_off(row, col0 + c * 32 + u * 8)) = v;
    }
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ CUtensorMap tm_pos,
                        const __half* __restrict__ key_mask, const int32_t* __restrict__ rel_table,
                        __half* __restrict__ ctx, int L, int heads, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  int16_t* s_tab = reinterpret_cast<int16_t*>(sm + kOffTab);
  float* s_add = reinterpret_cast<float*>(sm + kOffAdd);
  float* s_red = reinterpret_cast<float*>(sm + kOffRed);
  float* s_red_l = reinterpret_cast<float*>(sm + kOffRedL);
  int* s_flags = reinterpret_cast<int*>(sm + kOffFlags);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + kOffTmemSlot);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int q0 = blockIdx.x * kTile;
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int E = heads * 64;
  const int n_kt = (L + kTile - 1) / kTile;
  const long long row0 = (long long)b * L;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNumBars; ++i) ptx::mbar_init(&bars[i], 1);
    ptx::mbar_init(&bars[kBarCDone], kRowWarps);
    ptx::mbar_init(&bars[kBarProbs], kRowWarps);
    ptx::mbar_init(&bars[kBarODone], kRowWarps);
    ptx::mbar_init(&bars[kBarRow], kRowThreads);
    ptx::fence_barrier_init();
  }
  if (threadIdx.x < 4) s_flags[threadIdx.x] = 0;
  for (int i = threadIdx.x; i < 1023; i += kThreads) s_tab[i] = int16_t(rel_table[i]);
  if (warp == kRowWarps) {
    ptx::tmem_alloc(tmem_slot, kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  for (int k = threadIdx.x; k < L; k += kThreads)
    if (__half2float(key_mask[row0 + k]) > 0.f) s_flags[k / kTile] = 1;  // benign same-value race
  __syncthreads();
  int any_valid = 0;
  for (int t = 0; t < n_kt; ++t) any_valid |= s_flags[t];
  const uint32_t tbase = *tmem_slot;

  // key tile kt is processed unless every key in it is padding (and the row has a valid key)
  auto process = [&](int kt) { return !any_valid || s_flags[kt] != 0; };
  auto next_tile = [&](int kt) {
    for (++kt; kt < n_kt; ++kt)
      if (process(kt)) return kt;
    return n_kt;
  };
  auto window_lo = [&](int k0) {
    const int lo = s_tab[q0 - (k0 + kTile - 1) + 511];
    return lo < 512 - kWin ? lo : 512 - kWin;
  };

  if (warp == kRowWarps) {
    if (lane == 0) {
      uint8_t* sQ = sm + kOffQ;
      uint8_t* sPK = sm + kOffW;
      uint8_t* sPQ = sm + kOffW + 32768;
      const uint32_t id_s = ptx::idesc_f16_f32(128, 128);
      const uint32_t id_cp = ptx::idesc_f16_f32(128, 256);
      const uint32_t id_pv = ptx::idesc_f16_f32(128, 64, 1);
      const uint32_t aQ = ptx::smem_u32(sQ), aPK = ptx::smem_u32(sPK), aPQ = ptx::smem_u32(sPQ);
      const uint32_t aProb = ptx::smem_u32(sm + kOffC);
      ptx::prefetch_tensor_map(&tm_qkv);
      ptx::prefetch_tensor_map(&tm_pos);
      auto issue_loads = [&](int kt, int buf) {
        const int k0 = kt * kTile;
        const int lo = window_lo(k0);
        uint64_t* bar = &bars[kBarKV0 + buf];
        ptx::mbar_arrive_expect_tx(bar, 2 * 16384 + 2 * 32768);
        ptx::tma_load_2d(sm + kOffK + buf * 16384, &tm_qkv, E + h * 64, int(row0 + k0), bar);
        ptx::tma_load_2d(sm + kOffV + buf * 16384, &tm_qkv, 2 * E + h * 64, int(row0 + k0), bar);
        ptx::tma_load_2d(sPK, &tm_pos, E + h * 64, lo, bar);
        ptx::tma_load_2d(sPQ, &tm_pos, h * 64, lo, bar);
      };
      ptx::mbar_arrive_expect_tx(&bars[kBarQ], 16384);
      ptx::tma_load_2d(sQ, &tm_qkv, h * 64, int(row0 + q0), &bars[kBarQ]);
      int kt = next_tile(-1);
      int np = 0;
      int loads_issued = 0;
      if (kt < n_kt) {
        issue_loads(kt, 0);
        loads_issued = 1;
      }
      bool ok = ptx::mbar_wait(&bars[kBarQ], 0, err);
      for (; ok && kt < n_kt; kt = next_tile(kt), ++np) {
        const int buf = np & 1;
        const uint32_t par = uint32_t(np & 1);
        if (!ptx::mbar_wait(&bars[kBarKV0 + buf], uint32_t((np >> 1) & 1), err)) break;
        ptx::tc_fence_after();
        const uint32_t aK = ptx::smem_u32(sm + kOffK + buf * 16384);
        const uint32_t aV = ptx::smem_u32(sm + kOffV + buf * 16384);
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
        // probabilities written; every row thread is past its gathers (windows free)
        if (!ptx::mbar_wait(&bars[kBarProbs], par, err)) break;
        // O of the previous pair has been read out of TMEM
        if (np > 0 && !ptx::mbar_wait(&bars[kBarODone], par ^ 1u, err)) break;
        ptx::tc_fence_after();
#pragma unroll
        for (int s = 0; s < 8; ++s)
          ptx::umma_f16_ss(tbase + kColO, ptx::desc_kmajor_sw128(aProb + (s >> 2) * 16384 + (s & 3) * 32),
                           ptx::desc_mnmajor_sw128(aV + s * 2048), id_pv, s > 0);
        ptx::umma_commit(&bars[kBarO]);
        // prefetch the next pair: its K/V buffer was last read by PV of pair np-1 (done,
        // O(np-1) was read), the windows were last read by this pair's P MMA (done)
        const int nk = next_tile(kt);
        if (nk < n_kt) {
          issue_loads(nk, buf ^ 1);
          ++loads_issued;
        }
      }
      // drain outstanding tensor-core work and TMA loads before TMEM is released
      ptx::umma_commit(&bars[kBarDrain]);
      const unsigned long long t0 = ptx::globaltimer();
      while (!ptx::mbar_try_wait(&bars[kBarDrain], 0) && ptx::globaltimer() - t0 < ptx::kTimeoutNs) {
      }
      // wait for the last issued K/V load of each buffer (bounded)
      for (int j = loads_issued - 2 < 0 ? 0 : loads_issued - 2; j < loads_issued; ++j) {
        const unsigned long long t1 = ptx::globaltimer();
        while (!ptx::mbar_try_wait(&bars[kBarKV0 + (j & 1)], uint32_t((j >> 1) & 1)) &&
               ptx::globaltimer() - t1 < ptx::kTimeoutNs) {
        }
      }
      if (!ok) {
        const unsigned long long t2 = ptx::globaltimer();
        while (!ptx::mbar_try_wait(&bars[kBarQ], 0) && ptx::globaltimer() - t2 < ptx::kTimeoutNs) {
        }
      }
    }
  } else {
    // ---------------------------------------------------------------- row threads
    const int quarter = warp & 3;
    const int half = warp >> 2;
    const int t = quarter * 32 + lane;  // TMEM lane; query row q0 + t; key row k0 + t
    const int q = q0 + t;
    const uint32_t lane_base = tbase + (uint32_t(quarter * 32) << 16);
    uint8_t* sC = sm + kOffC;
    uint8_t* sPst = sm + kOffW;
    const uint32_t c_row = uint32_t(t) * 512u;
    const uint32_t c_xor = uint32_t(t & 7) << 4;
    RowSync rs{&bars[kBarRow]};
    float o[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) o[i] = 0.f;
    float m_run = -INFINITY, l_half = 0.f;
    int np = 0;
    bool ok = true;
    for (int kt = next_tile(-1); kt < n_kt; kt = next_tile(kt), ++np) {
      const int k0 = kt * kTile;
      const int lo = window_lo(k0);
      const uint32_t par = uint32_t(np & 1);
      if (half == 0) {
        const int k = k0 + t;
        s_add[t] = k >= L ? -INFINITY : (__half2float(key_mask[row0 + k]) > 0.f ? 0.f : -65504.0f);
      }
      // ---- drain C (own query row, this half's 128 columns)
      if (!ptx::mbar_wait(&bars[kBarSC], par, err)) {
        ok = false;
        break;
      }
      ptx::tc_fence_after();
      drain_rows_f16(lane_base + kColCP + half * 128, sC, t, half * 128);
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&bars[kBarCDone]);
      // ---- drain P (own key row) over the consumed windows
      if (!ptx::mbar_wait(&bars[kBarP], par, err)) {
        ok = false;
        break;
      }
      ptx::tc_fence_after();
      drain_rows_f16(lane_base + kColCP + half * 128, sPst, t, half * 128);
      ptx::tc_fence_before();
      if (!rs.sync(err)) {
        ok = false;
        break;
      }
      // ---- scores of keys [half*64, half*64 + 64) with the gathered relative bias
      const int16_t* tab_q = s_tab + (q - k0 + 511);  // tab_q[-kk] = i(q - (k0 + kk))
      float sc[64];
      float part_max = -INFINITY;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t r[32];
        ptx::tmem_ld_32x32b_x32(lane_base + kColS + half * 64 + c * 32, r);
        ptx::tmem_wait_ld();
#pragma unroll
        for (int u = 0; u < 32; ++u) {
          const int kk = half * 64 + c * 32 + u;
          const uint32_t w2 = uint32_t(int(tab_q[-kk]) - lo) << 1;  // 2 * window column
          const __half cv = *reinterpret_cast<const __half*>(sC + c_row + (w2 ^ c_xor));
          const __half pv =
              *reinterpret_cast<const __half*>(sPst + uint32_t(kk) * 512u + (w2 ^ (uint32_t(kk & 7) << 4)));
          const float rb = __half2float(__float2half_rn(__half2float(__hadd(cv, pv)) * kInvScale16));
          const float add = s_add[kk];
          const float s = fmaf(__uint_as_float(r[u]), kInvSqrt192f, add == 0.f ? rb : add);
          sc[c * 32 + u] = s;
          part_max = fmaxf(part_max, s);
        }
      }
      s_red[half * 128 + t] = part_max;
      // all rows are past their C / P reads (probabilities overwrite the C rows, the next
      // pair's windows overwrite the P rows) and both halves' maxima are visible
      if (!rs.sync(err)) {
        ok = false;
        break;
      }
      const float m_new = fmaxf(m_run, fmaxf(s_red[t], s_red[128 + t]));
      const float alpha = __expf(m_run - m_new);
      float psum = 0.f;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint32_t pk[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int i = c * 8 + 2 * j;
          const __half2 p2 = __floats2half2_rn(__expf(sc[i] - m_new), __expf(sc[i + 1] - m_new));
          const float2 pf = __half22float2(p2);
          psum += pf.x + pf.y;
          pk[j] = *reinterpret_cast<const uint32_t*>(&p2);
        }
        // K-major SW128 operand: atom `half` holds keys half*64..+63 of row t
        const uint32_t off = uint32_t(half) * 16384u + uint32_t(t >> 3) * 1024u + uint32_t(t & 7) * 128u +
                             ((uint32_t(c) ^ uint32_t(t & 7)) << 4);
        *reinterpret_cast<uint4*>(sC + off) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
      ptx::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&bars[kBarProbs]);
      l_half = l_half * alpha + psum;
      m_run = m_new;
      // ---- accumulate this half's 32 columns of O_j
      if (!ptx::mbar_wait(&bars[kBarO], par, err)) {
        ok = false;
        break;
      }
      ptx::tc_fence_after();
      {
        uint32_t r[32];
        ptx::tmem_ld_32x32b_x32(lane_base + kColO + half * 32, r);
        ptx::tmem_wait_ld();
#pragma unroll
        for (int u = 0; u < 32; ++u) o[u] = o[u] * alpha + __uint_as_float(r[u]);
      }
      ptx::tc_fence_before();
      ptx::fence_proxy_async_smem();  // generic P-row / C-row writes precede later TMA / MMA use
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&bars[kBarODone]);
    }
    // combine the two halves' softmax denominators and store this half's 32 columns
    if (ok) {
      s_red_l[half * 128 + t] = l_half;
      if (!rs.sync(err)) ok = false;
    }
    if (ok && q < L && np > 0) {
      const float inv = 1.0f / (s_red_l[t] + s_red_l[128 + t]);
      __half* dst = ctx + (row0 + q) * (long long)E + h * 64 + half * 32;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
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
  if (warp == kRowWarps) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tbase, kTmemCols);
  }
}

}  // namespace attn
}  // namespace gdc
