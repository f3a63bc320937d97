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
// Persistent: one CTA per SM takes work items (128-query tile, h, b) one at a time (from an
// atomic counter, heaviest first, or a static split; see Schedule) and, inside an item,
// walks the 128-key tiles of the row (tiles whose keys are all padding are skipped: their
// softmax weight is exactly zero). With packed rows (Schedule::seq_off) a batch row's
// positions sit at rows seq_off[b] + t of qkv / ctx, query tiles past its extent are never
// handed out and keys past it get weight zero. For a (query tile, key tile) pair the
// distances q-k span 255 values, so the needed position rows form one window
// [lo, lo+256) of PQ / PK.
// Per pair:
//   TMA   K, V tiles [128 x 64] (double-buffered) and the PK / PQ windows [256 x 64];
//         Q [128 x 64] once per item. The next pair's loads (possibly of the next item)
//         are issued as soon as this pair's gathers are done.
//   MMA   S = Q K^T (TMEM cols 0-127), C = Q PKw^T (cols 128-383)
//   rows  drain C -> fp16 in SMEM (row q, 16-byte chunks XOR-swizzled by row)
//   MMA   P = K PQw^T into cols 128-383
//   rows  drain P -> fp16 in SMEM (row k) over the consumed windows; gather c2p from the
//         own row and p2c across rows, add the fp16 relative bias to S, online softmax
//         (fp32), write fp16 probabilities as a K-major SW128 operand
//   MMA   O += Prob . V (cols 384-447, V as an MN-major operand); before it the rows
//         rescale O in TMEM by exp(m_old - m_new) when a row's running max changed
// Threads: 4 * kParts row warps; warp w owns TMEM lane quarter w % 4 (query rows / key rows
// 32*(w%4)..+32) and part w / 4 of the columns / keys of every phase. The next warp's lane 0
// issues the MMAs; the last warp issues the TMA loads (and scans key masks). Every wait is a
// bounded mbarrier wait; the row warps sleep in theirs.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>

#include "kernels.h"
#include "ptx.cuh"

namespace gdc {
namespace attn {

constexpr int kTile = 128;      // query rows per item and keys per tile
constexpr int kWin = 256;       // relative-position window rows per pair
#ifndef GDC_ATTN_PARTS
#define GDC_ATTN_PARTS 2
#endif
constexpr int kParts = GDC_ATTN_PARTS;   // row warps per TMEM lane quarter (2 or 4)
constexpr int kRowWarps = 4 * kParts;
constexpr int kColsPP = 256 / kParts;    // C / P columns drained per row warp
constexpr int kKeysPP = 128 / kParts;    // keys scored per row warp
constexpr int kOPP = 64 / kParts;        // O columns accumulated per row warp
constexpr int kRowThreads = kRowWarps * 32;
constexpr int kThreads = kRowThreads + 64;  // + MMA issuer warp + TMA producer warp
constexpr int kTmemCols = 512;
constexpr uint32_t kColS = 0, kColCP = 128, kColO = 384;

// shared memory map (offsets from the 1024-aligned base)
constexpr int kOffQ = 0;                       // Q tile                16 KB
constexpr int kOffK = kOffQ + 16384;           // K tiles (2 buffers)   32 KB
constexpr int kOffV = kOffK + 32768;           // V tiles (2 buffers)   32 KB
constexpr int kOffW = kOffV + 32768;           // PK | PQ windows 2 x 32 KB, then P rows (64 KB)
constexpr int kOffC = kOffW + 65536;           // C rows 64 KB, then probabilities (32 KB)
constexpr int kOffTab = kOffC + 65536;         // relative index table, 1024 x int16
constexpr int kOffAdd = kOffTab + 2048;        // per item (2 slots) and key: 0 valid, -65504 masked, -inf past
                                               // the extent; 2 x 512 f32
constexpr int kOffRed = kOffAdd + 4096;        // cross-part max exchange, 4 x 128 f32
constexpr int kOffRedL = kOffRed + 2048;       // cross-part denominator exchange, 4 x 128 f32
constexpr int kOffFlags = kOffRedL + 2048;     // per item (2 slots): key-tile mask, item index, extent, row base
constexpr int kOffBar = kOffFlags + 64;        // mbarriers
constexpr int kNumBars = 15;
constexpr int kOffTmemSlot = kOffBar + kNumBars * 8;
constexpr int kSmemBytes = kOffTmemSlot + 16 + 1024;  // + alignment slack

enum Bar {
  kBarQ = 0, kBarKV0, kBarKV1, kBarSC, kBarCDone, kBarP, kBarProbs, kBarO, kBarODone, kBarRow, kBarDrain, kBarFlags,
  kBarKVFree0, kBarKVFree1, kBarScored
};

constexpr float kInvSqrt192f = 0.07216878364870322f;
constexpr float kInvScale16 = 1.0f / 13.859375f;  // 1 / fp16(sqrt(192))

// Byte offset of fp16 element (row, col) in a [rows x 256] fp16 block: rows of 512 bytes,
// 16-byte chunks XOR-swizzled by (row & 7). (col >> 3) << 4 == (2 col) & ~15, and the XOR
// touches only bits 4-6, so the offset inside a row is (2 col) ^ ((row & 7) << 4).
__device__ __forceinline__ uint32_t rowblk_off(int row, int col) {
  return uint32_t(row) * 512u + ((uint32_t(col) << 1) ^ (uint32_t(row & 7) << 4));
}

// 2^x with the hardware approximation (MUFU.EX2); the exp phase computes
// exp(s - m) = 2^(s log2 e - m log2 e) with one FFMA per probability.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Bounded rendezvous of all row threads.
struct RowSync {
  uint64_t* bar;
  uint32_t phase = 0;
  __device__ __forceinline__ bool sync(int* err) {
    ptx::mbar_arrive(bar);
    const bool ok = ptx::mbar_wait_sleep(bar, phase, err);
    phase ^= 1u;
    return ok;
  }
};

// kColsPP fp32 TMEM columns of this thread's lane -> fp16, 16-byte stores into the swizzled row.
__device__ __forceinline__ void drain_rows_f16(uint32_t taddr, uint8_t* base, int row, int col0) {
#pragma unroll
  for (int c = 0; c < kColsPP / 32; ++c) {
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

__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[32]) { ptx::tmem_ld_32x32b_x32(taddr, r); }
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[16]) { ptx::tmem_ld_32x32b_x16(taddr, r); }
__device__ __forceinline__ void tmem_st_cols(uint32_t taddr, const uint32_t (&r)[32]) { ptx::tmem_st_32x32b_x32(taddr, r); }
__device__ __forceinline__ void tmem_st_cols(uint32_t taddr, const uint32_t (&r)[16]) { ptx::tmem_st_32x32b_x16(taddr, r); }

// Work item decomposition: item = (b * heads + h) * n_qt + qt.
struct Item {
  int qt, h, b;
};

__device__ __forceinline__ Item decode_item(int item, int n_qt, int heads) {
  Item it;
  it.qt = item % n_qt;
  it.h = (item / n_qt) % heads;
  it.b = item / (n_qt * heads);
  return it;
}

// Key-mask values of one batch row as seen by one lane of a warp: lane l holds keys
// [8l, 8l + 8) and [256 + 8l, 256 + 8l + 8) (L <= 512), loaded up front so the scan for
// the next work item can be issued one item ahead and its latency hidden.
struct MaskChunk {
  uint4 v[2];
};

__device__ __forceinline__ MaskChunk load_mask_chunk(const __half* key_mask, long long row0, int L) {
  MaskChunk c;
  const int lane = int(ptx::lane_id());
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int k = h * 256 + lane * 8;
    const __half* src = key_mask + row0 + k;
    if (k + 8 <= L && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
      c.v[h] = __ldg(reinterpret_cast<const uint4*>(src));
    } else {
      uint32_t w[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t lo16 = (k + 2 * j < L) ? uint32_t(__half_as_ushort(src[2 * j])) : 0u;
        const uint32_t hi16 = (k + 2 * j + 1 < L) ? uint32_t(__half_as_ushort(src[2 * j + 1])) : 0u;
        w[j] = lo16 | (hi16 << 16);
      }
      c.v[h] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
  return c;
}

// Mask of key tiles to process for a batch row: tiles with a valid key, or every tile when
// the row has none (the mask then only shifts all scores equally). Executed by a full warp.
__device__ __forceinline__ uint32_t key_tile_mask(const MaskChunk& c, int n_kt) {
  uint32_t m = 0;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const __half2* p = reinterpret_cast<const __half2*>(&c.v[h]);
    bool any = false;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __half22float2(p[j]);
      any |= (f.x > 0.f) | (f.y > 0.f);
    }
    const uint32_t bits = __ballot_sync(0xffffffffu, any);  // lanes 0-15: tile 2h, 16-31: tile 2h+1
    if (bits & 0x0000ffffu) m |= 1u << (2 * h);
    if (bits & 0xffff0000u) m |= 1u << (2 * h + 1);
  }
  m &= (1u << n_kt) - 1u;
  return m != 0 ? m : ((1u << n_kt) - 1u);
}

// Work distribution of a launch. Without a counter every CTA takes every gridDim.x-th
// item. With one, CTAs take items one at a time from a shared atomic counter (reset to zero
// by the last CTA to finish); with row_order / groups (packed rows) the counter's values
// map to the live items heaviest first: rows grouped by their number of key tiles c
// (groups[c] rows each, row_order lists them by descending c), each row's items ordered
// (query tile, head). An item costs up to c pairs, so the cheap items come last.
using Schedule = ::gdc::AttentionWork;

__device__ __forceinline__ int next_tile(uint32_t mask, int kt) {
  const uint32_t rest = kt < 0 ? mask : mask & ~((2u << kt) - 1u);  // tiles after kt
  return rest ? __ffs(int(rest)) - 1 : -1;
}

// 4 * kParts + 2 warps per CTA; with kParts = 2 (10 warps) an SM sub-partition holds at
// most 3 of them, leaving 168 registers per thread.
__global__ void __launch_bounds__(kThreads, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ CUtensorMap tm_pos,
                        const __half* __restrict__ key_mask, const int32_t* __restrict__ rel_table,
                        __half* __restrict__ ctx, int B, int L, int heads, int* err, const Schedule sc) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  int16_t* s_tab = reinterpret_cast<int16_t*>(sm + kOffTab);
  float* s_add = reinterpret_cast<float*>(sm + kOffAdd);
  float* s_red = reinterpret_cast<float*>(sm + kOffRed);
  float* s_red_l = reinterpret_cast<float*>(sm + kOffRedL);
  volatile uint32_t* s_flags = reinterpret_cast<volatile uint32_t*>(sm + kOffFlags);
  volatile int32_t* s_item = reinterpret_cast<volatile int32_t*>(sm + kOffFlags + 16);
  volatile int32_t* s_ext = reinterpret_cast<volatile int32_t*>(sm + kOffFlags + 32);
  volatile int32_t* s_row = reinterpret_cast<volatile int32_t*>(sm + kOffFlags + 48);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + kOffTmemSlot);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int E = heads * 64;
  const int n_kt = (L + kTile - 1) / kTile;
  const int n_items = n_kt * heads * B;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNumBars; ++i) ptx::mbar_init(&bars[i], 1);
    ptx::mbar_init(&bars[kBarCDone], kRowWarps);
    ptx::mbar_init(&bars[kBarProbs], kRowWarps);
    ptx::mbar_init(&bars[kBarODone], kRowWarps);
    ptx::mbar_init(&bars[kBarRow], kRowThreads);
    ptx::fence_barrier_init();
  }
  for (int i = threadIdx.x; i < 1023; i += kThreads) s_tab[i] = int16_t(rel_table[i]);
  if (warp == kRowWarps) {
    ptx::tmem_alloc(tmem_slot, kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  auto window_lo = [&](int q0, int k0) {
    const int lo = s_tab[q0 - (k0 + kTile - 1) + 511];
    return lo < 512 - kWin ? lo : 512 - kWin;
  };
  // Packed rows (sc.seq_off != null): batch row b occupies qkv / ctx rows [seq_off[b],
  // seq_off[b+1]); positions at or past its extent are not computed and items whose query
  // tile starts past the extent are never handed out. The producer picks the items and
  // publishes each one (s_item) to the MMA issuer and the row warps.
  const int32_t* __restrict__ seq_off = sc.seq_off;
  auto row_base = [&](int b) -> int { return seq_off != nullptr ? seq_off[b] : b * L; };
  auto extent = [&](int b) -> int { return seq_off != nullptr ? seq_off[b + 1] - seq_off[b] : L; };
  auto next_live = [&](int item) {
    if (seq_off != nullptr) {
      while (item < n_items) {
        const Item x = decode_item(item, n_kt, heads);
        if (x.qt * kTile < extent(x.b)) break;
        item += int(gridDim.x);
      }
    }
    return item;
  };
  // counter value j -> item, or -1 past the last one
  auto map_item = [&](int j) -> int {
    if (sc.row_order == nullptr) return j < n_items ? j : -1;
    int row = 0;
    for (int c = n_kt; c >= 1; --c) {
      const int rows_c = sc.groups[c];
      const int per_row = c * heads;
      if (j < rows_c * per_row) {
        const int r = j / per_row;
        const int rem = j - r * per_row;
        const int b = sc.row_order[row + r];
        return (b * heads + rem % heads) * n_kt + rem / heads;
      }
      j -= rows_c * per_row;
      row += rows_c;
    }
    return -1;
  };

  if (warp == kRowWarps + 1) {
    // ------------------------------------------------------------ TMA producer warp
    // Picks the work items (from the launch's counter, or every gridDim.x-th) and publishes
    // each one with its key-tile mask, extent, first qkv row and additive key mask; loads each
    // pair's K / V tile (double-buffered) and PK / PQ windows, plus Q per item, as soon as
    // their buffers are free: the windows and Q once the previous pair's gathers are done
    // (kBarScored, before its exp phase), the K / V buffer once PV of the pair two back has
    // completed.
    uint8_t* sQ = sm + kOffQ;
    uint8_t* sPK = sm + kOffW;
    uint8_t* sPQ = sm + kOffW + 32768;
    if (lane == 0) {
      ptx::prefetch_tensor_map(&tm_qkv);
      ptx::prefetch_tensor_map(&tm_pos);
    }
    int cursor = int(blockIdx.x);  // static distribution: next candidate item (lane 0)
    auto fetch = [&]() -> int {
      int v = -1;
      if (lane == 0) {
        if (sc.counter == nullptr) {
          const int x = next_live(cursor);
          cursor = x + int(gridDim.x);
          v = x < n_items ? x : -1;
        } else {
          v = map_item(atomicAdd(sc.counter, 1));
        }
      }
      return __shfl_sync(0xffffffffu, v, 0);
    };
    int item = fetch(), item_idx = 0, kt = -1, np = 0, loads_issued = 0, q_issued = 0;
    uint32_t tmask = 0;
    Item it{};
    MaskChunk pre{};  // key-mask registers prefetched for the upcoming item (batch row pre_b)
    int pre_b = -1, pre_ext = 0, pre_row = 0;  // and that row's extent / first qkv row
    bool ok = true;
    while (item >= 0) {
      // pair np is the first of item `item`: publish its tile mask and load Q
      it = decode_item(item, n_kt, heads);
      if (pre_b != it.b) {
        pre = load_mask_chunk(key_mask, (long long)it.b * L, L);
        pre_b = it.b;
        pre_ext = extent(it.b);
        pre_row = row_base(it.b);
      }
      const int it_ext = pre_ext, it_row = pre_row;
      tmask = key_tile_mask(pre, n_kt);
      int nxt = -1;
      bool first = true;
      for (kt = next_tile(tmask, -1); kt >= 0; kt = next_tile(tmask, kt)) {
        if (lane == 0 && np > 0) {
          // the previous pair's gathers are done (its P rows in the window region and its C
          // rows are no longer read): windows and Q are free while its exp phase runs
          ok = ptx::mbar_wait_sleep(&bars[kBarScored], uint32_t((np - 1) & 1), err);
          // PV of pair np-2, the last reader of this K / V buffer, has completed
          if (ok && np > 1)
            ok = ptx::mbar_wait_sleep(&bars[kBarKVFree0 + (np & 1)], uint32_t(((np - 2) >> 1) & 1), err);
        }
        ok = __shfl_sync(0xffffffffu, ok, 0) != 0;
        if (!ok) break;
        if (first) {
          // the item's additive key mask, one value per key (lane l: keys 8l.. and 256 + 8l..)
          float* sa = s_add + (item_idx & 1) * 512;
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const __half* mh = reinterpret_cast<const __half*>(&pre.v[hh]);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const int k = hh * 256 + lane * 8 + j;
              sa[k] = k >= it_ext ? -INFINITY : (__half2float(mh[j]) > 0.f ? 0.f : -65504.0f);
            }
          }
          __syncwarp();
        }
        if (lane == 0) {
          if (first) {
            s_flags[item_idx & 1] = tmask;
            s_item[item_idx & 1] = item;
            s_ext[item_idx & 1] = it_ext;
            s_row[item_idx & 1] = it_row;
            ptx::mbar_arrive(&bars[kBarFlags]);  // release: mask and item are visible to the consumers
            ptx::mbar_arrive_expect_tx(&bars[kBarQ], 16384);
            ptx::tma_load_2d(sQ, &tm_qkv, it.h * 64, it_row + it.qt * kTile, &bars[kBarQ]);
          }
          const int buf = np & 1;
          const int k0 = kt * kTile;
          const int lo = window_lo(it.qt * kTile, k0);
          const int krow = it_row + k0;
          uint64_t* bar = &bars[kBarKV0 + buf];
          ptx::mbar_arrive_expect_tx(bar, 2 * 16384 + 2 * 32768);
          ptx::tma_load_2d(sm + kOffK + buf * 16384, &tm_qkv, E + it.h * 64, krow, bar);
          ptx::tma_load_2d(sm + kOffV + buf * 16384, &tm_qkv, 2 * E + it.h * 64, krow, bar);
          ptx::tma_load_2d(sPK, &tm_pos, E + it.h * 64, lo, bar);
          ptx::tma_load_2d(sPQ, &tm_pos, it.h * 64, lo, bar);
        }
        if (first) {
          ++q_issued;
          // the next item, fetched while this pair computes, and its key-mask registers
          nxt = fetch();
          if (nxt >= 0) {
            const int nb = decode_item(nxt, n_kt, heads).b;
            if (nb != pre_b) {
              pre = load_mask_chunk(key_mask, (long long)nb * L, L);  // consumed at the next item
              pre_b = nb;
              pre_ext = extent(nb);
              pre_row = row_base(nb);
            }
          }
        }
        first = false;
        ++loads_issued;
        ++np;
      }
      if (!ok) break;
      item = nxt;
      ++item_idx;
    }
    if (ok && lane == 0) {
      // End of the work list: item -1. Published only after the last pair's gathers, so
      // every consumer has already seen the previous publication (a barrier phase cannot
      // complete twice ahead of a waiter). The wait is on kBarScored, which this warp has
      // followed pair by pair: a parity wait is only exact on a barrier at most one phase
      // ahead of it, and kBarProbs, never waited here before, may still be two behind.
      if (np == 0 || ptx::mbar_wait_sleep(&bars[kBarScored], uint32_t((np - 1) & 1), err)) {
        s_flags[item_idx & 1] = 0;
        s_item[item_idx & 1] = -1;
        ptx::mbar_arrive(&bars[kBarFlags]);
      }
    }
    if (lane == 0) {
      // wait (bounded) for the last issued loads to land before the CTA can exit
      for (int j = loads_issued - 2 < 0 ? 0 : loads_issued - 2; j < loads_issued; ++j) {
        const unsigned long long t1 = ptx::globaltimer();
        while (!ptx::mbar_try_wait(&bars[kBarKV0 + (j & 1)], uint32_t((j >> 1) & 1)) &&
               ptx::globaltimer() - t1 < ptx::kTimeoutNs) {
        }
      }
      if (q_issued > 0) {
        const unsigned long long t2 = ptx::globaltimer();
        while (!ptx::mbar_try_wait(&bars[kBarQ], uint32_t((q_issued - 1) & 1)) &&
               ptx::globaltimer() - t2 < ptx::kTimeoutNs) {
        }
      }
    }
  } else if (warp == kRowWarps) {
    // ------------------------------------------------------------ MMA issuer (one thread)
    if (lane == 0) {
      const uint32_t id_s = ptx::idesc_f16_f32(128, 128);
      const uint32_t id_cp = ptx::idesc_f16_f32(128, 256);
      const uint32_t id_pv = ptx::idesc_f16_f32(128, 64, 1);
      const uint32_t aQ = ptx::smem_u32(sm + kOffQ), aPK = ptx::smem_u32(sm + kOffW);
      const uint32_t aPQ = ptx::smem_u32(sm + kOffW + 32768), aProb = ptx::smem_u32(sm + kOffC);
      int np = 0, item_idx = 0;
      bool ok = true;
      for (; ok; ++item_idx) {
        if (!ptx::mbar_wait(&bars[kBarFlags], uint32_t(item_idx & 1), err)) break;
        if (s_item[item_idx & 1] < 0) break;
        const uint32_t tmask = s_flags[item_idx & 1];
        bool first = true;
        for (int kt = next_tile(tmask, -1); kt >= 0; kt = next_tile(tmask, kt), ++np) {
          const int buf = np & 1;
          const uint32_t par = uint32_t(np & 1);
          const bool first_pair = first;
          ok = ptx::mbar_wait(&bars[kBarKV0 + buf], uint32_t((np >> 1) & 1), err);
          if (ok && first) ok = ptx::mbar_wait(&bars[kBarQ], uint32_t(item_idx & 1), err);
          first = false;
          if (!ok) break;
          ptx::tc_fence_after();
          const uint32_t aK = ptx::smem_u32(sm + kOffK + buf * 16384);
          const uint32_t aV = ptx::smem_u32(sm + kOffV + buf * 16384);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            ptx::umma_f16_ss(tbase + kColS, ptx::desc_kmajor_sw128(aQ + k * 32),
                             ptx::desc_kmajor_sw128(aK + k * 32), id_s, k > 0);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            ptx::umma_f16_ss(tbase + kColCP, ptx::desc_kmajor_sw128(aQ + k * 32),
                             ptx::desc_kmajor_sw128(aPK + k * 32), id_cp, k > 0);
          ptx::umma_commit(&bars[kBarSC]);
          if (!(ok = ptx::mbar_wait(&bars[kBarCDone], par, err))) break;
          ptx::tc_fence_after();
#pragma unroll
          for (int k = 0; k < 4; ++k)
            ptx::umma_f16_ss(tbase + kColCP, ptx::desc_kmajor_sw128(aK + k * 32),
                             ptx::desc_kmajor_sw128(aPQ + k * 32), id_cp, k > 0);
          ptx::umma_commit(&bars[kBarP]);
          // probabilities written and O rescaled to this pair's running max
          if (!(ok = ptx::mbar_wait(&bars[kBarProbs], par, err))) break;
          // the previous item's O has been read out of TMEM before this item overwrites it
          if (first_pair && item_idx > 0 &&
              !(ok = ptx::mbar_wait(&bars[kBarODone], uint32_t((item_idx - 1) & 1), err)))
            break;
          ptx::tc_fence_after();
#pragma unroll
          for (int s = 0; s < 8; ++s)
            ptx::umma_f16_ss(tbase + kColO, ptx::desc_kmajor_sw128(aProb + (s >> 2) * 16384 + (s & 3) * 32),
                             ptx::desc_mnmajor_sw128(aV + s * 2048), id_pv, (s > 0 || !first_pair) ? 1u : 0u);
          ptx::umma_commit(&bars[kBarO]);
          ptx::umma_commit(&bars[kBarKVFree0 + buf]);
        }
      }
      // drain outstanding tensor-core work before TMEM is released
      ptx::umma_commit(&bars[kBarDrain]);
      const unsigned long long t0 = ptx::globaltimer();
      while (!ptx::mbar_try_wait(&bars[kBarDrain], 0) && ptx::globaltimer() - t0 < ptx::kTimeoutNs) {
      }
    }
  } else {
    // ---------------------------------------------------------------- row threads
    const int quarter = warp & 3;
    const int part = warp >> 2;
    const int t = quarter * 32 + lane;  // TMEM lane; query row q0 + t; key row k0 + t
    const uint32_t lane_base = tbase + (uint32_t(quarter * 32) << 16);
    uint8_t* sC = sm + kOffC;
    uint8_t* sPst = sm + kOffW;
    const uint32_t c_row = uint32_t(t) * 512u;
    const uint32_t c_xor = uint32_t(t & 7) << 4;
    RowSync rs{&bars[kBarRow]};
    int np = 0;
    int item_idx = 0;
    bool ok = true;
    for (; ok; ++item_idx) {
      if (!ptx::mbar_wait_sleep(&bars[kBarFlags], uint32_t(item_idx & 1), err)) {
        ok = false;
        break;
      }
      const int item = s_item[item_idx & 1];
      if (item < 0) break;
      const uint32_t tmask = s_flags[item_idx & 1];
      const Item it = decode_item(item, n_kt, heads);
      const int q0 = it.qt * kTile;
      const int q = q0 + t;
      const long long orow0 = s_row[item_idx & 1];  // qkv / ctx row of position 0
      const int ext = s_ext[item_idx & 1];
      const float* s_add_item = s_add + (item_idx & 1) * 512;
      float m_run = -INFINITY, l_part = 0.f;
      bool first_pair = true;
      for (int kt = next_tile(tmask, -1); kt >= 0; kt = next_tile(tmask, kt), ++np) {
        const int k0 = kt * kTile;
        const int lo = window_lo(q0, k0);
        const uint32_t par = uint32_t(np & 1);
        const float* s_add_pair = s_add_item + k0;
        // ---- drain C (own query row, this part's 64 columns)
        if (!ptx::mbar_wait_sleep(&bars[kBarSC], par, err)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        drain_rows_f16(lane_base + kColCP + part * kColsPP, sC, t, part * kColsPP);
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&bars[kBarCDone]);
        // ---- drain P (own key row) over the consumed windows
        if (!ptx::mbar_wait_sleep(&bars[kBarP], par, err)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        drain_rows_f16(lane_base + kColCP + part * kColsPP, sPst, t, part * kColsPP);
        ptx::tc_fence_before();
        if (!rs.sync(err)) {
          ok = false;
          break;
        }
        // ---- scores of keys [part*kKeysPP, +kKeysPP) with the gathered relative bias
        const int16_t* tab_q = s_tab + (q - k0 + 511);  // tab_q[-kk] = i(q - (k0 + kk))
        // final scores go back into this lane's S columns (TMEM), not registers
        float part_max = -INFINITY;
#pragma unroll
        for (int c = 0; c < kKeysPP / 32; ++c) {
          uint32_t sraw[32];
          ptx::tmem_ld_32x32b_x32(lane_base + kColS + part * kKeysPP + c * 32, sraw);
          ptx::tmem_wait_ld();
#pragma unroll
          for (int u = 0; u < 32; ++u) {
            const int kk = part * kKeysPP + c * 32 + u;
            const uint32_t w2 = uint32_t(int(tab_q[-kk]) - lo) << 1;  // 2 * window column
            const __half cv = *reinterpret_cast<const __half*>(sC + c_row + (w2 ^ c_xor));
            const __half pv =
                *reinterpret_cast<const __half*>(sPst + uint32_t(kk) * 512u + (w2 ^ (uint32_t(kk & 7) << 4)));
            const float rb = __half2float(__float2half_rn(__half2float(__hadd(cv, pv)) * kInvScale16));
            const float add = s_add_pair[kk];
            const float sv = fmaf(__uint_as_float(sraw[u]), kInvSqrt192f, add == 0.f ? rb : add);
            sraw[u] = __float_as_uint(sv);
            part_max = fmaxf(part_max, sv);
          }
          ptx::tmem_st_32x32b_x32(lane_base + kColS + part * kKeysPP + c * 32, sraw);
        }
        ptx::tmem_wait_st();
        s_red[part * 128 + t] = part_max;
        // every row is past its C / P reads (probabilities overwrite the C rows, the next
        // pair's windows the P rows) and all parts' maxima are visible
        if (!rs.sync(err)) {
          ok = false;
          break;
        }
        if (threadIdx.x == 0) ptx::mbar_arrive(&bars[kBarScored]);  // the producer may load the next windows
        float m_tile = s_red[t];
#pragma unroll
        for (int pp = 1; pp < kParts; ++pp) m_tile = fmaxf(m_tile, s_red[pp * 128 + t]);
        const float m_new = fmaxf(m_run, m_tile);
        const float alpha = __expf(m_run - m_new);
        // the softmax denominator sums the fp32 exponentials (the reference's SDPA softmax is
        // fp32); the PV MMA multiplies their fp16 roundings
        float psum = 0.f;
        const float m_l2 = m_new * 1.4426950408889634f;
#pragma unroll
        for (int c = 0; c < kKeysPP / 32; ++c) {
          uint32_t sv[32];
          ptx::tmem_ld_32x32b_x32(lane_base + kColS + part * kKeysPP + c * 32, sv);
          ptx::tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint32_t pk[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int i = j * 8 + 2 * e;
              const float e0 = ex2_approx(fmaf(__uint_as_float(sv[i]), 1.4426950408889634f, -m_l2));
              const float e1 = ex2_approx(fmaf(__uint_as_float(sv[i + 1]), 1.4426950408889634f, -m_l2));
              const __half2 p2 = __floats2half2_rn(e0, e1);
              psum += e0 + e1;
              pk[e] = *reinterpret_cast<const uint32_t*>(&p2);
            }
            // K-major SW128 operand: atom kb / 64 holds keys 64*(kb/64)..+63 of row t
            const int kb = part * kKeysPP + c * 32 + j * 8;
            const uint32_t ch = uint32_t((kb & 63) >> 3);
            const uint32_t off = uint32_t(kb >> 6) * 16384u + uint32_t(t >> 3) * 1024u + uint32_t(t & 7) * 128u +
                                 ((ch ^ uint32_t(t & 7)) << 4);
            *reinterpret_cast<uint4*>(sC + off) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          }
        }
        ptx::fence_proxy_async_smem();
        // ---- O accumulates in TMEM across the item's pairs: rescale it to the new running
        // max before this pair's PV (skipped when no row of the warp changed its max)
        if (!first_pair) {
          if (!ptx::mbar_wait_sleep(&bars[kBarO], par ^ 1u, err)) {  // PV of the previous pair done
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          if (!__all_sync(0xffffffffu, alpha == 1.0f)) {
            uint32_t r[kOPP];
            tmem_ld_cols(lane_base + kColO + part * kOPP, r);
            ptx::tmem_wait_ld();
#pragma unroll
            for (int u = 0; u < kOPP; ++u) r[u] = __float_as_uint(__uint_as_float(r[u]) * alpha);
            tmem_st_cols(lane_base + kColO + part * kOPP, r);
            ptx::tmem_wait_st();
          }
        }
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&bars[kBarProbs]);
        l_part = l_part * alpha + psum;
        m_run = m_new;
        first_pair = false;
      }
      if (!ok) break;
      // ---- read this part's O columns after the item's last PV
      if (!ptx::mbar_wait_sleep(&bars[kBarO], uint32_t((np - 1) & 1), err)) {
        ok = false;
        break;
      }
      ptx::tc_fence_after();
      float o[kOPP];
      {
        uint32_t r[kOPP];
        tmem_ld_cols(lane_base + kColO + part * kOPP, r);
        ptx::tmem_wait_ld();
#pragma unroll
        for (int u = 0; u < kOPP; ++u) o[u] = __uint_as_float(r[u]);
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&bars[kBarODone]);
      // combine the parts' softmax denominators and store this part's 16 columns
      s_red_l[part * 128 + t] = l_part;
      if (!rs.sync(err)) {
        ok = false;
        break;
      }
      if (q < ext) {
        float lsum = s_red_l[t];
#pragma unroll
        for (int pp = 1; pp < kParts; ++pp) lsum += s_red_l[pp * 128 + t];
        const float inv = 1.0f / lsum;
        __half* dst = ctx + (orow0 + q) * (long long)E + it.h * 64 + part * kOPP;
#pragma unroll
        for (int c = 0; c < kOPP / 8; ++c) {
          uint4 v;
          v.x = ptx::pack_half2(o[c * 8 + 0] * inv, o[c * 8 + 1] * inv);
          v.y = ptx::pack_half2(o[c * 8 + 2] * inv, o[c * 8 + 3] * inv);
          v.z = ptx::pack_half2(o[c * 8 + 4] * inv, o[c * 8 + 5] * inv);
          v.w = ptx::pack_half2(o[c * 8 + 6] * inv, o[c * 8 + 7] * inv);
          reinterpret_cast<uint4*>(dst)[c] = v;
        }
      }
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == kRowWarps) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tbase, kTmemCols);
  }
  if (sc.counter != nullptr && threadIdx.x == 0) {
    // every fetch of this CTA has completed (its producer saw the end of the list)
    __threadfence();
    if (atomicAdd(sc.counter + 1, 1) == int(gridDim.x) - 1) {
      atomicExch(sc.counter, 0);
      atomicExch(sc.counter + 1, 0);
    }
  }
}

}  // namespace attn
}  // namespace gdc
