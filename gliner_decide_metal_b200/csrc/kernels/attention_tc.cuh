// Disentangled attention on tcgen05 tensor cores (sm_100a).
//
// Computes, per (batch b, head h), exactly the reference's default path
// (DeBERTa.swift:322-395):
//   c2p[q,k] = fp16(q . PK[i(q-k)]),  p2c[q,k] = fp16(k . PQ[i(q-k)])
//   rb[q,k]  = fp16(fp16(c2p + p2c) / fp16(sqrt 192))
//   s[q,k]   = (q . k) / sqrt(192) + (key valid ? rb : -65504)
//   ctx[q]   = softmax_k(s) . V
// with i(r) = clip(bucket(r) + 256, 0, 511).
//
// Expanded position tables. The kernel reads PQ / PK through the expanded table
// pos_exp[r + 511] = [PQ | PK][i(r)], r = q - k in [-511, 511] (1023 rows, built once per
// layer by launch_expand_positions). For a (128-query tile, 128-key tile) pair the distances
// span r in [q0-k0-127, q0-k0+127], i.e. the 256-row window starting at expanded row
// lo = q0 - k0 + 384, and in window coordinates the relative terms are pure skews:
//   C = Q . PKw^T,  c2p[t][kk] = C[t][t - kk + 127]     (own row)
//   P = K . PQw^T,  p2c[t][kk] = P[kk][t - kk + 127]    (row kk)
// for every tile pair, log-bucket region included (t, kk: row / key inside the tiles), so the
// gathers need no index table and their addresses are per-thread constants plus
// compile-time offsets.
//
// Persistent: one CTA per SM takes work items (128-query tile, h, b) one at a time (from an
// atomic counter, heaviest first, or a static split; see Schedule) and, inside an item, walks
// the 128-key tiles of the row that hold a valid key (tiles of padding only have exactly zero
// softmax weight). With packed rows (Schedule::seq_off) a batch row's positions sit at rows
// seq_off[b] + t of qkv / ctx and query tiles past its extent are never handed out.
//
// Roles (one TMA producer warp, one MMA-issuing thread, 8 row warps; row warp w owns TMEM
// lane quarter w % 4 = query rows / key rows 32*(w%4)..+32 and key part w / 4 = keys
// 64*(w/4)..+64 of every tile):
//   TMA   Q per item (double-buffered); per pair K and the PK / PQ windows once the previous
//         pair's P MMA has consumed them, V once the previous pair's PV has.
//   MMA   per pair n:  P(n) = K PQw^T after the C drain; then, looking ahead, C(n+1) =
//         Q PKw^T as soon as P(n) has been drained and the next windows landed (it runs while
//         the rows score pair n) and PV(n) once the probabilities are in TMEM, in whichever
//         order their inputs become ready; then S(n+1) = Q K^T.
//         TMEM: S cols 0-127, C / P cols 128-383, O cols 384-447, probabilities 448-511.
//   rows  drain the C columns their own rows need (the band [t0+64-64p, +96) of 255) to
//         shared memory, the P rows of their lane quarter over the columns any query row needs
//         (5 chunks of 32), score their 64 keys in registers (S from TMEM, c2p / p2c from
//         shared memory), exchange row maxima, exponentiate, write fp16 probabilities to TMEM
//         (the PV MMA's A operand) and rescale O in TMEM when a row's running max changed.
// Every wait is a bounded mbarrier wait; the row warps sleep in theirs.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>

#include "kernels.h"
#include "ptx.cuh"

namespace gdc {
namespace attn {

constexpr int kTile = 128;       // query rows per item and keys per tile
constexpr int kWin = 256;        // expanded position rows per pair window
constexpr int kExpRows = 1023;   // expanded position table rows (r + 511, r in [-511, 511])
constexpr int kParts = 2;        // row warps per TMEM lane quarter
constexpr int kRowWarps = 4 * kParts;
constexpr int kKeysPP = 128 / kParts;   // keys scored per row warp
constexpr int kOPP = 64 / kParts;       // O columns read per row warp
constexpr int kRowThreads = kRowWarps * 32;
constexpr int kThreads = kRowThreads + 64;  // + MMA issuer warp + TMA producer warp
constexpr int kTmemCols = 512;
constexpr uint32_t kColS = 0, kColCP = 128, kColO = 384, kColProb = 448;

// C band of one row warp: 32 rows x 96 columns fp16, rows 208 bytes apart (13 chunks of 16 B:
// the 16-byte drain stores of 32 rows hit distinct bank groups, the skewed 2-byte reads at
// most two ways).
constexpr int kCBCols = 96;
constexpr int kCBPitch = 208;
constexpr int kCBWarpBytes = 32 * kCBPitch;
// P band: 128 key rows x 160 columns fp16, rows 336 bytes apart (21 chunks, odd: conflict-free
// 16-byte drain stores; the reads of one row are contiguous).
constexpr int kPBCols = 160;
constexpr int kPBPitch = 336;
// Context staging at an item's end, per row warp inside the P band: 32 rows x 64 bytes, rows
// 80 bytes apart (5 chunks of 16 B: conflict-free 16-byte stores of 8 consecutive rows).
constexpr int kStagePitch = 80;
constexpr int kStageWarpBytes = 32 * kStagePitch;
static_assert(kRowWarps * kStageWarpBytes <= 128 * kPBPitch, "context staging exceeds the P band");

// shared memory map (offsets from the 1024-aligned base)
constexpr int kOffQ = 0;                                 // Q tiles, 2 x 16 KB
constexpr int kOffK = kOffQ + 2 * 16384;                 // K tile 16 KB
constexpr int kOffV = kOffK + 16384;                     // V tile 16 KB
constexpr int kOffW = kOffV + 16384;                     // PK window 32 KB, then PQ window 32 KB
constexpr int kOffCB = kOffW + 65536;                    // C bands, 8 x 6.5 KB
constexpr int kOffPB = kOffCB + kRowWarps * kCBWarpBytes;  // P band 42 KB
constexpr int kOffBits = kOffPB + 128 * kPBPitch;        // per item slot: 16 words of key-valid bits
constexpr int kOffRed = kOffBits + 2 * 64;               // cross-part max exchange, kParts x 128 f32
constexpr int kOffRedL = kOffRed + kParts * 512;         // cross-part denominator exchange
constexpr int kOffFlags = kOffRedL + kParts * 512;       // per item slot: tile mask, item, extent, row base,
                                                         // row-has-a-valid-key, query tile | head
constexpr int kOffBar = kOffFlags + 64;
enum Bar {
  kBarFlags = 0, kBarQ0, kBarQ1, kBarQFree0, kBarQFree1, kBarKW, kBarWinFree, kBarV, kBarVFree, kBarC, kBarCDone,
  kBarP, kBarPDrained, kBarS, kBarProbs, kBarO, kBarODone, kBarRow, kBarDrain, kNumBars
};
constexpr int kOffTmemSlot = kOffBar + kNumBars * 8;
constexpr int kSmemBytes = kOffTmemSlot + 16 + 1024;  // + alignment slack
static_assert(kSmemBytes <= 232448, "attention shared memory exceeds the per-block limit");

constexpr float kInvSqrt192f = 0.07216878364870322f;
constexpr float kInvScale16 = 1.0f / 13.859375f;  // 1 / fp16(sqrt(192))
constexpr float kLog2e = 1.4426950408889634f;

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

// 32 fp32 TMEM columns of this thread's lane -> fp16, four 16-byte stores at byte offsets
// dst + off(0..3) (off(u) for the u-th group of 8 columns).
template <typename Off>
__device__ __forceinline__ void drain32_f16(uint32_t taddr, uint8_t* dst, Off off) {
  uint32_t r[32];
  ptx::tmem_ld_32x32b_x32(taddr, r);
  ptx::tmem_wait_ld();
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    uint4 v;
    v.x = ptx::pack_half2(__uint_as_float(r[u * 8 + 0]), __uint_as_float(r[u * 8 + 1]));
    v.y = ptx::pack_half2(__uint_as_float(r[u * 8 + 2]), __uint_as_float(r[u * 8 + 3]));
    v.z = ptx::pack_half2(__uint_as_float(r[u * 8 + 4]), __uint_as_float(r[u * 8 + 5]));
    v.w = ptx::pack_half2(__uint_as_float(r[u * 8 + 6]), __uint_as_float(r[u * 8 + 7]));
    *reinterpret_cast<uint4*>(dst + off(u)) = v;
  }
}

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

// Valid-key byte of this lane for half h: bit j = key (256 h + 8 lane + j) has mask > 0.
__device__ __forceinline__ uint32_t mask_byte(const MaskChunk& c, int h) {
  const __half2* p = reinterpret_cast<const __half2*>(&c.v[h]);
  uint32_t b = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __half22float2(p[j]);
    b |= (f.x > 0.f ? 1u : 0u) << (2 * j);
    b |= (f.y > 0.f ? 1u : 0u) << (2 * j + 1);
  }
  return b;
}

// The 16 valid-key words of a batch row (word w: keys 32w..32w+31), returned in lanes 0-15
// (lane w holds word w). Executed by a full warp.
__device__ __forceinline__ uint32_t mask_words(const MaskChunk& c) {
  const int lane = int(ptx::lane_id());
  const uint32_t b0 = mask_byte(c, 0), b1 = mask_byte(c, 1);
  uint32_t word = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int src = 4 * (lane & 7) + i;
    const uint32_t v0 = __shfl_sync(0xffffffffu, b0, src);
    const uint32_t v1 = __shfl_sync(0xffffffffu, b1, src);
    word |= ((lane & 8) ? v1 : v0) << (8 * i);
  }
  return word;
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

// 10 warps per CTA (8 row warps, MMA, TMA); one CTA per SM.
__global__ void __launch_bounds__(kThreads, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ CUtensorMap tm_pos,
                        const __half* __restrict__ key_mask, __half* __restrict__ ctx, int B, int L, int heads,
                        int* err, const Schedule sc) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint32_t* s_bits = reinterpret_cast<uint32_t*>(sm + kOffBits);
  float* s_red = reinterpret_cast<float*>(sm + kOffRed);
  float* s_red_l = reinterpret_cast<float*>(sm + kOffRedL);
  volatile uint32_t* s_tmask = reinterpret_cast<volatile uint32_t*>(sm + kOffFlags);
  volatile int32_t* s_item = reinterpret_cast<volatile int32_t*>(sm + kOffFlags + 8);
  volatile int32_t* s_ext = reinterpret_cast<volatile int32_t*>(sm + kOffFlags + 16);
  volatile int32_t* s_row = reinterpret_cast<volatile int32_t*>(sm + kOffFlags + 24);
  volatile int32_t* s_hasv = reinterpret_cast<volatile int32_t*>(sm + kOffFlags + 32);
  volatile int32_t* s_qh = reinterpret_cast<volatile int32_t*>(sm + kOffFlags + 40);  // (query tile << 16) | head
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
    ptx::mbar_init(&bars[kBarPDrained], kRowWarps);
    ptx::mbar_init(&bars[kBarProbs], kRowWarps);
    ptx::mbar_init(&bars[kBarODone], kRowWarps);
    ptx::mbar_init(&bars[kBarRow], kRowThreads);
    ptx::fence_barrier_init();
  }
  if (warp == kRowWarps) {
    ptx::tmem_alloc(tmem_slot, kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  // Packed rows (sc.seq_off != null): batch row b occupies qkv / ctx rows [seq_off[b],
  // seq_off[b+1]); items whose query tile starts past the extent are never handed out.
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
    // Picks the work items and publishes each one (tile mask, extent, first qkv row,
    // valid-key bits) at its first pair; loads Q per item into the item's buffer once the
    // MMAs of the item two back are done with it, each pair's K and PK / PQ windows once the
    // previous pair's P MMA has completed (its last reader), and V once the previous pair's
    // PV has.
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
    int item = fetch(), ni = 0, np = 0;
    MaskChunk pre{};  // key-mask registers prefetched for the upcoming item (batch row pre_b)
    int pre_b = -1, pre_ext = 0, pre_row = 0;
    bool ok = true;
    while (item >= 0 && ok) {
      const Item it = decode_item(item, n_kt, heads);
      if (pre_b != it.b) {
        pre = load_mask_chunk(key_mask, (long long)it.b * L, L);
        pre_b = it.b;
        pre_ext = extent(it.b);
        pre_row = row_base(it.b);
      }
      const int it_ext = pre_ext, it_row = pre_row;
      const uint32_t words = mask_words(pre);
      uint32_t tm = 0;
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const uint32_t any = __ballot_sync(0xffffffffu, lane < 16 && (lane >> 2) == t && words != 0u);
        if (any) tm |= 1u << t;
      }
      tm &= (1u << n_kt) - 1u;
      const bool has_valid = tm != 0;
      const uint32_t tmask = has_valid ? tm : ((1u << n_kt) - 1u);
      int nxt = -1;
      bool first = true;
      for (int kt = next_tile(tmask, -1); kt >= 0 && ok; kt = next_tile(tmask, kt)) {
        // the previous pair's P MMA has completed: K and the windows are free
        if (lane == 0 && np > 0) ok = ptx::mbar_wait_sleep(&bars[kBarWinFree], uint32_t((np - 1) & 1), err);
        ok = __shfl_sync(0xffffffffu, ok, 0) != 0;
        if (!ok) break;
        const int slot = ni & 1;
        if (first) {
          if (lane < 16) s_bits[slot * 16 + lane] = words;
          __syncwarp();
          if (lane == 0) {
            s_tmask[slot] = tmask;
            s_item[slot] = item;
            s_ext[slot] = it_ext;
            s_row[slot] = it_row;
            s_hasv[slot] = has_valid ? 1 : 0;
            s_qh[slot] = (it.qt << 16) | it.h;  // decoded once here, not by every row thread
            ptx::mbar_arrive(&bars[kBarFlags]);  // release: the item is visible to the consumers
            // Q buffer `slot` is free once the MMAs of item ni - 2 are done with it
            if (ni >= 2) ok = ptx::mbar_wait_sleep(&bars[kBarQFree0 + slot], uint32_t(((ni - 2) >> 1) & 1), err);
            if (ok) {
              ptx::mbar_arrive_expect_tx(&bars[kBarQ0 + slot], 16384);
              ptx::tma_load_2d(sm + kOffQ + slot * 16384, &tm_qkv, it.h * 64, it_row + it.qt * kTile,
                               &bars[kBarQ0 + slot]);
            }
          }
          ok = __shfl_sync(0xffffffffu, ok, 0) != 0;
          if (!ok) break;
        }
        if (lane == 0) {
          const int k0 = kt * kTile;
          const int lo = it.qt * kTile - k0 + 384;  // expanded row of r = q0 - k0 - 127
          const int krow = it_row + k0;
          ptx::mbar_arrive_expect_tx(&bars[kBarKW], 16384 + 2 * 32768);
          ptx::tma_load_2d(sm + kOffK, &tm_qkv, E + it.h * 64, krow, &bars[kBarKW]);
          ptx::tma_load_2d(sm + kOffW, &tm_pos, E + it.h * 64, lo, &bars[kBarKW]);
          ptx::tma_load_2d(sm + kOffW + 32768, &tm_pos, it.h * 64, lo, &bars[kBarKW]);
          // V: free once the previous pair's PV has completed
          if (np > 0) ok = ptx::mbar_wait_sleep(&bars[kBarVFree], uint32_t((np - 1) & 1), err);
          if (ok) {
            ptx::mbar_arrive_expect_tx(&bars[kBarV], 16384);
            ptx::tma_load_2d(sm + kOffV, &tm_qkv, 2 * E + it.h * 64, krow, &bars[kBarV]);
          }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0) != 0;
        if (first) {
          // the next item, fetched while this pair computes, and its key-mask registers
          nxt = fetch();
          if (nxt >= 0) {
            const int nb = decode_item(nxt, n_kt, heads).b;
            if (nb != pre_b) {
              pre = load_mask_chunk(key_mask, (long long)nb * L, L);
              pre_b = nb;
              pre_ext = extent(nb);
              pre_row = row_base(nb);
            }
          }
        }
        first = false;
        ++np;
      }
      item = nxt;
      ++ni;
    }
    if (lane == 0) {
      // End of the work list: item -1, published once the last pair's P MMA has completed
      // (as every other item: the consumers have seen the previous publication).
      if (ok && (np == 0 || ptx::mbar_wait_sleep(&bars[kBarWinFree], uint32_t((np - 1) & 1), err))) {
        s_tmask[ni & 1] = 0;
        s_item[ni & 1] = -1;
        ptx::mbar_arrive(&bars[kBarFlags]);
      }
      // wait (bounded) for loads that may still be in flight before the CTA can exit
      if (np > 0) {
        const unsigned long long t1 = ptx::globaltimer();
        while (!(ptx::mbar_try_wait(&bars[kBarKW], uint32_t((np - 1) & 1)) &&
                 ptx::mbar_try_wait(&bars[kBarV], uint32_t((np - 1) & 1))) &&
               ptx::globaltimer() - t1 < ptx::kTimeoutNs) {
        }
      }
      for (int j = (ni >= 2 ? ni - 2 : 0); j < ni; ++j) {
        const unsigned long long t2 = ptx::globaltimer();
        while (!ptx::mbar_try_wait(&bars[kBarQ0 + (j & 1)], uint32_t((j >> 1) & 1)) &&
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
      const uint32_t aK = ptx::smem_u32(sm + kOffK), aV = ptx::smem_u32(sm + kOffV);
      const uint32_t aPK = ptx::smem_u32(sm + kOffW), aPQ = ptx::smem_u32(sm + kOffW + 32768);
      auto aQ = [&](int buf) { return ptx::smem_u32(sm + kOffQ + buf * 16384); };
      auto issue_c = [&](int qbuf) {
#pragma unroll
        for (int k = 0; k < 4; ++k)
          ptx::umma_f16_ss(tbase + kColCP, ptx::desc_kmajor_sw128(aQ(qbuf) + k * 32),
                           ptx::desc_kmajor_sw128(aPK + k * 32), id_cp, k > 0);
        ptx::umma_commit(&bars[kBarC]);
      };
      auto issue_s = [&](int qbuf) {
#pragma unroll
        for (int k = 0; k < 4; ++k)
          ptx::umma_f16_ss(tbase + kColS, ptx::desc_kmajor_sw128(aQ(qbuf) + k * 32),
                           ptx::desc_kmajor_sw128(aK + k * 32), id_s, k > 0);
        ptx::umma_commit(&bars[kBarS]);
      };
      bool ok = ptx::mbar_wait(&bars[kBarFlags], 0u, err);
      int ni = 0, np = 0;
      uint32_t tmask = ok ? s_tmask[0] : 0u;
      int kt = (ok && s_item[0] >= 0) ? next_tile(tmask, -1) : -1;
      if (kt >= 0) {
        // prologue: C(0) and S(0) of the first item
        ok = ptx::mbar_wait(&bars[kBarKW], 0u, err) && ptx::mbar_wait(&bars[kBarQ0], 0u, err);
        if (ok) {
          ptx::tc_fence_after();
          issue_c(0);
          issue_s(0);
        }
      }
      bool first_in_item = true;
      while (ok && kt >= 0) {
        const uint32_t par = uint32_t(np & 1);
        // P(np) = K . PQw^T once the rows have drained C(np) out of the shared columns
        if (!(ok = ptx::mbar_wait(&bars[kBarCDone], par, err))) break;
        ptx::tc_fence_after();
#pragma unroll
        for (int k = 0; k < 4; ++k)
          ptx::umma_f16_ss(tbase + kColCP, ptx::desc_kmajor_sw128(aK + k * 32),
                           ptx::desc_kmajor_sw128(aPQ + k * 32), id_cp, k > 0);
        ptx::umma_commit(&bars[kBarP]);
        ptx::umma_commit(&bars[kBarWinFree]);  // K and the windows are free once P(np) completes
        // look ahead: the next pair, possibly of the next item
        int nkt = next_tile(tmask, kt);
        bool new_item = false;
        uint32_t ntmask = tmask;
        if (nkt < 0) {
          if (!(ok = ptx::mbar_wait(&bars[kBarFlags], uint32_t((ni + 1) & 1), err))) break;
          if (s_item[(ni + 1) & 1] >= 0) {
            new_item = true;
            ntmask = s_tmask[(ni + 1) & 1];
            nkt = next_tile(ntmask, -1);
          }
        }
        const bool has_next = nkt >= 0;
        const int qbuf = new_item ? ((ni + 1) & 1) : (ni & 1);
        // C(np+1), looking ahead, as soon as P(np) has been drained and the next K / windows
        // (and Q) have landed: it runs while the rows score pair np. PV(np) once the
        // probabilities are in TMEM, O is rescaled and the previous item's O read out. The two
        // touch different TMEM columns and operands, so whichever is ready is issued first:
        // when the next loads land late, PV(np) does not queue behind C(np+1) in the tensor
        // pipe (nor its completion behind C's). Every barrier polled here is at most one phase
        // ahead of this thread, so the parity tests are exact.
        bool c_todo = has_next, pv_todo = true;
        ptx::PollLimit lim;
        while (c_todo || pv_todo) {
          if (c_todo && ptx::mbar_test_wait(&bars[kBarKW], uint32_t((np + 1) & 1)) &&
              ptx::mbar_test_wait(&bars[kBarPDrained], par) &&
              (!new_item || ptx::mbar_test_wait(&bars[kBarQ0 + qbuf], uint32_t(((ni + 1) >> 1) & 1)))) {
            ptx::tc_fence_after();
            issue_c(qbuf);
            c_todo = false;
          }
          if (pv_todo && ptx::mbar_test_wait(&bars[kBarProbs], par) && ptx::mbar_test_wait(&bars[kBarV], par) &&
              (!first_in_item || ni == 0 || ptx::mbar_test_wait(&bars[kBarODone], uint32_t((ni - 1) & 1)))) {
            ptx::tc_fence_after();
#pragma unroll
            for (int s = 0; s < 8; ++s)
              ptx::umma_f16_ts(tbase + kColO, tbase + kColProb + uint32_t(8 * s),
                               ptx::desc_mnmajor_sw128(aV + s * 2048), id_pv, (s > 0 || !first_in_item) ? 1u : 0u);
            ptx::umma_commit(&bars[kBarO]);
            ptx::umma_commit(&bars[kBarVFree]);
            pv_todo = false;
          }
          // no pause between polls: measured against 32 and 100 ns pauses, the row warps
          // sharing this SM sub-partition lost nothing to the spin and the issue came sooner
          if (!(ok = lim.ok(err))) break;
        }
        if (!ok) break;
        if (has_next) {
          // S(np+1): the rows have consumed S(np) (their probabilities are written)
          issue_s(qbuf);
          if (new_item) ptx::umma_commit(&bars[kBarQFree0 + (ni & 1)]);  // item ni's Q reads are issued
        }
        ++np;
        if (new_item) {
          ++ni;
          tmask = ntmask;
          first_in_item = true;
        } else {
          first_in_item = false;
        }
        kt = nkt;
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
    const int t0 = quarter * 32;
    const int t = t0 + lane;  // TMEM lane; query row q0 + t; key row k0 + t
    const uint32_t lane_base = tbase + (uint32_t(t0) << 16);
    uint8_t* cband = sm + kOffCB + warp * kCBWarpBytes;
    uint8_t* pband = sm + kOffPB;
    // C band of this warp: window columns [cb0, cb0 + 96); c2p(t, 64 part + j) is band column
    // lane - j + 63 of this lane's row
    const int cb0 = t0 + 64 - 64 * part;
    const uint8_t* c2p_base = cband + lane * kCBPitch + 2 * (lane + 63);
    // P band row kk holds window columns [96 - 32 (kk / 32), +160); p2c(t, kk) is its column
    // t + 31 - kk % 32
    const uint8_t* p2c_base = pband + 2 * (t + 31) + part * 64 * kPBPitch;
    RowSync rs{&bars[kBarRow]};
    int np = 0;
    bool ok = true;
    for (int ni = 0; ok; ++ni) {
      if (!ptx::mbar_wait_sleep(&bars[kBarFlags], uint32_t(ni & 1), err)) {
        ok = false;
        break;
      }
      const int slot = ni & 1;
      const int item = s_item[slot];
      if (item < 0) break;
      const uint32_t tmask = s_tmask[slot];
      const bool has_valid = s_hasv[slot] != 0;
      const int qh = s_qh[slot];
      const int it_qt = qh >> 16, it_h = qh & 0xffff;
      const long long orow0 = s_row[slot];  // qkv / ctx row of position 0
      const int ext = s_ext[slot];
      float m_run = -INFINITY, l_part = 0.f;
      bool first_pair = true;
      for (int kt = next_tile(tmask, -1); kt >= 0; kt = next_tile(tmask, kt), ++np) {
        const uint32_t par = uint32_t(np & 1);
        // this part's 64 keys: valid bits; a part with none is skipped (its probabilities
        // are exactly zero) unless the row has no valid key at all
        const int kw = (kt * kTile + part * kKeysPP) >> 5;
        const uint32_t vb0 = s_bits[slot * 16 + kw], vb1 = s_bits[slot * 16 + kw + 1];
        const bool live = !has_valid || (vb0 | vb1) != 0u;
        // the P rows of this lane quarter are read only by the part that owns their keys
        const int pq_part = quarter >> 1;
        const int pkw = (kt * kTile + pq_part * kKeysPP) >> 5;
        const bool p_live = !has_valid || (s_bits[slot * 16 + pkw] | s_bits[slot * 16 + pkw + 1]) != 0u;
        // ---- drain C: the band of window columns this warp's rows need
        if (!ptx::mbar_wait_sleep(&bars[kBarC], par, err)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        if (live) {
#pragma unroll
          for (int c = 0; c < 3; ++c)
            drain32_f16(lane_base + kColCP + uint32_t(cb0 + 32 * c), cband + lane * kCBPitch,
                        [&](int u) { return (4 * c + u) * 16; });
        }
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&bars[kBarCDone]);
        // ---- drain P: rows of this lane quarter, window columns [96 - t0, 256 - t0)
        if (!ptx::mbar_wait_sleep(&bars[kBarP], par, err)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        if (p_live) {
#pragma unroll
          for (int c = part; c < 5; c += kParts)
            drain32_f16(lane_base + kColCP + uint32_t(96 - t0 + 32 * c), pband + t * kPBPitch,
                        [&](int u) { return (4 * c + u) * 16; });
        }
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&bars[kBarPDrained]);
        if (!rs.sync(err)) {  // every P row is in shared memory
          ok = false;
          break;
        }
        // ---- scores of keys [64 part, +64) with the gathered relative bias, in registers
        if (!ptx::mbar_wait_sleep(&bars[kBarS], par, err)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        float s[kKeysPP];
        float part_max = -INFINITY;
        if (live) {
#pragma unroll
          for (int c = 0; c < kKeysPP / 32; ++c) {
            uint32_t sraw[32];
            ptx::tmem_ld_32x32b_x32(lane_base + kColS + uint32_t(part * kKeysPP + c * 32), sraw);
            ptx::tmem_wait_ld();
            const uint32_t vb = c == 0 ? vb0 : vb1;
#pragma unroll
            for (int u = 0; u < 32; ++u) {
              const int j = c * 32 + u;
              // c2p: own row, band column lane - j + 63; p2c: P row 64 part + j, column
              // t + 31 - (j % 32)
              const __half cv = *reinterpret_cast<const __half*>(c2p_base - 2 * j);
              const __half pv = *reinterpret_cast<const __half*>(p2c_base + j * kPBPitch - 2 * (j & 31));
              const float rb = __half2float(__float2half_rn(__half2float(__hadd(cv, pv)) * kInvScale16));
              const float sv = fmaf(__uint_as_float(sraw[u]), kInvSqrt192f, ((vb >> u) & 1u) ? rb : -65504.0f);
              s[j] = sv;
              part_max = fmaxf(part_max, sv);
            }
          }
        } else {
#pragma unroll
          for (int j = 0; j < kKeysPP; ++j) s[j] = -INFINITY;
        }
        s_red[part * 128 + t] = part_max;
        // every row is past its C / P band reads and all parts' maxima are visible
        if (!rs.sync(err)) {
          ok = false;
          break;
        }
        float m_tile = s_red[t];
#pragma unroll
        for (int pp = 1; pp < kParts; ++pp) m_tile = fmaxf(m_tile, s_red[pp * 128 + t]);
        const float m_new = fmaxf(m_run, m_tile);
        const float alpha = __expf(m_run - m_new);
        // the softmax denominator sums the fp32 exponentials (the reference's SDPA softmax is
        // fp32); the PV MMA multiplies their fp16 roundings
        float psum = 0.f;
        const float m_l2 = m_new * kLog2e;
        uint32_t pk[kKeysPP / 2];
#pragma unroll
        for (int i = 0; i < kKeysPP / 2; ++i) {
          const float e0 = ex2_approx(fmaf(s[2 * i], kLog2e, -m_l2));
          const float e1 = ex2_approx(fmaf(s[2 * i + 1], kLog2e, -m_l2));
          psum += e0 + e1;
          pk[i] = ptx::pack_half2(e0, e1);
        }
        // PV of the previous pair has completed: the probability columns are free and O holds
        // every earlier pair of this item
        if (np > 0) {
          if (!ptx::mbar_wait_sleep(&bars[kBarO], par ^ 1u, err)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
        }
        if (!first_pair && !__all_sync(0xffffffffu, alpha == 1.0f)) {
          uint32_t r[kOPP];
          ptx::tmem_ld_32x32b_x32(lane_base + kColO + uint32_t(part * kOPP), r);
          ptx::tmem_wait_ld();
#pragma unroll
          for (int u = 0; u < kOPP; ++u) r[u] = __float_as_uint(__uint_as_float(r[u]) * alpha);
          ptx::tmem_st_32x32b_x32(lane_base + kColO + uint32_t(part * kOPP), r);
        }
        ptx::tmem_st_32x32b_x32(lane_base + kColProb + uint32_t(part * (kKeysPP / 2)), pk);
        ptx::tmem_wait_st();
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
        ptx::tmem_ld_32x32b_x32(lane_base + kColO + uint32_t(part * kOPP), r);
        ptx::tmem_wait_ld();
#pragma unroll
        for (int u = 0; u < kOPP; ++u) o[u] = __uint_as_float(r[u]);
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&bars[kBarODone]);
      // combine the parts' softmax denominators and store this part's 32 columns
      s_red_l[part * 128 + t] = l_part;
      if (!rs.sync(err)) {
        ok = false;
        break;
      }
      {
        float lsum = s_red_l[t];
#pragma unroll
        for (int pp = 1; pp < kParts; ++pp) lsum += s_red_l[pp * 128 + t];
        const float inv = 1.0f / lsum;  // rows past the extent are staged but never stored
        // Stage the warp's 32 rows x 32 columns (64 bytes a row) in its slice of the P band,
        // then store whole 64-byte row segments: 16 full sectors per store instruction instead
        // of 32 half-filled ones (one row per lane). The slice is free: every row warp has
        // read the P band of this item's last pair, and the next P drain into it follows the
        // next pair's C drain of every row warp, which follows these stores.
        uint8_t* stg = pband + warp * kStageWarpBytes;
#pragma unroll
        for (int c = 0; c < kOPP / 8; ++c) {
          uint4 v;
          v.x = ptx::pack_half2(o[c * 8 + 0] * inv, o[c * 8 + 1] * inv);
          v.y = ptx::pack_half2(o[c * 8 + 2] * inv, o[c * 8 + 3] * inv);
          v.z = ptx::pack_half2(o[c * 8 + 4] * inv, o[c * 8 + 5] * inv);
          v.w = ptx::pack_half2(o[c * 8 + 6] * inv, o[c * 8 + 7] * inv);
          *reinterpret_cast<uint4*>(stg + lane * kStagePitch + 16 * c) = v;
        }
        __syncwarp();
        __half* dst0 = ctx + it_h * 64 + part * kOPP + 8 * (lane & 3);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int r = 8 * j + (lane >> 2);  // row of this warp's 32
          const int qr = it_qt * kTile + t0 + r;
          const uint4 v = *reinterpret_cast<const uint4*>(stg + r * kStagePitch + 16 * (lane & 3));
          if (qr < ext) *reinterpret_cast<uint4*>(dst0 + (orow0 + qr) * (long long)E) = v;
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

// pos_exp[x] = pos_qk[rel_table[x]] for x in [0, 1023): one row of 2E fp16 per block.
__global__ void expand_positions_kernel(const __half* __restrict__ pos_qk, const int32_t* __restrict__ rel_table,
                                        __half* __restrict__ pos_exp, int cols) {
  const int x = blockIdx.x;
  const int src = rel_table[x];
  const uint4* s = reinterpret_cast<const uint4*>(pos_qk + size_t(src) * size_t(cols));
  uint4* d = reinterpret_cast<uint4*>(pos_exp + size_t(x) * size_t(cols));
  for (int i = threadIdx.x; i < cols / 8; i += blockDim.x) d[i] = s[i];
}

}  // namespace attn
}  // namespace gdc
