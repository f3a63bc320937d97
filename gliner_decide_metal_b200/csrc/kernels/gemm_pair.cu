// Pair-CTA (cta_group::2) tcgen05 GEMM: out = act(A . W^T + bias) with 256-row tiles.
//
// Same contract as gemm_tn_kernel (gemm.cu) for the encoder projections
// (DeBERTa.swift:60-92, 420-427). A single CTA issuing M=128 x N=256 MMAs needs more
// shared-memory bandwidth than an SM has (TMA writes plus MMA reads of A and B), so
// large-M GEMMs run on CTA pairs (a cluster of 2 on neighbouring SMs):
//   * each CTA TMA-loads its own 128 rows of the A tile and its own BN/2 rows of the W
//     tile into identical shared-memory offsets; completion of both CTAs' loads is
//     signalled on the leader CTA's "full" barrier (cp.async.bulk.tensor .cta_group::2);
//   * the leader issues tcgen05.mma.cta_group::2 (M=256, N=BN, K=16): each CTA's tensor
//     core produces its 128 rows x BN columns in its own TMEM, B is shared across the pair;
//   * the leader's commits arrive on both CTAs' "empty" (ring slot free) and "tmem full"
//     barriers; both CTAs' epilogues arrive on the leader's "tmem empty" barrier.
// Persistent over tiles (one tile sequence per pair), 2 TMEM accumulators so the
// epilogue of one tile overlaps the main loop of the next. All waits are bounded.
//
// Tail split: the tiles are 256 x BN; when the last wave over the CTA pairs would be at most
// half (a quarter) full, its tiles are split into two (four) 256 x BN/2 (BN/4) tiles each, so
// that wave runs narrower tiles on more pairs. The row count may come from device memory
// (packed encoder rows), so the split is decided in the kernel; every role derives the same
// tile list from (M, N, pairs).
#include <cuda.h>

#include "kernels.h"
#include "gelu.cuh"
#include "ptx.cuh"

namespace gdc {
namespace {

// A stage holds 128 K-columns as two 64-column (128-byte) swizzle atoms per operand, so the
// issuing thread waits, issues 8 MMAs and commits once per 128 columns: the per-stage
// wait / commit cost of the single issuing thread is what bounded the main loop at 64.
constexpr int kBK = 128;
constexpr int kAtomK = 64;
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + 32 * kEpiWarps;

template <int BN>
struct PairShape {
  static constexpr int kAHalf = 128 * kAtomK * 2;       // one K-atom of this CTA's 128 rows of A
  static constexpr int kBHalf = (BN / 2) * kAtomK * 2;  // one K-atom of this CTA's BN/2 rows of W
  static constexpr int kABytes = 2 * kAHalf;
  static constexpr int kBBytes = 2 * kBHalf;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = (200 * 1024) / kStageBytes;
  static constexpr int kTmemCols = (2 * BN <= 256) ? 256 : 512;
  static constexpr int kOutBytes = kEpiWarps * 2048;    // per epilogue warp: a 32 x 32 fp16 store box
  static constexpr int kBiasBytes = kEpiWarps * 256;    // per epilogue warp: its <= 128 bias columns
  static constexpr int kSmemBytes = kStages * kStageBytes + kOutBytes + kBiasBytes + 1024 + 256;
};


// One output tile: 256-row block mb, columns [n0, n0 + bn).
struct PairTile {
  int mb, n0, bn;
};

// Tile t of the launch's list: full-width tiles in M-fastest order, then (when the tail is
// split) the `sp` parts of each of the last `rem` full-width tiles.
struct PairTiles {
  int num_m, n_main, rem, sp, num_tiles, bn;
  // max_split: the widest split the tile width allows (the parts' columns per epilogue
  // warp stay whole 32-column chunks: BN / (2 sp) % 32 == 0)
  __device__ PairTiles(int M, int N, int BN, int pairs, int max_split) : bn(BN) {
    num_m = (M + 255) / 256;
    const int num_big = num_m * (N / BN);
    rem = pairs > 0 ? num_big % pairs : 0;
    sp = 1;
    if (rem > 0)
      for (int f = max_split; f >= 2; f >>= 1)
        if (f * rem <= pairs) {
          sp = f;
          break;
        }
    if (sp == 1) rem = 0;
    n_main = num_big - rem;
    num_tiles = n_main + sp * rem;
  }
  __device__ PairTile operator()(int t) const {
    if (t < n_main) return PairTile{t % num_m, (t / num_m) * bn, bn};
    const int u = t - n_main;
    const int big = n_main + u / sp;
    const int w = bn / sp;
    return PairTile{big % num_m, (big / num_m) * bn + (u % sp) * w, w};
  }
};

template <int BN, int ACT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_w,
                     const __grid_constant__ CUtensorMap tm_w_half, const __grid_constant__ CUtensorMap tm_w_quarter,
                     const __grid_constant__ CUtensorMap tm_out,
                     const __half* __restrict__ bias, int M_cap, int N, int K, int* err,
                     const int32_t* __restrict__ m_dev) {
  using S = PairShape<BN>;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // The descriptor fetches and the device row count's load are issued first, so their
  // latency overlaps the barrier / TMEM set-up below instead of following it.
  if (threadIdx.x == 0) {
    ptx::prefetch_tensor_map(&tm_a);
    ptx::prefetch_tensor_map(&tm_w);
    ptx::prefetch_tensor_map(&tm_w_half);
    ptx::prefetch_tensor_map(&tm_w_quarter);
    ptx::prefetch_tensor_map(&tm_out);
  }
  const int m_read = m_dev != nullptr ? *m_dev : M_cap;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* s_a = smem;
  uint8_t* s_b = smem + S::kStages * S::kABytes;
  uint8_t* s_out = s_b + S::kStages * S::kBBytes;  // epilogue store boxes (1024-aligned)
  uint8_t* s_bias = s_out + S::kOutBytes;          // epilogue bias columns
  uint64_t* full = reinterpret_cast<uint64_t*>(s_bias + S::kBiasBytes);
  uint64_t* empty = full + S::kStages;
  uint64_t* tfull = empty + S::kStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const uint32_t rank = ptx::cluster_ctarank();
  const bool leader = rank == 0;
  const int kblocks = (K + kBK - 1) / kBK;  // a last half block reads TMA zero fill
  const int pair = blockIdx.x >> 1;
  const int num_pairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::kStages; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      ptx::mbar_init(&tfull[a], 1);
      ptx::mbar_init(&tempty[a], 2 * kEpiWarps);
    }
    ptx::mbar_init(drain, 1);
    ptx::fence_barrier_init();
  }
  if (warp == 1) {
    ptx::tmem_alloc_pair(tmem_slot, S::kTmemCols);
    ptx::tmem_relinquish_pair();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::cluster_sync();  // both CTAs' barriers are initialised before any cross-CTA signal
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int M = min(M_cap, m_read);  // rows computed (same in both CTAs)
  // parts of BN keep the epilogue's 32-column chunks whole: BN = 256 splits in 2 or 4,
  // BN = 128 in 2, BN = 192 not at all
  const PairTiles tiles(M, N, BN, num_pairs, BN % 256 == 0 ? 4 : (BN % 128 == 0 ? 2 : 1));
  const int num_tiles = tiles.num_tiles;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += num_pairs) {
        const PairTile ti = tiles(tile);
        const CUtensorMap* tw = ti.bn == BN ? &tm_w : (ti.bn == BN / 2 ? &tm_w_half : &tm_w_quarter);
        const int w_rows = ti.bn / 2;  // rows of W this CTA loads
        const uint32_t tx = 2u * uint32_t(S::kABytes + 2 * w_rows * kAtomK * 2);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!ptx::mbar_wait(&empty[stage], phase ^ 1u, err)) {
            ok = false;
            break;
          }
          const uint32_t leader_full = ptx::mapa_shared(ptx::smem_u32(&full[stage]), 0);
          if (leader) ptx::mbar_arrive_expect_tx(&full[stage], tx);
          // one box per operand: both 64-column atoms of the K block ([atom][row][64])
          ptx::tma_load_3d_pair(s_a + stage * S::kABytes, &tm_a, 0, ti.mb * 256 + int(rank) * 128, kb * 2,
                                leader_full);
          ptx::tma_load_3d_pair(s_b + stage * S::kBBytes, tw, 0, ti.n0 + int(rank) * w_rows, kb * 2, leader_full);
          ++issued;
          if (++stage == S::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // The leader's MMAs read this CTA's ring slots; their "empty" arrivals mean the loads
      // landed and were consumed. Wait (bounded) for the last issue of each slot.
      const long long tail = issued < S::kStages ? issued : S::kStages;
      for (long long j = 0; j < tail; ++j) {
        int s = stage - 1 - int(j);
        uint32_t ph = phase;
        while (s < 0) {
          s += S::kStages;
          ph ^= 1u;
        }
        const unsigned long long t0 = ptx::globaltimer();
        while (!ptx::mbar_try_wait(&empty[s], ph) && ptx::globaltimer() - t0 < ptx::kTimeoutNs) {
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      constexpr uint32_t idesc_full = ptx::idesc_f16_f32(256, BN);
      constexpr uint32_t idesc_half = ptx::idesc_f16_f32(256, BN / 2);
      constexpr uint32_t idesc_quarter = ptx::idesc_f16_f32(256, BN / 4);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int local = 0;
      for (int tile = pair; tile < num_tiles && ok; tile += num_pairs, ++local) {
        const int acc = local & 1;
        const uint32_t aphase = (local >> 1) & 1;
        if (!ptx::mbar_wait(&tempty[acc], aphase ^ 1u, err)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t(acc * BN);
        const int tbn = tiles(tile).bn;
        const uint32_t idesc = tbn == BN ? idesc_full : (tbn == BN / 2 ? idesc_half : idesc_quarter);
        const uint32_t b_atom = uint32_t(tbn) * 64;  // the W box's second atom: tbn / 2 rows of 128 bytes
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!ptx::mbar_wait(&full[stage], phase, err)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint32_t a_addr = ptx::smem_u32(s_a + stage * S::kABytes);
          const uint32_t b_addr = ptx::smem_u32(s_b + stage * S::kBBytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint32_t off_a = uint32_t((k >> 2) * S::kAHalf + (k & 3) * 32);
            const uint32_t off_b = uint32_t(k >> 2) * b_atom + uint32_t((k & 3) * 32);
            ptx::umma_f16_ss_pair(d_tmem, ptx::desc_kmajor_sw128(a_addr + off_a),
                                  ptx::desc_kmajor_sw128(b_addr + off_b), idesc, (kb | k) != 0 ? 1u : 0u);
          }
          ptx::umma_commit_pair_mc(&empty[stage], 0x3);  // frees the slot in both CTAs
          if (++stage == S::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        ptx::umma_commit_pair_mc(&tfull[acc], 0x3);
      }
      ptx::umma_commit_pair(ptx::mapa_shared(ptx::smem_u32(drain), 0));
      const unsigned long long t0 = ptx::globaltimer();
      while (!ptx::mbar_try_wait(drain, 0) && ptx::globaltimer() - t0 < ptx::kTimeoutNs) {
      }
    }
  } else {
    // Epilogue warps 2..(1 + kEpiWarps): TMEM lane quarter warp % 4, column half (warp-2)/4.
    // Each 32-row x 32-column chunk goes through this warp's 2 KB box in shared memory
    // (64-byte swizzle) and out with one TMA tensor store: full-line global writes instead
    // of 16-byte stores to 32 different rows. The warp's bias columns of a tile are copied
    // to shared memory before it waits for the accumulator, so their load latency hides
    // behind the tile's main loop.
    const int quarter = warp & 3;
    const int col_half = (warp - 2) >> 2;
    uint8_t* box = s_out + (warp - 2) * 2048;
    uint4* wbias = reinterpret_cast<uint4*>(s_bias + (warp - 2) * 256);
    uint8_t* box_row = box + lane * 64;
    const uint32_t box_swz = uint32_t((lane >> 1) & 3);
    int local = 0;
    for (int tile = pair; tile < num_tiles; tile += num_pairs, ++local) {
      const int acc = local & 1;
      const uint32_t aphase = (local >> 1) & 1;
      const PairTile ti = tiles(tile);
      const int half_cols = ti.bn / 2;  // columns of this warp's half of the tile
      __syncwarp();                     // every lane is done reading the previous tile's bias
      if (lane < half_cols / 8)
        wbias[lane] = __ldg(reinterpret_cast<const uint4*>(bias + ti.n0 + col_half * half_cols) + lane);
      __syncwarp();
      if (!ptx::mbar_wait(&tfull[acc], aphase, err)) break;
      ptx::tc_fence_after();
      const int row0 = ti.mb * 256 + int(rank) * 128 + quarter * 32;
      const uint32_t t_row = tmem_base + (uint32_t(quarter * 32) << 16) + uint32_t(acc * BN);
#pragma unroll 1
      for (int c = 0; c < half_cols; c += 32) {
        const int col = col_half * half_cols + c;
        uint32_t r[32];
        ptx::tmem_ld_32x32b_x32(t_row + uint32_t(col), r);
        ptx::tmem_wait_ld();
        const int n0 = ti.n0 + col;
        uint32_t packed[16];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 bv = wbias[(c >> 3) + q];
          const __half2* bh = reinterpret_cast<const __half2*>(&bv);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float2 v = __fadd2_rn(make_float2(__uint_as_float(r[q * 8 + 2 * j]), __uint_as_float(r[q * 8 + 2 * j + 1])),
                                  __half22float2(bh[j]));
            if (ACT == kActGelu) {
              v = gelu_erf2(v);
            } else if (ACT == kActRelu) {
              v = make_float2(fmaxf(v.x, 0.f), fmaxf(v.y, 0.f));
            }
            packed[q * 4 + j] = ptx::pack_half2(v.x, v.y);
          }
        }
        // the previous chunk's store has finished reading the box
        if (lane == 0) ptx::bulk_wait_group_read0();
        __syncwarp();
#pragma unroll
        for (int q = 0; q < 4; ++q)
          *reinterpret_cast<uint4*>(box_row + ((uint32_t(q) ^ box_swz) << 4)) =
              make_uint4(packed[q * 4], packed[q * 4 + 1], packed[q * 4 + 2], packed[q * 4 + 3]);
        ptx::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          ptx::tma_store_2d(&tm_out, n0, row0, box);
          ptx::bulk_commit_group();
        }
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive_cluster(ptx::mapa_shared(ptx::smem_u32(&tempty[acc]), 0));
    }
    // the stores have read this warp's box before the CTA exits (the grid's completion covers
    // their global writes)
    if (lane == 0) ptx::bulk_wait_group_read0();
  }

  ptx::tc_fence_before();
  __syncthreads();
  ptx::cluster_sync();  // neither CTA leaves while the pair may still touch its memory
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc_pair(tmem_base, S::kTmemCols);
  }
}

template <int BN, int ACT>
gdc_status launch_pair_variant(const CUtensorMap& ta, const CUtensorMap& tw, const CUtensorMap& twh,
                               const CUtensorMap& twq, const CUtensorMap& to, const __half* bias, int M, int N, int K,
                               cudaStream_t stream, int* err, const int32_t* m_dev) {
  using S = PairShape<BN>;
  auto kern = gemm_pair_kernel<BN, ACT>;
  static PerDeviceOnce configured;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return set_error(GDC_ERR_CUDA, "device ordinal out of range");
  const cudaError_t ce = cudaError_t(per_device_once(configured, dev, [&] {
    return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kSmemBytes);
  }));
  if (ce != cudaSuccess) return set_error(GDC_ERR_CUDA, "pair gemm smem attribute: %s", cudaGetErrorString(ce));
  const int num_tiles = ((M + 255) / 256) * (N / BN);
  const int pairs_avail = device_sm_count(dev) / 2;
  const int pairs = num_tiles < pairs_avail ? num_tiles : pairs_avail;
  kern<<<2 * pairs, kThreads, S::kSmemBytes, stream>>>(ta, tw, twh, twq, to, bias, M, N, K, err, m_dev);
  return check_launch("gemm_pair_kernel");
}

// Tile width giving the best last-wave occupancy over the available CTA pairs.
int choose_bn(int64_t M, int N, int pairs) {
  const int cands[3] = {256, 192, 128};
  int best = 0;
  double best_eff = -1.0;
  for (int bn : cands) {
    if (N % bn) continue;
    const double tiles = double((M + 255) / 256) * (N / bn);
    const double waves = double(int64_t((tiles + pairs - 1) / pairs));
    const double eff = tiles / (waves * pairs) * (bn == 128 ? 0.9 : 1.0);  // narrow tiles cost more per FLOP
    if (eff > best_eff + 1e-9) {
      best_eff = eff;
      best = bn;
    }
  }
  return best;
}

}  // namespace

gdc_status launch_linear_pair(const __half* a, int64_t lda, const __half* w, const __half* bias, __half* out,
                              int64_t ldo, int64_t M, int N, int K, int act, cudaStream_t stream, int* err,
                              const int32_t* m_dev) {
  int dev = 0;
  cudaGetDevice(&dev);
  // With a device row count the kernel splits a sparse last wave itself; full-width 256
  // tiles are then the best start wherever N allows them.
  const int bn = (m_dev != nullptr && N % 256 == 0) ? 256 : choose_bn(M, N, device_sm_count(dev) / 2);
  if (bn == 0) return set_error(GDC_ERR_UNSUPPORTED, "linear: N=%d is not a multiple of 128", N);
  CUtensorMap ta, tw, twh, twq, to;
  GDC_TRY(make_tmap_katoms(&ta, a, uint64_t(M), uint64_t(K), uint64_t(lda), 128, 2));
  GDC_TRY(make_tmap_katoms(&tw, w, uint64_t(N), uint64_t(K), uint64_t(K), uint32_t(bn / 2), 2));
  GDC_TRY(make_tmap_katoms(&twh, w, uint64_t(N), uint64_t(K), uint64_t(K), uint32_t(bn / 4), 2));
  GDC_TRY(make_tmap_katoms(&twq, w, uint64_t(N), uint64_t(K), uint64_t(K), uint32_t(bn / 8 > 0 ? bn / 8 : 1), 2));
  GDC_TRY(make_tmap_2d_out32(&to, out, uint64_t(M), uint64_t(N), uint64_t(ldo)));
  const int m = int(M);
#define GDC_PAIR_CASE(BNV)                                                                              \
  if (bn == BNV) {                                                                                      \
    if (act == kActGelu) return launch_pair_variant<BNV, kActGelu>(ta, tw, twh, twq, to, bias, m, N, K, stream, err, m_dev); \
    if (act == kActRelu) return launch_pair_variant<BNV, kActRelu>(ta, tw, twh, twq, to, bias, m, N, K, stream, err, m_dev); \
    return launch_pair_variant<BNV, kActNone>(ta, tw, twh, twq, to, bias, m, N, K, stream, err, m_dev); \
  }
  GDC_PAIR_CASE(256)
  GDC_PAIR_CASE(192)
  GDC_PAIR_CASE(128)
#undef GDC_PAIR_CASE
  return set_error(GDC_ERR_UNSUPPORTED, "linear: no tile width for N=%d", N);
}

}  // namespace gdc
