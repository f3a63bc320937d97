// tcgen05 GEMM for the encoder projections: out = act(A . W^T + bias).
//
// Replaces the reference's addMM(bias, x, W^T) projections (DeBERTa.swift:60-92: the
// fused QKV projection, attention output, FFN up with GELU, FFN down) and the
// classifier's first Linear + ReLU (DeBERTa.swift:437).
//
// Design (one CTA per SM, persistent over output tiles of BM x BN):
//   warp 0      TMA producer: A tile [128 x 64] and W tile [BN x 64] per K-block into a
//               STAGES-deep ring of 128B-swizzled shared-memory buffers (full/empty mbarriers).
//   warp 1      allocates 2*BN TMEM columns; lane 0 issues tcgen05.mma (M=128, N=BN, K=16)
//               into one of two TMEM accumulators and commits to the ring's empty barriers
//               and, per tile, to the accumulator-full barrier.
//   warps 2-17  epilogue: tcgen05.ld the accumulator (warp w reads TMEM lanes
//               32*(w%4)..+32, four warps per lane quarter split the columns), add bias,
//               apply GELU / ReLU, round to fp16, store 16-byte vectors; then release the
//               accumulator so the MMA warp can start the tile after next.
// Every mbarrier wait is bounded (ptx::mbar_wait); on a timeout the kernel flags the error
// word, drains its in-flight TMA loads and MMAs, frees TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>

#include "kernels.h"
#include "gelu.cuh"
#include "ptx.cuh"

namespace gdc {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kEpiWarps = 16;                  // 4 per TMEM lane quarter, each 1/4 of the columns
constexpr int kThreads = 64 + 32 * kEpiWarps;

template <int BN>
struct GemmShape {
  static constexpr int kStages = (BN == 256) ? 4 : 6;
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = 2 * BN;
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024 /*align slack*/ + 256 /*barriers*/;
};


template <int BN, int ACT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tn_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_w,
                   const __half* __restrict__ bias, __half* __restrict__ out, int M_cap, int N, int K, long long ldo,
                   int* err, const int32_t* __restrict__ m_dev) {
  using S = GemmShape<BN>;
  const int M = m_dev != nullptr ? min(M_cap, *m_dev) : M_cap;  // rows computed
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* s_a = smem;
  uint8_t* s_b = smem + S::kStages * S::kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(s_b + S::kStages * S::kBBytes);
  uint64_t* empty = full + S::kStages;
  uint64_t* tfull = empty + S::kStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_m = (M + kBM - 1) / kBM;
  const int num_tiles = num_m * (N / BN);
  const int kblocks = K / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::kStages; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      ptx::mbar_init(&tfull[a], 1);
      ptx::mbar_init(&tempty[a], kEpiWarps);
    }
    ptx::mbar_init(drain, 1);
    ptx::fence_barrier_init();
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, S::kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      ptx::prefetch_tensor_map(&tm_a);
      ptx::prefetch_tensor_map(&tm_w);
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int mb = tile % num_m;
        const int nb = tile / num_m;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!ptx::mbar_wait(&empty[stage], phase ^ 1u, err)) {
            ok = false;
            break;
          }
          ptx::mbar_arrive_expect_tx(&full[stage], S::kStageBytes);
          ptx::tma_load_2d(s_a + stage * S::kABytes, &tm_a, kb * kBK, mb * kBM, &full[stage]);
          ptx::tma_load_2d(s_b + stage * S::kBBytes, &tm_w, kb * kBK, nb * BN, &full[stage]);
          ++issued;
          if (++stage == S::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Drain: the last issue to each ring slot must have landed before the CTA exits.
      const long long tail = issued < S::kStages ? issued : S::kStages;
      for (long long j = 0; j < tail; ++j) {
        // walk back from the most recent issue
        int s = stage - 1 - int(j);
        uint32_t ph = phase;
        while (s < 0) {
          s += S::kStages;
          ph ^= 1u;
        }
        if (!ptx::mbar_try_wait(&full[s], ph)) {
          const unsigned long long t0 = ptx::globaltimer();
          while (!ptx::mbar_try_wait(&full[s], ph) && ptx::globaltimer() - t0 < ptx::kTimeoutNs) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = ptx::idesc_f16_f32(kBM, BN);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int local = 0;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t aphase = (local >> 1) & 1;
        if (!ptx::mbar_wait(&tempty[acc], aphase ^ 1u, err)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t(acc * BN);
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
            ptx::umma_f16_ss(d_tmem, ptx::desc_kmajor_sw128(a_addr + k * 32), ptx::desc_kmajor_sw128(b_addr + k * 32),
                             idesc, (kb | k) != 0 ? 1u : 0u);
          }
          ptx::umma_commit(&empty[stage]);
          if (++stage == S::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        ptx::umma_commit(&tfull[acc]);
      }
      // Drain all issued MMAs before TMEM is released.
      ptx::umma_commit(drain);
      if (!ptx::mbar_try_wait(drain, 0)) {
        const unsigned long long t0 = ptx::globaltimer();
        while (!ptx::mbar_try_wait(drain, 0) && ptx::globaltimer() - t0 < ptx::kTimeoutNs) {
        }
      }
    }
  } else {
    // Epilogue warps 2..(2 + kEpiWarps): warp w reads TMEM lane quarter w % 4 and the
    // column group (w - 2) / 4 (BN / 4 columns, two 32-column chunks in flight per wait).
    const int quarter = warp & 3;
    const int group = (warp - 2) >> 2;
    constexpr int kGroupCols = BN / 4;
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t aphase = (local >> 1) & 1;
      if (!ptx::mbar_wait(&tfull[acc], aphase, err)) break;
      ptx::tc_fence_after();
      const int mb = tile % num_m;
      const int nb = tile / num_m;
      const int row = mb * kBM + quarter * 32 + lane;
      const uint32_t t_row = tmem_base + (uint32_t(quarter * 32) << 16) + uint32_t(acc * BN);
#pragma unroll 1
      for (int c = 0; c < kGroupCols; c += 64) {
        const int col = group * kGroupCols + c;
        uint32_t r[2][32];
        ptx::tmem_ld_32x32b_x32(t_row + uint32_t(col), r[0]);
        if (kGroupCols >= 64) ptx::tmem_ld_32x32b_x32(t_row + uint32_t(col + 32), r[1]);
        ptx::tmem_wait_ld();
#pragma unroll
        for (int half = 0; half < (kGroupCols >= 64 ? 2 : 1); ++half) {
          const int n0 = nb * BN + col + half * 32;
          const uint4* bsrc = reinterpret_cast<const uint4*>(bias + n0);
          uint32_t packed[16];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint4 bv = __ldg(bsrc + q);
            const __half2* bh = reinterpret_cast<const __half2*>(&bv);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              float2 v = __fadd2_rn(
                  make_float2(__uint_as_float(r[half][q * 8 + 2 * j]), __uint_as_float(r[half][q * 8 + 2 * j + 1])),
                  __half22float2(bh[j]));
              if (ACT == kActGelu) {
                v = gelu_erf2(v);
              } else if (ACT == kActRelu) {
                v = make_float2(fmaxf(v.x, 0.f), fmaxf(v.y, 0.f));
              }
              packed[q * 4 + j] = ptx::pack_half2(v.x, v.y);
            }
          }
          if (row < M) {
            uint4* dst = reinterpret_cast<uint4*>(out + (long long)row * ldo + n0);
#pragma unroll
            for (int q = 0; q < 4; ++q)
              dst[q] = make_uint4(packed[q * 4], packed[q * 4 + 1], packed[q * 4 + 2], packed[q * 4 + 3]);
          }
        }
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&tempty[acc]);
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, S::kTmemCols);
  }
}

// ------------------------------------------------------------------ host side

template <int BN, int ACT>
gdc_status launch_gemm_variant(const CUtensorMap& ta, const CUtensorMap& tw, const __half* bias, __half* out,
                               long long ldo, int M, int N, int K, cudaStream_t stream, int* err,
                               const int32_t* m_dev) {
  using S = GemmShape<BN>;
  auto kern = gemm_tn_kernel<BN, ACT>;
  static PerDeviceOnce configured;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return set_error(GDC_ERR_CUDA, "device ordinal out of range");
  const cudaError_t ce = cudaError_t(per_device_once(configured, dev, [&] {
    return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kSmemBytes);
  }));
  if (ce != cudaSuccess) return set_error(GDC_ERR_CUDA, "gemm smem attribute: %s", cudaGetErrorString(ce));
  const int num_tiles = ((M + kBM - 1) / kBM) * (N / BN);
  const int grid = num_tiles < device_sm_count(dev) ? num_tiles : device_sm_count(dev);
  kern<<<grid, kThreads, S::kSmemBytes, stream>>>(ta, tw, bias, out, M, N, K, ldo, err, m_dev);
  return check_launch("gemm_tn_kernel");
}

// ------------------------------------------------------------------ skinny path (M <= 128)
//
// With at most 128 rows (a batch of one short row: BASELINE config 0 has M = 32) a GEMM is
// weight streaming: every weight byte is read once and the arithmetic is small. One
// persistent CTA per 256-column tile (the kernel above) leaves most SMs idle, each of the
// few busy ones streaming megabytes alone. Here every CTA owns one narrow column tile
// (BN = 16, 32 or 64 columns) over all of K, so 64-148 CTAs stream the weights at once:
//   warp 0 lane 0  TMA: per 256-column K block, the A rows [round_up(M, 8) x 256] and the W
//                  tile [BN x 256], one box each (four 64-column atoms back to back), into a
//                  ring of up to 8 stages. A TMA box costs about the same whatever its size
//                  up to 32 KB, so few, large boxes stream the weights fastest. The MMA reads
//                  128 rows from each A atom: rows past round_up(M, 8) are whatever follows in
//                  shared memory, and the MMA rows they feed are not stored;
//   warp 1 lane 0  tcgen05.mma M=128, N=BN, K=16 (16 per K block) into one TMEM accumulator;
//   warps 0-3      epilogue: TMEM lane quarter w, rows 32w..32w+31 below M: bias, GELU / ReLU,
//                  fp16, 16-byte stores.
// Each output element is one accumulation chain over K in order, as in the kernels above.
constexpr int kSkBK = 256;
constexpr int kSkAtoms = kSkBK / 64;
constexpr int kSkThreads = 128;
constexpr int kSkMaxStages = 8;
constexpr int kSkRingBytes = 200 * 1024;
constexpr int kSkSmemBytes = kSkRingBytes + 1024 + 256;

// Ring layout for `box_rows` rows of A (a multiple of 8): per stage the A atoms box_rows x
// 128 bytes apart, then room for the last atom's 128-row MMA read, then the W atoms.
struct SkinnyRing {
  int a_atom, a_bytes, stage_bytes, stages;
};
inline SkinnyRing skinny_ring(int box_rows, int bn) {
  SkinnyRing r;
  r.a_atom = box_rows * 128;
  r.a_bytes = (kSkAtoms - 1) * r.a_atom + 128 * 128;
  r.stage_bytes = r.a_bytes + kSkAtoms * bn * 128;
  r.stages = kSkRingBytes / r.stage_bytes;
  if (r.stages > kSkMaxStages) r.stages = kSkMaxStages;
  return r;
}

template <int BN>
struct SkinnyShape {
  static constexpr int kBAtom = BN * 64 * 2;
  static constexpr int kTmemCols = BN < 32 ? 32 : BN;
};

template <int BN, int ACT>
__global__ void __launch_bounds__(kSkThreads, 1)
    gemm_skinny_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_w,
                       const __half* __restrict__ bias, __half* __restrict__ out, int M_cap, int K, long long ldo,
                       SkinnyRing ring, int* err, const int32_t* __restrict__ m_dev) {
  using S = SkinnyShape<BN>;
  if (threadIdx.x == 0) {
    ptx::prefetch_tensor_map(&tm_a);
    ptx::prefetch_tensor_map(&tm_w);
  }
  const int M = m_dev != nullptr ? min(M_cap, *m_dev) : M_cap;  // rows stored
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int stages = ring.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kSkRingBytes);
  uint64_t* empty = full + kSkMaxStages;
  uint64_t* done = empty + kSkMaxStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BN;
  const int kblocks = (K + kSkBK - 1) / kSkBK;  // a last half block reads TMA zero fill

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
    }
    ptx::mbar_init(done, 1);
    ptx::fence_barrier_init();
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, S::kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  auto stage_a = [&](int s) { return smem + s * ring.stage_bytes; };
  auto stage_b = [&](int s) { return smem + s * ring.stage_bytes + ring.a_bytes; };

  bool ok = true;
  if (warp == 0 && lane == 0) {
    const uint32_t tx = uint32_t(kSkAtoms) * uint32_t(ring.a_atom + S::kBAtom);
    int issued = 0;
    for (int kb = 0; kb < kblocks && ok; ++kb) {
      const int s = kb % stages;
      if (!(ok = ptx::mbar_wait(&empty[s], uint32_t(((kb / stages) & 1) ^ 1), err))) break;
      ptx::mbar_arrive_expect_tx(&full[s], tx);
      ptx::tma_load_3d(stage_a(s), &tm_a, 0, 0, kb * kSkAtoms, &full[s]);
      ptx::tma_load_3d(stage_b(s), &tm_w, 0, n0, kb * kSkAtoms, &full[s]);
      ++issued;
    }
    // loads still in flight land before the CTA can exit (bounded)
    for (int j = issued - stages < 0 ? 0 : issued - stages; j < issued; ++j) {
      const unsigned long long t0 = ptx::globaltimer();
      while (!ptx::mbar_try_wait(&full[j % stages], uint32_t((j / stages) & 1)) &&
             ptx::globaltimer() - t0 < ptx::kTimeoutNs) {
      }
    }
  } else if (warp == 1 && lane == 0) {
    constexpr uint32_t idesc = ptx::idesc_f16_f32(128, BN);
    for (int kb = 0; kb < kblocks; ++kb) {
      const int s = kb % stages;
      if (!(ok = ptx::mbar_wait(&full[s], uint32_t((kb / stages) & 1), err))) break;
      ptx::tc_fence_after();
      const uint32_t a_addr = ptx::smem_u32(stage_a(s)), b_addr = ptx::smem_u32(stage_b(s));
#pragma unroll
      for (int k = 0; k < kSkBK / 16; ++k)
        ptx::umma_f16_ss(tmem_base,
                         ptx::desc_kmajor_sw128(a_addr + uint32_t(k >> 2) * uint32_t(ring.a_atom) + (k & 3) * 32),
                         ptx::desc_kmajor_sw128(b_addr + (k >> 2) * S::kBAtom + (k & 3) * 32), idesc,
                         (kb | k) != 0 ? 1u : 0u);
      ptx::umma_commit(&empty[s]);
    }
    // `done` also drains every issued MMA before TMEM is released
    ptx::umma_commit(done);
  }
  __syncwarp();
  // ---- epilogue: rows 32 warp + lane below M
  // (warp-uniform: the TMEM load below is a warp-collective instruction)
  const bool have = __all_sync(0xffffffffu, ptx::mbar_wait_sleep(done, 0u, err));
  ptx::tc_fence_after();
  const int row = warp * 32 + lane;
  if (have) {
#pragma unroll
    for (int c0 = 0; c0 < BN; c0 += 16) {
      uint32_t r[16];
      ptx::tmem_ld_32x32b_x16(tmem_base + (uint32_t(warp * 32) << 16) + uint32_t(c0), r);
      ptx::tmem_wait_ld();
      if (row < M) {
        uint32_t packed[8];
        const uint4* bsrc = reinterpret_cast<const uint4*>(bias + n0 + c0);
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const uint4 bv = __ldg(bsrc + q);
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
        uint4* dst = reinterpret_cast<uint4*>(out + (long long)row * ldo + n0 + c0);
        dst[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
        dst[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
      }
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, S::kTmemCols);
  }
}

template <int BN, int ACT>
gdc_status launch_skinny_variant(const CUtensorMap& ta, const CUtensorMap& tw, const __half* bias, __half* out,
                                 long long ldo, int M, int N, int K, int a_box_rows, cudaStream_t stream, int* err,
                                 const int32_t* m_dev) {
  auto kern = gemm_skinny_kernel<BN, ACT>;
  static PerDeviceOnce configured;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return set_error(GDC_ERR_CUDA, "device ordinal out of range");
  const cudaError_t ce = cudaError_t(per_device_once(configured, dev, [&] {
    return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSkSmemBytes);
  }));
  if (ce != cudaSuccess) return set_error(GDC_ERR_CUDA, "skinny gemm smem attribute: %s", cudaGetErrorString(ce));
  const SkinnyRing ring = skinny_ring(a_box_rows, BN);
  kern<<<N / BN, kSkThreads, kSkSmemBytes, stream>>>(ta, tw, bias, out, M, K, ldo, ring, err, m_dev);
  return check_launch("gemm_skinny_kernel");
}

// Column tile of the skinny path: the estimated time of a launch is its waves over the SMs
// times the bytes one CTA streams (its W columns plus all of A); the narrowest tile wins ties.
int choose_skinny_bn(int64_t M, int N, int K, int sms) {
  int best = 16;
  double best_cost = 1e300;
  for (int bn : {16, 32, 64}) {
    if (N % bn) continue;
    const double tiles = double(N / bn);
    const double waves = double(int64_t((tiles + sms - 1) / sms));
    const double cost = waves * (double(bn) + double((M + 7) / 8 * 8)) * double(K);
    if (cost < best_cost * 0.999) {
      best_cost = cost;
      best = bn;
    }
  }
  return best;
}

gdc_status launch_linear_skinny(const __half* a, int64_t lda, const __half* w, const __half* bias, __half* out,
                                int64_t ldo, int64_t M, int N, int K, int act, cudaStream_t stream, int* err,
                                const int32_t* m_dev) {
  int dev = 0;
  cudaGetDevice(&dev);
  const int bn = choose_skinny_bn(M, N, K, device_sm_count(dev));
  const int box_rows = int((M + 7) / 8 * 8);
  CUtensorMap ta, tw;
  GDC_TRY(make_tmap_katoms(&ta, a, uint64_t(M), uint64_t(K), uint64_t(lda), uint32_t(box_rows), kSkAtoms));
  GDC_TRY(make_tmap_katoms(&tw, w, uint64_t(N), uint64_t(K), uint64_t(K), uint32_t(bn), kSkAtoms));
  const int m = int(M);
#define GDC_SKINNY_CASE(BNV)                                                                                      \
  if (bn == BNV) {                                                                                                \
    if (act == kActGelu)                                                                                          \
      return launch_skinny_variant<BNV, kActGelu>(ta, tw, bias, out, ldo, m, N, K, box_rows, stream, err, m_dev); \
    if (act == kActRelu)                                                                                          \
      return launch_skinny_variant<BNV, kActRelu>(ta, tw, bias, out, ldo, m, N, K, box_rows, stream, err, m_dev); \
    return launch_skinny_variant<BNV, kActNone>(ta, tw, bias, out, ldo, m, N, K, box_rows, stream, err, m_dev);   \
  }
  GDC_SKINNY_CASE(16)
  GDC_SKINNY_CASE(32)
  GDC_SKINNY_CASE(64)
#undef GDC_SKINNY_CASE
  return set_error(GDC_ERR_UNSUPPORTED, "linear: no skinny tile for N=%d", N);
}

}  // namespace

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D fp16 tensor map: `rows` x `cols` (cols contiguous), row pitch `ld` elements,
// box = box_rows x 64 columns, 128-byte swizzle, out-of-bounds rows read as zero.
gdc_status make_tmap_2d(void* map_out, const __half* base, uint64_t rows, uint64_t cols, uint64_t ld,
                        uint32_t box_rows) {
  CUtensorMap* map = static_cast<CUtensorMap*>(map_out);
  auto fn = get_encode_fn();
  if (!fn) return set_error(GDC_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * sizeof(__half)};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(GDC_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", int(r));
  return GDC_OK;
}

gdc_status make_tmap_katoms(void* map_out, const __half* base, uint64_t rows, uint64_t cols, uint64_t ld,
                            uint32_t box_rows, uint32_t atoms) {
  CUtensorMap* map = static_cast<CUtensorMap*>(map_out);
  auto fn = get_encode_fn();
  if (!fn) return set_error(GDC_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  if (cols % 64 != 0) return set_error(GDC_ERR_UNSUPPORTED, "K-atom tensor map: %llu columns", (unsigned long long)cols);
  // dimension order follows the shared-memory box (columns, rows, atoms); the atom stride
  // (128 bytes) is below the row pitch, as in any tiled view whose modes are ordered by
  // their shared-memory placement
  cuuint64_t dims[3] = {64, rows, cols / 64};
  cuuint64_t strides[2] = {ld * sizeof(__half), 64 * sizeof(__half)};
  cuuint32_t box[3] = {64, box_rows, atoms};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<__half*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(GDC_ERR_CUDA, "cuTensorMapEncodeTiled (K atoms) failed (%d)", int(r));
  return GDC_OK;
}

gdc_status make_tmap_2d_out32(void* map_out, const __half* base, uint64_t rows, uint64_t cols, uint64_t ld) {
  CUtensorMap* map = static_cast<CUtensorMap*>(map_out);
  auto fn = get_encode_fn();
  if (!fn) return set_error(GDC_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * sizeof(__half)};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(GDC_ERR_CUDA, "cuTensorMapEncodeTiled (output) failed (%d)", int(r));
  return GDC_OK;
}

int device_sm_count(int device) {
  static PerDeviceOnce counts;
  if (device < 0 || device >= 64) return 148;
  return per_device_once(counts, device, [&] {
    int c = 0;
    if (cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || c <= 0) c = 148;
    return c;
  });
}

gdc_status launch_linear(const __half* a, int64_t lda, const __half* w, const __half* bias, __half* out,
                         int64_t ldo, int64_t M, int N, int K, int act, cudaStream_t stream, int* err,
                         const int32_t* m_dev) {
  if (M <= 0) return GDC_OK;
  if (N <= 0 || K <= 0 || N % 128 != 0 || K % kBK != 0)
    return set_error(GDC_ERR_UNSUPPORTED, "linear: N=%d must be a multiple of 128 and K=%d of 64", N, K);
  if (M > (int64_t(1) << 30)) return set_error(GDC_ERR_UNSUPPORTED, "linear: M too large");
  if ((lda % 8) || (ldo % 8) || (reinterpret_cast<uintptr_t>(a) & 15) || (reinterpret_cast<uintptr_t>(w) & 15) ||
      (reinterpret_cast<uintptr_t>(out) & 15) || (reinterpret_cast<uintptr_t>(bias) & 15))
    return set_error(GDC_ERR_INVALID_INPUT, "linear: pointers must be 16-byte aligned and strides multiples of 8");
  if (act < 0 || act > 2) return set_error(GDC_ERR_INVALID_INPUT, "linear: unknown activation %d", act);
  // Large M runs on CTA pairs (gemm_pair.cu), M <= 128 on the skinny kernel; GDC_GEMM_SINGLE_CTA=1
  // selects the persistent single-CTA kernel for every M (a cross-check of the implementations).
  static const bool force_single = [] {
    const char* e = std::getenv("GDC_GEMM_SINGLE_CTA");
    return e != nullptr && e[0] == '1';
  }();
  if (M > 128 && !force_single)
    return launch_linear_pair(a, lda, w, bias, out, ldo, M, N, K, act, stream, err, m_dev);
  if (!force_single) return launch_linear_skinny(a, lda, w, bias, out, ldo, M, N, K, act, stream, err, m_dev);
  const int bn = (N % 256 == 0) ? 256 : 128;
  CUtensorMap ta, tw;
  GDC_TRY(make_tmap_2d(&ta, a, uint64_t(M), uint64_t(K), uint64_t(lda), kBM));
  GDC_TRY(make_tmap_2d(&tw, w, uint64_t(N), uint64_t(K), uint64_t(K), uint32_t(bn)));
  const int m = int(M);
  if (bn == 256) {
    if (act == kActGelu) return launch_gemm_variant<256, kActGelu>(ta, tw, bias, out, ldo, m, N, K, stream, err, m_dev);
    if (act == kActRelu) return launch_gemm_variant<256, kActRelu>(ta, tw, bias, out, ldo, m, N, K, stream, err, m_dev);
    return launch_gemm_variant<256, kActNone>(ta, tw, bias, out, ldo, m, N, K, stream, err, m_dev);
  }
  if (act == kActGelu) return launch_gemm_variant<128, kActGelu>(ta, tw, bias, out, ldo, m, N, K, stream, err, m_dev);
  if (act == kActRelu) return launch_gemm_variant<128, kActRelu>(ta, tw, bias, out, ldo, m, N, K, stream, err, m_dev);
  return launch_gemm_variant<128, kActNone>(ta, tw, bias, out, ldo, m, N, K, stream, err, m_dev);
}

}  // namespace gdc
