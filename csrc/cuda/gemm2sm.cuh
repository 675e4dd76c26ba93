// 2-SM (CTA pair) bf16 GEMM for sm_100a: tcgen05.mma.cta_group::2.
//
// A cluster of two CTAs computes one 256x256 output tile. Each CTA stages its
// own 128 rows of A and its own 128-column half of B per K step, so a CTA
// streams 32 KB of operands per 128x256x64 of MMA work instead of 48 KB in the
// 1-SM kernel (128x256 tile): the shapes of GPT-2 and of the TP/MoE blocks are
// bound by L2 operand bandwidth, which this cuts by a third.
//
//   CTA rank 0 (leader)  issues every MMA (M = 256, N = 256, K = 16): A rows
//                        0-127 and B columns 0-127 come from its shared
//                        memory, rows / columns 128-255 from the peer's at the
//                        same offsets; D rows 0-127 land in its TMEM, rows
//                        128-255 in the peer's.
//   both CTAs            warp 0 lane 0 loads A and B into the CTA's own shared
//                        memory with TMA; the bytes are counted on the
//                        leader's "full" barrier (no multicast: each load reads
//                        this GPU's memory into one CTA). Warps 2-9 drain their
//                        CTA's half of the accumulator (same epilogue sinks as
//                        the 1-SM kernel): warp w reads TMEM lane quarter w % 4
//                        and the tile's column half (w - 2) / 4, so two warps
//                        share each SM sub-partition and hide each other's
//                        TMEM-load, operand-load and TMA-store latencies (the
//                        short-K GEMMs of a transformer block are epilogue-bound
//                        with one). All arrive on the leader's "TMEM empty"
//                        barrier.
// The leader's MMA commits arrive on both CTAs' "stage empty" / "TMEM full"
// barriers (tcgen05.commit multicast). Every mbarrier wait is bounded; a wait
// that gives up sets *err and the CTA unwinds to the final cluster barrier.
#pragma once
#include <type_traits>

#include "gemm.cuh"

namespace nexar {
namespace gemm2 {

using gemm::BK;
using gemm::EPI_BUF_BYTES;
using gemm::kWaitLimit;
constexpr int TM = 256;                    // pair tile rows
constexpr int HM = 128;                    // per-CTA share of A rows
constexpr int EPI_WARPS = 8;                       // 2 per TMEM lane quarter
constexpr int STAGES = 6, THREADS = 64 + 32 * EPI_WARPS;
constexpr int EPI_BYTES = EPI_WARPS * EPI_BUF_BYTES;  // one 32x64 bf16 staging block per warp (32 KB)
constexpr int A_BYTES = HM * BK * 2;
// Pair tile width TN (256; 128 compiles and is correct but measured slower);
// each CTA stages TN / 2 columns of B.
__host__ __device__ constexpr int smem_bytes_2sm(int tn) {
  return STAGES * (A_BYTES + (tn / 2) * BK * 2) + EPI_BYTES + 1024 + 256;
}

template <class Epi, int AMN, int BMN, int TN = 256>
__global__ void __launch_bounds__(THREADS, 1)
k_gemm_bf16_2sm(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmOut, const __grid_constant__ CUtensorMap tmPre, int M, int N,
                int K, int splits, Epi epi, unsigned int* err) {
  using namespace sm100;
  static_assert(TN == 256 || TN == 128, "pair tile width");
  constexpr int HN = TN / 2;               // per-CTA share of B columns
  constexpr int B_BYTES = HN * BK * 2, STAGE_BYTES = A_BYTES + B_BYTES;
  (void)B_BYTES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* epi_smem = smem + STAGES * STAGE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(epi_smem + EPI_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  __shared__ volatile int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t crank = cluster_ctarank();
  const bool leader = crank == 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 2 * EPI_WARPS);
    }
    s_abort = 0;
    mbar_fence_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before any cross-CTA arrive or load
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  gemm::TileSched sched{(M + TM - 1) / TM, (N + TN - 1) / TN, 0, splits};
  const int ntiles = sched.num();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int kblocks = (K + BK - 1) / BK;
  const int kb_per_split = (kblocks + splits - 1) / splits;
  constexpr uint32_t idesc = umma_idesc_bf16_f32(TM, TN, AMN != 0, BMN != 0);

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int t = pair; t < ntiles && !s_abort; t += npairs) {
        int tm, tn;
        sched.coords(t, tm, tn);
        const int m0 = tm * TM + (int)crank * HM;
        const int n0 = tn * TN + (int)crank * HN;
        const int kb0 = sched.split_of(t) * kb_per_split;
        const int kb1 = min(kblocks, kb0 + kb_per_split);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1, kWaitLimit)) {
            atomicExch(err, 11u);
            s_abort = 1;
            break;
          }
          const uint32_t fbar = mapa_shared(smem_u32(&full[stage]), 0);
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * STAGE_BYTES);
          uint8_t* a = smem + stage * STAGE_BYTES;
          uint8_t* b = a + A_BYTES;
          if constexpr (AMN) {
#pragma unroll
            for (int j = 0; j < HM / 64; ++j) tma_load_2d_pair(a + j * 8192, &tmA, fbar, m0 + 64 * j, kb * BK);
          } else {
            tma_load_2d_pair(a, &tmA, fbar, kb * BK, m0);
          }
          if constexpr (BMN) {
#pragma unroll
            for (int j = 0; j < HN / 64; ++j) tma_load_2d_pair(b + j * 8192, &tmB, fbar, n0 + 64 * j, kb * BK);
          } else {
            tma_load_2d_pair(b, &tmB, fbar, kb * BK, n0);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Every stage this CTA loaded has been consumed before it leaves.
      for (int s = 0; s < STAGES; ++s) {
        mbar_wait_bounded(&empty[stage], phase ^ 1, kWaitLimit >> 4);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int t = pair; t < ntiles && !s_abort; t += npairs) {
        if (!mbar_wait_bounded(&tempty[acc], acc_phase ^ 1, kWaitLimit)) {
          atomicExch(err, 12u);
          s_abort = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * TN);
        const int kb0 = sched.split_of(t) * kb_per_split;
        const int kb1 = min(kblocks, kb0 + kb_per_split);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_bounded(&full[stage], phase, kWaitLimit)) {
            atomicExch(err, 13u);
            s_abort = 1;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t b = a + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t da = AMN ? umma_desc_sw128_mnmajor(a + k * 2048) : umma_desc_sw128_kmajor(a + k * 32);
            const uint64_t db = BMN ? umma_desc_sw128_mnmajor(b + k * 2048) : umma_desc_sw128_kmajor(b + k * 32);
            umma_f16_pair(d, da, db, idesc, ((kb - kb0) | k) != 0 ? 1u : 0u);
          }
          umma_commit_pair_mc(&empty[stage], 0x3);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (s_abort) break;
        umma_commit_pair_mc(&tfull[acc], 0x3);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
    }
  } else {
    const int ew = warp - 2;
    const int q = warp & 3;                    // TMEM lane quarter (hardware: warp % 4)
    const int c_lo = (ew >> 2) * (TN / 2);     // this warp's column half of the tile
    uint8_t* buf = epi_smem + ew * EPI_BUF_BYTES;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = pair; t < ntiles; t += npairs) {
      int tm, tn;
      sched.coords(t, tm, tn);
      bool ok = true;
      if (lane == 0) ok = mbar_wait_bounded(&tfull[acc], acc_phase, kWaitLimit);
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok || s_abort) {
        if (lane == 0) {
          atomicExch(err, 14u);
          s_abort = 1;
        }
        break;
      }
      tc_fence_after();
      epi.begin_tile(tm, tn);
      const int row0 = tm * TM + (int)crank * HM + q * 32;
      const int row = row0 + lane;
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * TN);
#pragma unroll 1
      for (int c0 = c_lo; c0 < c_lo + TN / 2; c0 += 64) {
        if (tn * TN + c0 >= N) break;
        uint32_t r0[32], r1[32];
        tmem_ld_32x32b_x32(tbase + c0, r0);
        tmem_ld_32x32b_x32(tbase + c0 + 32, r1);
        tmem_ld_wait();
        float v[64];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          v[i] = __uint_as_float(r0[i]);
          v[32 + i] = __uint_as_float(r1[i]);
        }
        if constexpr (std::is_same<Epi, gemm::EpiStore>::value) {
          // Two phases: the pre-activation block is staged and stored from v
          // itself before the activation runs (no second 64-value array).
          epi.math_pre(row, tn * TN + c0, v, M, N);
          if (epi.has_pre) {
            if (lane == 0) tma_store_wait_read<0>();
            __syncwarp();
            gemm::stage_row64(buf, lane, v);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&tmPre, buf, tn * TN + c0, row0);
              tma_store_commit();
            }
          }
          epi.math_post(row, tn * TN + c0, v, M, N);
        } else {
          float pre[64];
          epi.math(row, tn * TN + c0, v, M, N, pre);
        }
        if constexpr (gemm::EpiTraits<Epi>::f32_split) {
          const int ks = sched.split_of(t);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (lane == 0) tma_store_wait_read<0>();
            __syncwarp();
            if (h == 0) gemm::stage_row32f<0>(buf, lane, v);
            else gemm::stage_row32f<1>(buf, lane, v);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_3d(&tmOut, buf, tn * TN + c0 + 32 * h, row0, ks);
              tma_store_commit();
            }
          }
          continue;
        }
        if (lane == 0) tma_store_wait_read<0>();
        __syncwarp();
        gemm::stage_row64(buf, lane, v);
        fence_proxy_async_smem();
        __syncwarp();
        epi.store_block(&tmOut, buf, row0, tn * TN + c0, lane);
        if (lane == 0) tma_store_commit();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[acc]), 0));
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
    if (lane == 0) tma_store_wait_all<0>();
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while its peer may still touch its barriers or shared memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, 512);
  }
}

}  // namespace gemm2
}  // namespace nexar
