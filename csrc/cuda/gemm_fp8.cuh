// Block-scaled fp8 (e4m3) GEMM for sm_100a: 1x128 activation scales and
// 128x128 weight-block scales, applied exactly in fp32.
//
//   C[M, N] = epilogue( sum_kb sa[m, kb] * sb[n / 128, kb] * (A_kb . B_kb^T) )
//
// The tensor cores cannot apply a per-K-block fp32 scale inside one
// accumulation, so every 128-wide K block is multiplied into a FRESH TMEM
// accumulator (tcgen05.mma kind::f8f6f4, M=128 N=256 K=32, four per block)
// and "promoted": eight warps read it back (tcgen05.ld), scale it by
// sa[row] * sb[tile] and add it to fp32 accumulators held in registers. Two
// TMEM buffers alternate, so the tensor cores multiply block kb+1 while the
// promotion warps fold block kb.
//
// CTA = 10 warps (+ EXTRA fused-collective warps):
//   warp 0 lane 0   TMA producer: 128x128-byte A and 256x128-byte B tiles,
//                   4-stage ring (48 KB per stage: at fp8 rate a 128-wide B
//                   tile would make shared-memory reads, not the MMA, the limit)
//   warp 1          TMEM allocation (512 columns); lane 0 issues the MMAs
//   warps 2..9      promotion + epilogue; warp w reads TMEM lane quarter
//                   w % 4 and column half (w - 2) / 4: 32 rows x 128 columns
//                   (one 128x128 weight-scale block), 128 fp32 accumulators
//                   per thread, read back 16 columns at a time
// The epilogue reuses the bf16 GEMM's sinks (EpiStore, EpiPeerRS): each
// promotion warp stages two 32x64 bf16 blocks per tile. TMA loads use no
// cluster multicast; every wait is bounded and sets *err on expiry.
#pragma once
#include "gemm.cuh"

namespace nexar {
namespace gemm8 {

using gemm::kWaitLimit;
constexpr int BM = 128, BN = 256, BK = 128, STAGES = 4;
constexpr int PROMO_WARPS = 8;
constexpr int THREADS = 64 + 32 * PROMO_WARPS;  // 320
constexpr int A_BYTES = BM * BK, B_BYTES = BN * BK, STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int EPI_BUF_BYTES = 32 * 64 * 2;
constexpr int EPI_BYTES = PROMO_WARPS * EPI_BUF_BYTES;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + EPI_BYTES + 1024 + 256;
constexpr int TMEM_COLS = 2 * BN;

// 10 warps sit 3-3-2-2 on the SM's four 16 K-register sub-partitions, so
// a thread gets at most 168 registers: 128 accumulators + one 16-column TMEM
// read-back, and no pre-activation output in this kernel's epilogue.
template <class Epi, class Gate = gemm::NoGate, int EXTRA = 0>
__global__ void __launch_bounds__(THREADS + 32 * EXTRA, 1)
k_gemm_fp8(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
           const __grid_constant__ CUtensorMap tmOut, const __grid_constant__ CUtensorMap tmPre,
           const float* __restrict__ sa, const float* __restrict__ sb, int M, int N, int K, int m_rotate, Epi epi,
           Gate gate, unsigned int* err) {
  using namespace sm100;
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
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], PROMO_WARPS);
    }
    s_abort = 0;
    mbar_fence_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  {
    const bool ok = gate.prologue() && epi.prologue();
    if (!ok && threadIdx.x == 0) {
      atomicExch(err, 6u);
      s_abort = 1;
    }
    __syncthreads();
  }

  gemm::TileSched sched{(M + BM - 1) / BM, (N + BN - 1) / BN, m_rotate, 1};
  const int ntiles = sched.num();
  const int kblocks = (K + BK - 1) / BK;
  constexpr uint32_t idesc = umma_idesc_e4m3_f32(BM, BN);

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < ntiles && !s_abort; t += gridDim.x) {
        int tm, tn;
        sched.coords(t, tm, tn);
        if (!gate.wait_a(tm)) {
          atomicExch(err, 5u);
          s_abort = 1;
          break;
        }
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1, kWaitLimit)) {
            atomicExch(err, 1u);
            s_abort = 1;
            break;
          }
          uint8_t* a = smem + stage * STAGE_BYTES;
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          tma_load_2d(a, &tmA, &full[stage], kb * BK, tm * BM);
          tma_load_2d(a + A_BYTES, &tmB, &full[stage], kb * BK, tn * BN);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      for (int s = 0; s < STAGES; ++s) {
        mbar_wait_bounded(&empty[stage], phase ^ 1, kWaitLimit >> 4);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      unsigned int it = 0;  // global K-block counter: TMEM buffer = it & 1
      for (int t = blockIdx.x; t < ntiles && !s_abort; t += gridDim.x) {
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int buf = it & 1;
          const uint32_t tphase = (it >> 1) & 1;
          if (!mbar_wait_bounded(&tempty[buf], tphase ^ 1, kWaitLimit)) {
            atomicExch(err, 2u);
            s_abort = 1;
            break;
          }
          if (!mbar_wait_bounded(&full[stage], phase, kWaitLimit)) {
            atomicExch(err, 3u);
            s_abort = 1;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t b = a + A_BYTES;
          const uint32_t d = tmem_base + (uint32_t)(buf * BN);
#pragma unroll
          for (int k = 0; k < BK / 32; ++k)
            umma_f8(d, umma_desc_sw128_kmajor(a + k * 32), umma_desc_sw128_kmajor(b + k * 32), idesc, k != 0 ? 1u : 0u);
          umma_commit(&empty[stage]);
          umma_commit(&tfull[buf]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (s_abort) break;
      }
    }
  } else if (warp >= 2 + PROMO_WARPS) {
    if (!s_abort) gate.copy_role(warp - 2 - PROMO_WARPS, lane);
  } else {
    const int pw = warp - 2;          // promotion warp 0..7
    const int q = warp & 3;           // TMEM lane quarter
    const int half = pw >> 2;         // column half of the 128-wide tile
    uint8_t* buf_smem = epi_smem + pw * EPI_BUF_BYTES;
    const int ksb = kblocks;          // scale row length
    unsigned int it = 0;
    bool alive = true;
    for (int t = blockIdx.x; t < ntiles && alive; t += gridDim.x) {
      int tm, tn;
      sched.coords(t, tm, tn);
      const int row0 = tm * BM + q * 32;
      const int row = row0 + lane;
      const int nblk = tn * 2 + half;  // 128x128 weight-scale block of this warp's columns
      const bool cols_live = nblk * 128 < N;
      const float* sa_row = sa + (size_t)(row < M ? row : 0) * ksb;
      const float* sb_row = sb + (size_t)(cols_live ? nblk : 0) * ksb;
      float acc[128];
#pragma unroll
      for (int i = 0; i < 128; ++i) acc[i] = 0.f;
      float sa_next = row < M ? __ldg(sa_row) : 0.f;
      float sb_next = __ldg(sb_row);
      for (int kb = 0; kb < kblocks; ++kb, ++it) {
        const float s = sa_next * sb_next;
        if (kb + 1 < kblocks) {
          sa_next = row < M ? __ldg(sa_row + kb + 1) : 0.f;
          sb_next = __ldg(sb_row + kb + 1);
        }
        const int buf = it & 1;
        const uint32_t tphase = (it >> 1) & 1;
        bool ok = true;
        if (lane == 0) ok = mbar_wait_bounded(&tfull[buf], tphase, kWaitLimit);
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok || s_abort) {
          if (lane == 0) {
            atomicExch(err, 4u);
            s_abort = 1;
          }
          alive = false;
          break;
        }
        tc_fence_after();
        const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * BN + half * 128);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          uint32_t r[16];
          tmem_ld_32x32b_x16(taddr + 16 * j, r);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i) acc[16 * j + i] = fmaf(s, __uint_as_float(r[i]), acc[16 * j + i]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[buf]);
      }
      if (!alive) break;
      // Epilogue: two 32x64 bf16 blocks per warp per tile.
      epi.begin_tile(tm, tn);
#pragma unroll
      for (int hb = 0; hb < 2; ++hb) {
        const int col0 = tn * BN + half * 128 + hb * 64;
        if (col0 >= N) break;
        float(&v)[64] = *reinterpret_cast<float(*)[64]>(&acc[hb * 64]);
        epi.math(row, col0, v, M, N, v);  // has_pre is 0 for every fp8 sink
        if (lane == 0) tma_store_wait_read<0>();
        __syncwarp();
        gemm::stage_row64(buf_smem, lane, v);
        fence_proxy_async_smem();
        __syncwarp();
        epi.store_block(&tmOut, buf_smem, row0, col0, lane);
        if (lane == 0) tma_store_commit();
      }
      epi.end_tile(tm, tn, lane);
    }
    if (lane == 0) tma_store_wait_all<0>();
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  epi.finalize();
  gate.finalize();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace gemm8
}  // namespace nexar
