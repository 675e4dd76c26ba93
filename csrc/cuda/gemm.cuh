// Persistent warp-specialised bf16 GEMM for sm_100a (tcgen05 + TMEM + TMA).
//
//   C[M, N] = epilogue( A[M, K] . B[N, K]^T )
//
// Operands are K-major (row-major [M, K] / [N, K]) by default; AMN / BMN
// select MN-major operands (A stored as row-major [K, M], B as [K, N]), which
// is how the backward pass of a linear layer reads dY^T, X^T and W without
// transposing anything: the tensor cores take the transposed layout directly.
// SPLIT > 0 splits K across CTAs; each split writes an fp32 partial tile
// (TMA store into [splits, M, N]) and a separate pass sums the splits in a
// fixed order (deterministic).
//
// CTA = 6 warps. Warp 0 lane 0 issues TMA loads of 128x64 A and 256x64 B
// tiles into a 4-stage ring of 128-byte-swizzled shared memory. Warp 1
// allocates 512 TMEM columns (two 128x256 fp32 accumulators) and its lane 0
// issues tcgen05.mma (M=128, N=256, K=16), committing completion to
// mbarriers. Warps 2-5 drain the previous tile's accumulator from TMEM
// (tcgen05.ld 32x32b.x32, one 32-lane quarter per warp) while the next tile
// is multiplied, apply the epilogue math in registers, stage 32x64 bf16
// blocks in 128-byte-swizzled shared memory (bank-conflict free) and write
// them out with TMA bulk stores (or, for the fused reduce-scatter, with
// coalesced stores into the owning peer's memory).
//
// Hooks let the fused collective kernels reuse this mainloop:
//   Sched::coords(t, tm, tn)      tile order
//   Gate::wait_a(tm)              producer waits until A rows of tm are local
//   Epi (see EpiStore)            tile sink
// TMA loads use no cluster multicast. Every mbarrier wait is bounded
// (2 s of %globaltimer); a wait that gives up sets *err, the kernel unwinds
// and TMEM is always freed.
#pragma once
#include "common.cuh"
#include "sm100.cuh"

namespace nexar {
namespace gemm {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4, THREADS = 192;
constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2, STAGE_BYTES = A_BYTES + B_BYTES;
// The tile width is a kernel parameter (any multiple of 64 up to 256). A
// 128x192 tile fixes the wave count of N = 768 GEMMs on 148 SMs but measured
// no faster there (L2 operand traffic per FLOP rises), so launches use 256.
__host__ __device__ constexpr int stages_for(int) { return 4; }
constexpr int EPI_WARPS = 4, EPI_BUF_BYTES = 32 * 64 * 2;  // one 32x64 bf16 block
constexpr int EPI_BYTES = EPI_WARPS * 2 * EPI_BUF_BYTES;   // double-buffered per warp
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + EPI_BYTES + 1024 /*align*/ + 256 /*barriers*/;
__host__ __device__ constexpr int smem_bytes_for(int tbn) {
  return stages_for(tbn) * (A_BYTES + tbn * BK * 2) + EPI_BYTES + 1024 + 256;
}
constexpr uint64_t kWaitLimit = 2000000000ull;  // ns: 2 s per wait, far above any legitimate wait

struct TileSched {
  int tiles_m, tiles_n;
  int m_rotate;  // tile rows start at this M-tile (fused kernels: local shard first)
  int splits;    // K splits; the split index varies slowest so co-resident CTAs share K ranges
  __device__ int num() const { return tiles_m * tiles_n * splits; }
  __device__ int split_of(int t) const { return t / (tiles_m * tiles_n); }
  __device__ void coords(int t, int& tm, int& tn) const {
    t %= tiles_m * tiles_n;
    // Groups of 8 M-tiles walk N together so concurrently running CTAs
    // share B tiles and A rows in L2.
    const int group = 8;
    const int per_group = group * tiles_n;
    const int g = t / per_group;
    const int first_m = g * group;
    const int gm = min(tiles_m - first_m, group);
    const int r = t % per_group;
    tm = (first_m + r % gm + m_rotate) % tiles_m;
    tn = r / gm;
  }
};

struct NoGate {
  __device__ __forceinline__ bool prologue() const { return true; }
  __device__ __forceinline__ bool wait_a(int) const { return true; }
  __device__ __forceinline__ void copy_role(int, int) const {}
  __device__ __forceinline__ void finalize() const {}
};

// GELU (tanh form) for GEMM epilogues: tanh from the hardware instruction
// tanh.approx.f32 (PTX ISA; max relative error about 2^-11, below the bf16
// rounding of the output), one MUFU op instead of a software tanh.
__device__ __forceinline__ float tanh_hw(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float gelu_tanh_f(float x) {
  const float u = 0.7978845608028654f * (x + 0.044715f * x * x * x);
  return 0.5f * x * (1.f + tanh_hw(u));
}

// Pack 64 floats of one row into the 128-byte-swizzled staging block
// (row `r` of 32, 8 chunks of 16 bytes; chunk j lands at j ^ (r & 7)).
__device__ __forceinline__ void stage_row64(uint8_t* buf, int r, const float (&v)[64]) {
  uint8_t* row = buf + r * 128;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    uint4 o;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(v[j * 8 + 2 * e], v[j * 8 + 2 * e + 1]);
    *reinterpret_cast<uint4*>(row + ((j ^ (r & 7)) << 4)) = o;
  }
}

// 32 fp32 values (columns h*32 .. h*32+31 of v) of row `r` into a 128-byte
// swizzled staging row (8 chunks of 4 floats; chunk j lands at j ^ (r & 7)).
template <int H>
__device__ __forceinline__ void stage_row32f(uint8_t* buf, int r, const float (&v)[64]) {
  uint8_t* row = buf + r * 128;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float4 o = make_float4(v[H * 32 + 4 * j], v[H * 32 + 4 * j + 1], v[H * 32 + 4 * j + 2],
                                 v[H * 32 + 4 * j + 3]);
    *reinterpret_cast<float4*>(row + ((j ^ (r & 7)) << 4)) = o;
  }
}

// Default sink: out = act(alpha * acc + bias) (+ residual), via TMA store;
// optionally the pre-activation through a second tensor map.
struct EpiStore {
  const __nv_bfloat16* bias;      // [N] or null
  const __nv_bfloat16* residual;  // [M, ldr] or null
  long long ldr;
  float alpha;
  int act;                        // 0 none, 1 gelu(tanh)
  int has_pre;

  __device__ __forceinline__ bool prologue() const { return true; }
  __device__ __forceinline__ bool begin_tile(int, int) const { return true; }
  // v: 64 accumulators of row `row`, columns col0..col0+63 (in-place math).
  // Phase 1: alpha * acc + bias (the pre-activation value).
  __device__ __forceinline__ void math_pre(int, int col0, float (&v)[64], int, int N) const {
#pragma unroll
    for (int i = 0; i < 64; ++i) v[i] *= alpha;
    if (bias) {
      const int valid = min(64, N - col0);
      if (valid == 64 && ((reinterpret_cast<uintptr_t>(bias + col0) & 15u) == 0)) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          uint4 b = *reinterpret_cast<const uint4*>(bias + col0 + j * 8);
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&b);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float2 f = __bfloat1622float2(h[e]);
            v[j * 8 + 2 * e] += f.x;
            v[j * 8 + 2 * e + 1] += f.y;
          }
        }
      } else {
#pragma unroll
        for (int i = 0; i < 64; ++i)
          if (i < valid) v[i] += __bfloat162float(bias[col0 + i]);
      }
    }
  }
  // Phase 2: activation, then + residual.
  __device__ __forceinline__ void math_post(int row, int col0, float (&v)[64], int M, int N) const {
    if (act == 1) {
#pragma unroll
      for (int i = 0; i < 64; ++i) v[i] = gelu_tanh_f(v[i]);
    }
    if (residual && row < M) {
      const __nv_bfloat16* rp = residual + (long long)row * ldr + col0;
      const int valid = min(64, N - col0);
      if (valid == 64 && ((reinterpret_cast<uintptr_t>(rp) & 15u) == 0)) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          uint4 b = *reinterpret_cast<const uint4*>(rp + j * 8);
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&b);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float2 f = __bfloat1622float2(h[e]);
            v[j * 8 + 2 * e] += f.x;
            v[j * 8 + 2 * e + 1] += f.y;
          }
        }
      } else {
#pragma unroll
        for (int i = 0; i < 64; ++i)
          if (i < valid) v[i] += __bfloat162float(rp[i]);
      }
    }
  }
  __device__ __forceinline__ void math(int row, int col0, float (&v)[64], int M, int N, float (&pre)[64]) const {
    math_pre(row, col0, v, M, N);
    if (has_pre) {
#pragma unroll
      for (int i = 0; i < 64; ++i) pre[i] = v[i];
    }
    math_post(row, col0, v, M, N);
  }
  // Called by every lane of the warp after the 32x64 block is staged and fenced.
  __device__ __forceinline__ void store_block(const CUtensorMap* out, const uint8_t* buf, int row0, int col0,
                                              int lane) const {
    if (lane == 0) sm100::tma_store_2d(out, buf, col0, row0);
  }
  __device__ __forceinline__ void end_tile(int, int, int) const {}
  __device__ __forceinline__ void finalize() const {}
};

// Split-K partial sink: alpha * acc as fp32 into [splits, M, N] (3-D tensor
// map, so rows past M are clipped per split).
struct EpiSplitF32 {
  float alpha;
  static constexpr int has_pre = 0;
  __device__ __forceinline__ bool prologue() const { return true; }
  __device__ __forceinline__ bool begin_tile(int, int) const { return true; }
  __device__ __forceinline__ void math(int, int, float (&v)[64], int, int, float (&)[64]) const {
#pragma unroll
    for (int i = 0; i < 64; ++i) v[i] *= alpha;
  }
  // Unused: the mainloop stores fp32 partials itself (EpiTraits::f32_split).
  __device__ __forceinline__ void store_block(const CUtensorMap*, const uint8_t*, int, int, int) const {}
  __device__ __forceinline__ void end_tile(int, int, int) const {}
  __device__ __forceinline__ void finalize() const {}
};

template <class Epi> struct EpiTraits { static constexpr bool f32_split = false; };
template <> struct EpiTraits<EpiSplitF32> { static constexpr bool f32_split = true; };

template <class Epi, class Gate = NoGate, int EXTRA = 0, int AMN = 0, int BMN = 0, int TBN = 256>
__global__ void __launch_bounds__(THREADS + 32 * EXTRA, 1)
k_gemm_bf16(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
            const __grid_constant__ CUtensorMap tmOut, const __grid_constant__ CUtensorMap tmPre, int M, int N,
            int K, int m_rotate, int splits, Epi epi, Gate gate, unsigned int* err) {
  using namespace sm100;
  static_assert(TBN % 64 == 0 && TBN >= 64 && TBN <= 256, "tile width");
  // Tile-width-dependent geometry (shadows the 256-wide defaults).
  constexpr int BN = TBN;
  constexpr int B_BYTES = BN * BK * 2;
  constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  constexpr int STAGES = stages_for(TBN);
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
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], EPI_WARPS);
    }
    s_abort = 0;
    mbar_fence_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Fused kernels: stage inputs / signal peers before any role starts.
  {
    const bool ok = gate.prologue() && epi.prologue();
    if (!ok && threadIdx.x == 0) {
      atomicExch(err, 6u);
      s_abort = 1;
    }
    __syncthreads();
  }

  TileSched sched{(M + BM - 1) / BM, (N + BN - 1) / BN, m_rotate, splits};
  const int ntiles = sched.num();
  const int kblocks = (K + BK - 1) / BK;
  const int kb_per_split = (kblocks + splits - 1) / splits;
  constexpr uint32_t idesc = umma_idesc_bf16_f32(BM, BN, AMN != 0, BMN != 0);

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
        const int kb0 = sched.split_of(t) * kb_per_split;
        const int kb1 = min(kblocks, kb0 + kb_per_split);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1, kWaitLimit)) {
            atomicExch(err, 1u);
            s_abort = 1;
            break;
          }
          uint8_t* a = smem + stage * STAGE_BYTES;
          uint8_t* b = a + A_BYTES;
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          if constexpr (AMN) {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j) tma_load_2d(a + j * 8192, &tmA, &full[stage], tm * BM + 64 * j, kb * BK);
          } else {
            tma_load_2d(a, &tmA, &full[stage], kb * BK, tm * BM);
          }
          if constexpr (BMN) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tma_load_2d(b + j * 8192, &tmB, &full[stage], tn * BN + 64 * j, kb * BK);
          } else {
            tma_load_2d(b, &tmB, &full[stage], kb * BK, tn * BN);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Wait (bounded) until the MMA warp consumed everything loaded, so no
      // TMA write into this CTA's shared memory is outstanding at exit.
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
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int t = blockIdx.x; t < ntiles && !s_abort; t += gridDim.x) {
        if (!mbar_wait_bounded(&tempty[acc], acc_phase ^ 1, kWaitLimit)) {
          atomicExch(err, 2u);
          s_abort = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * BN);
        const int kb0 = sched.split_of(t) * kb_per_split;
        const int kb1 = min(kblocks, kb0 + kb_per_split);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_bounded(&full[stage], phase, kWaitLimit)) {
            atomicExch(err, 3u);
            s_abort = 1;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t b = a + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // K step of 16: 32 bytes inside the swizzle atom (K-major) or
            // two 8-row groups = 2048 bytes (MN-major).
            const uint64_t da = AMN ? umma_desc_sw128_mnmajor(a + k * 2048) : umma_desc_sw128_kmajor(a + k * 32);
            const uint64_t db = BMN ? umma_desc_sw128_mnmajor(b + k * 2048) : umma_desc_sw128_kmajor(b + k * 32);
            umma_f16(d, da, db, idesc, ((kb - kb0) | k) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        umma_commit(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
    }
  } else if (warp >= 6) {
    if (!s_abort) gate.copy_role(warp - 6, lane);
  } else {
    const int ew = warp - 2;  // epilogue warp index 0..3
    const int q = warp & 3;   // TMEM lane quarter this warp may access
    uint8_t* bufs = epi_smem + ew * 2 * EPI_BUF_BYTES;
    int acc = 0;
    uint32_t acc_phase = 0;
    int nb = 0;  // staging buffer toggle
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
      int tm, tn;
      sched.coords(t, tm, tn);
      bool ok = true;
      if (lane == 0) ok = mbar_wait_bounded(&tfull[acc], acc_phase, kWaitLimit);
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok || s_abort) {
        if (lane == 0) {
          atomicExch(err, 4u);
          s_abort = 1;
        }
        break;
      }
      tc_fence_after();
      epi.begin_tile(tm, tn);
      const int row0 = tm * BM + q * 32;
      const int row = row0 + lane;
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 64) {
        if (tn * BN + c0 >= N) break;
        uint32_t r0[32], r1[32];
        tmem_ld_32x32b_x32(tbase + c0, r0);
        tmem_ld_32x32b_x32(tbase + c0 + 32, r1);
        tmem_ld_wait();
        float v[64], pre[64];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          v[i] = __uint_as_float(r0[i]);
          v[32 + i] = __uint_as_float(r1[i]);
        }
        epi.math(row, tn * BN + c0, v, M, N, pre);
        if constexpr (EpiTraits<Epi>::f32_split) {
          const int ks = sched.split_of(t);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (lane == 0) tma_store_wait_read<1>();
            __syncwarp();
            uint8_t* buf = bufs + nb * EPI_BUF_BYTES;
            if (h == 0) stage_row32f<0>(buf, lane, v);
            else stage_row32f<1>(buf, lane, v);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_3d(&tmOut, buf, tn * BN + c0 + 32 * h, row0, ks);
              tma_store_commit();
            }
            nb ^= 1;
          }
          continue;
        }
        // Wait until the store that last read this staging buffer is done.
        if (lane == 0) tma_store_wait_read<1>();
        __syncwarp();
        uint8_t* buf = bufs + nb * EPI_BUF_BYTES;
        stage_row64(buf, lane, v);
        fence_proxy_async_smem();
        __syncwarp();
        epi.store_block(&tmOut, buf, row0, tn * BN + c0, lane);
        if (epi.has_pre) {
          if (lane == 0) {
            tma_store_commit();
            tma_store_wait_read<0>();
          }
          __syncwarp();
          stage_row64(buf, lane, pre);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) tma_store_2d(&tmPre, buf, tn * BN + c0, row0);
        }
        if (lane == 0) tma_store_commit();
        nb ^= 1;
      }
      // The accumulator is in registers / staging now: release TMEM early.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      epi.end_tile(tm, tn, lane);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
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
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace gemm
}  // namespace nexar
