// Persistent warp-specialised bf16 GEMM for sm_100a (tcgen05 + TMEM + TMA).
//
//   C[M, N] = epilogue( A[M, K] . B[N, K]^T )      (both operands K-major)
//
// CTA = 6 warps: warp 0 lane 0 issues TMA loads of 128x64 A and 256x64 B
// tiles into a 4-stage ring of 128-byte-swizzled shared memory; warp 1
// allocates 512 TMEM columns (two 128x256 fp32 accumulators) and its lane 0
// issues tcgen05.mma (M=128, N=256, K=16) and commits completion to
// mbarriers; warps 2-5 drain the accumulator of the previous tile from TMEM
// (tcgen05.ld 32x32b) while the next tile is being multiplied, and apply the
// epilogue policy. TMA loads use no cluster multicast. Every mbarrier wait is
// bounded; a wait that gives up sets *err and the kernel unwinds (TMEM is
// always freed).
#pragma once
#include "common.cuh"
#include "sm100.cuh"

namespace nexar {
namespace gemm {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4, THREADS = 192;
constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2, STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
constexpr uint64_t kWaitLimit = 2000000000ull;  // ns: 2 s per wait, far above any legitimate wait

struct TileSched {
  int tiles_m, tiles_n;
  __device__ int num() const { return tiles_m * tiles_n; }
  __device__ void coords(int t, int& tm, int& tn) const {
    // Groups of 8 M-tiles walk N together so concurrently running CTAs
    // share B tiles and A rows in L2.
    const int group = 8;
    const int per_group = group * tiles_n;
    const int g = t / per_group;
    const int first_m = g * group;
    const int gm = min(tiles_m - first_m, group);
    const int r = t % per_group;
    tm = first_m + r % gm;
    tn = r / gm;
  }
};

// Epilogue policy contract:
//   __device__ void apply(int row, int col0, float (&v)[32], int M, int N) const;
// called by each epilogue thread for 32 consecutive columns of one row.
template <class Epi>
__global__ void __launch_bounds__(THREADS, 1)
k_gemm_bf16(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M, int N,
            int K, Epi epi, unsigned int* err) {
  using namespace sm100;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
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
      mbar_init(&tempty[b], 4);
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

  TileSched sched{(M + BM - 1) / BM, (N + BN - 1) / BN};
  const int ntiles = sched.num();
  const int kblocks = (K + BK - 1) / BK;
  constexpr uint32_t idesc = umma_idesc_bf16_f32(BM, BN);

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < ntiles && !s_abort; t += gridDim.x) {
        int tm, tn;
        sched.coords(t, tm, tn);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1, kWaitLimit)) {
            atomicExch(err, 1u);
            s_abort = 1;
            break;
          }
          uint8_t* a = smem + stage * STAGE_BYTES;
          uint8_t* b = a + A_BYTES;
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          tma_load_2d(a, &tmA, &full[stage], kb * BK, tm * BM);
          tma_load_2d(b, &tmB, &full[stage], kb * BK, tn * BN);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Wait (bounded) until the MMA warp consumed everything we loaded, so
      // no TMA write into this CTA's shared memory is outstanding at exit.
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
        for (int kb = 0; kb < kblocks; ++kb) {
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
            umma_f16(d, umma_desc_sw128_kmajor(a + k * 32), umma_desc_sw128_kmajor(b + k * 32), idesc,
                     (kb | k) != 0 ? 1u : 0u);
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
  } else {
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    int acc = 0;
    uint32_t acc_phase = 0;
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
      const int row = tm * BM + q * 32 + lane;
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tbase + c0, r);
        tmem_ld_wait();
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
        epi.apply(row, tn * BN + c0, v, M, N);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

// ---------------------------------------------------------------- epilogues
__device__ __forceinline__ float gelu_tanh_f(float x) {
  const float u = 0.7978845608028654f * (x + 0.044715f * x * x * x);
  return 0.5f * x * (1.f + tanhf(u));
}

__device__ __forceinline__ void store_row32_bf16(__nv_bfloat16* dst, const float (&v)[32], int valid) {
  if (valid >= 32 && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      uint4 o;
      __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
      for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(v[k * 8 + 2 * e], v[k * 8 + 2 * e + 1]);
      reinterpret_cast<uint4*>(dst)[k] = o;
    }
  } else {
    for (int i = 0; i < valid; ++i) dst[i] = __float2bfloat16_rn(v[i]);
  }
}

// out = act(alpha * acc + bias) (+ residual); optionally also the
// pre-activation (for the activation's backward pass).
struct EpiStore {
  __nv_bfloat16* out;
  long long ldo;
  const __nv_bfloat16* bias;      // [N] or null
  const __nv_bfloat16* residual;  // [M, ld=ldr] or null
  long long ldr;
  __nv_bfloat16* pre;             // [M, ld=ldo] or null
  float alpha;
  int act;                        // 0 none, 1 gelu(tanh)

  __device__ __forceinline__ void apply(int row, int col0, float (&v)[32], int M, int N) const {
    if (row >= M || col0 >= N) return;
    const int valid = min(32, N - col0);
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] *= alpha;
    if (bias) {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i < valid) v[i] += __bfloat162float(bias[col0 + i]);
    }
    if (pre) store_row32_bf16(pre + (long long)row * ldo + col0, v, valid);
    if (act == 1) {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = gelu_tanh_f(v[i]);
    }
    if (residual) {
      const __nv_bfloat16* rp = residual + (long long)row * ldr + col0;
      for (int i = 0; i < valid; ++i) v[i] += __bfloat162float(rp[i]);
    }
    store_row32_bf16(out + (long long)row * ldo + col0, v, valid);
  }
};

}  // namespace gemm
}  // namespace nexar
