// GEMM fused with its collective over NVLink peer memory (sm_100a).
//
// gemm_reduce_scatter (row-parallel linear, e.g. the TP MLP down projection):
//   every rank computes a full partial C_r = A_r . B_r^T; rank o must end
//   with sum_r C_r[rows of o]. The epilogue writes each finished 128x256 tile
//   straight into the owner's symmetric staging slot (slot index = source
//   rank) with TMA stores (a tensor map per owner's slot, in device memory;
//   a plain store to a peer's memory, no multicast) and publishes a per-tile
//   flag (st.release.sys) once they have completed. Tiles are produced owner by owner starting at
//   rank+1, so at any moment the ranks write to different peers and the
//   NVLink traffic overlaps the MMAs of the following tiles. After its GEMM
//   tiles every CTA reduces the tiles this rank owns as soon as all sources
//   flagged them (fp32 sum, bias added once, bf16 out).
//
// all_gather_gemm (column-parallel linear, e.g. the TP MLP up projection):
//   rank p holds rows [p*M/W, (p+1)*M/W) of A. Every CTA first stages its
//   share of the local shard into the symmetric staging slot (for the
//   peers) and into the local gather buffer; two extra copy warps per CTA
//   then pull the peers' shards over NVLink (plain loads from the peer VA)
//   into the local gather buffer, 128-row tile by tile, nearest shard first,
//   and count completed pieces per M-tile. The TMA producer of the GEMM
//   waits on that count before loading A rows of a remote tile, and starts
//   with the local shard, so the copies of later shards overlap the MMAs of
//   earlier ones. Remote tiles cross NVLink exactly once; TMA only ever reads
//   this GPU's memory and never uses cluster multicast.
//
// Both kernels take their epochs from the communicator's device call
// counter, announce "started call e" to every peer (ready flags) so staging
// buffers are never overwritten while a peer still reads them, and bound
// every wait (the status word records the rank that never arrived).
#include "coll.cuh"
#include "coll_api.h"
#include "gemm_launch.cuh"
#include "gemm_fp8.cuh"

namespace nexar {
namespace gemm {

__device__ __forceinline__ unsigned long long* fused_ready(const CommDev& c, int owner, int src) {
  return reinterpret_cast<unsigned long long*>(c.peer_base[owner] + kFusedReadyOff) + src;
}
__device__ __forceinline__ unsigned long long* fused_tile_flag(const CommDev& c, int owner, int src, int tile) {
  return reinterpret_cast<unsigned long long*>(c.peer_base[owner] + kFusedTileOff) +
         (size_t)src * kMaxFusedTiles + tile;
}
__device__ __forceinline__ unsigned long long& s_call() {
  __shared__ unsigned long long v;
  return v;
}
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
// Bounded spin until *p >= target (system scope). Returns false on timeout.
__device__ __forceinline__ bool wait_flag_sys(const unsigned long long* p, unsigned long long target,
                                              unsigned long long timeout_ns) {
  if (ld_acquire_sys(p) >= target) return true;
  const unsigned long long t0 = globaltimer_ns();
  unsigned int spins = 0;
  while (ld_acquire_sys(p) < target) {
    if ((++spins & 255u) == 0 && globaltimer_ns() - t0 > timeout_ns) return false;
  }
  return true;
}
__device__ __forceinline__ void announce_ready(const CommDev& c, unsigned long long epoch) {
  fence_sys();
  for (int p = 0; p < c.world; ++p)
    if (p != c.rank) st_release_sys(fused_ready(c, p, c.rank), epoch);
}

// ------------------------------------------------------------ GEMM -> RS
struct EpiPeerRS {
  CommDev c;
  int rpr;        // rows per rank (multiple of BM)
  int N;
  int tiles_n;
  float alpha;
  const __nv_bfloat16* bias;  // [N], added once after the reduction
  __nv_bfloat16* out;         // [rpr, ldo] this rank's reduced rows
  long long ldo;
  int op_id;
  int arrivals;   // epilogue warps that store each tile (4 bf16 kernel, 8 fp8 kernel)
  const CUtensorMap* maps;  // [2 slots][kMaxRanks owners] in device memory
  static constexpr int has_pre = 0;

  __device__ __forceinline__ unsigned long long epoch() const { return epoch_of(s_call(), 0); }
  __device__ __forceinline__ int slot() const { return (int)(s_call() & 1ull); }

  __device__ bool prologue() const {
    if (!entry_ok(c, op_id)) return false;  // uniform: every thread checks the same arguments
    if (threadIdx.x == 0) {
      s_call() = call_index(c);
      s_tile_arrivals() = 0u;
      s_tile_seq() = 0u;
      if (blockIdx.x == 0) announce_ready(c, epoch_of(s_call(), 0));
    }
    __syncthreads();
    return true;
  }
  __device__ bool begin_tile(int tm, int) const {
    const int owner = tm * BM / rpr;
    if (owner == c.rank) return true;
    int ok = 1;
    if ((threadIdx.x & 31) == 0) {
      ok = wait_flag_sys(fused_ready(c, c.rank, owner), epoch(), c.timeout_ns);
      if (!ok) record_timeout(c, owner, op_id, epoch());
    }
    return __shfl_sync(0xffffffffu, ok, 0) != 0;
  }
  __device__ __forceinline__ void math(int, int, float (&v)[64], int, int, float (&)[64]) const {
#pragma unroll
    for (int i = 0; i < 64; ++i) v[i] *= alpha;
  }
  // TMA-store the staged 32x64 block into the owner's slot, at this source
  // rank's rows (the store clips columns past N).
  __device__ void store_block(const CUtensorMap*, const uint8_t* buf, int row0, int col0, int lane) const {
    const int owner = row0 / rpr;
    const int lrow0 = c.rank * rpr + (row0 - owner * rpr);
    if (lane == 0) sm100::tma_store_2d(maps + slot() * kMaxRanks + owner, buf, col0, lrow0);
  }
  // Publish the tile once all epilogue warps have stored their rows. A
  // shared counter (not a named barrier) joins the warps so that a warp that
  // gave up on an earlier wait can never leave the others blocked forever.
  __device__ void end_tile(int tm, int tn, int lane) const {
    if (lane == 0) {
      // This warp's stores of the tile have completed; order them (async
      // proxy) before the generic release chain that publishes the flag.
      sm100::tma_store_wait_all<0>();
      fence_proxy_async_global();
    }
    __syncwarp();
    if (lane == 0) {
      // CTA-scope release is enough here: the flag writer below issues the
      // system-scope fence, and release is cumulative over what it observed.
      __threadfence_block();
      atomicAdd(&s_tile_arrivals(), 1u);
    }
    if (threadIdx.x == 64) {
      const unsigned int target = (s_tile_seq() += (unsigned)arrivals);
      const unsigned long long t0 = globaltimer_ns();
      while (*reinterpret_cast<volatile unsigned int*>(&s_tile_arrivals()) < target) {
        if (globaltimer_ns() - t0 > c.timeout_ns) return;
      }
      const int owner = tm * BM / rpr;
      const int ltile = ((tm * BM - owner * rpr) / BM) * tiles_n + tn;
      fence_sys();
      st_release_sys(fused_tile_flag(c, owner, c.rank, ltile), epoch());
    }
  }
  static __device__ __forceinline__ unsigned int& s_tile_arrivals() {
    __shared__ unsigned int v;
    return v;
  }
  static __device__ __forceinline__ unsigned int& s_tile_seq() {
    __shared__ unsigned int v;
    return v;
  }
  __device__ void finalize() const {
    const int tiles_local = (rpr / BM) * tiles_n;
    const unsigned long long e = epoch();
    const __nv_bfloat16* slot0 =
        reinterpret_cast<const __nv_bfloat16*>(c.peer_base[c.rank] + c.stage_off + (unsigned long long)slot() * c.slot_bytes);
    for (int j = blockIdx.x; j < tiles_local; j += gridDim.x) {
      int ok = 1;
      if ((int)threadIdx.x < c.world) {
        const int src = threadIdx.x;
        ok = wait_flag_sys(fused_tile_flag(c, c.rank, src, j), e, c.timeout_ns);
        if (!ok) record_timeout(c, src, op_id, e);
      }
      if (!__syncthreads_and(ok)) break;
      const int ltm = j / tiles_n, tn = j % tiles_n;
      const int cols = min(BN, N - tn * BN);
      const int cpr = cols / 8;  // 16-byte packs per row
      const int packs = BM * cpr;
      // Four packs per thread in flight for every source rank: the loads of
      // one pass are independent, so the reduction streams instead of paying
      // one L2/NVLink round trip per pack (plain L2 loads: the tile flags
      // observed above order them after the producers' stores).
      constexpr int U = 4;
      const int step = (int)blockDim.x;
      for (int base = threadIdx.x; base < packs; base += U * step) {
        float acc[U][8];
        long long row[U];
        int col[U];
        bool live[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int idx = base + u * step;
          live[u] = idx < packs;
          const int r = live[u] ? idx / cpr : 0, c8 = live[u] ? idx % cpr : 0;
          row[u] = (long long)ltm * BM + r;
          col[u] = tn * BN + c8 * 8;
#pragma unroll
          for (int k = 0; k < 8; ++k) acc[u][k] = 0.f;
        }
        for (int src = 0; src < c.world; ++src) {
          uint4 v[U];
#pragma unroll
          for (int u = 0; u < U; ++u)
            v[u] = live[u] ? ld16_cg(slot0 + ((long long)src * rpr + row[u]) * N + col[u]) : make_uint4(0, 0, 0, 0);
#pragma unroll
          for (int u = 0; u < U; ++u) {
            const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v[u]);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const float2 f = __bfloat1622float2(h[k]);
              acc[u][2 * k] += f.x;
              acc[u][2 * k + 1] += f.y;
            }
          }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          if (!live[u]) continue;
          if (bias) {
#pragma unroll
            for (int k = 0; k < 8; ++k) acc[u][k] += __bfloat162float(bias[col[u] + k]);
          }
          uint4 o;
          __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
          for (int k = 0; k < 4; ++k) oh[k] = __floats2bfloat162_rn(acc[u][2 * k], acc[u][2 * k + 1]);
          *reinterpret_cast<uint4*>(out + row[u] * ldo + col[u]) = o;
        }
      }
      __syncthreads();
    }
    finish_call(c, s_call());
  }
};

// ------------------------------------------------------------ AG -> GEMM
struct GateAG {
  CommDev c;
  int rpr, K, tiles_m;
  const __nv_bfloat16* x;  // [rpr, ldx] local shard
  long long ldx;
  __nv_bfloat16* afull;    // [M, K] local gather buffer (the GEMM's A)
  unsigned int* cnt;       // [tiles_m + 2] zeroed; left zeroed on exit
  int cpt;                 // copy pieces per M-tile
  int extra;               // copy warps per CTA
  int op_id;

  __device__ __forceinline__ unsigned long long epoch() const { return epoch_of(s_call(), 0); }
  __device__ __forceinline__ int slot() const { return (int)(s_call() & 1ull); }

  __device__ bool prologue() const {
    if (!entry_ok(c, op_id)) return false;  // uniform: every thread checks the same arguments
    if (threadIdx.x == 0) s_call() = call_index(c);
    __syncthreads();
    // Stage the local shard: symmetric slot (peers read it) + gather buffer.
    __nv_bfloat16* stage = reinterpret_cast<__nv_bfloat16*>(c.peer_base[c.rank] + c.stage_off +
                                                            (unsigned long long)slot() * c.slot_bytes);
    const long long packs = (long long)rpr * (K / 8);
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < packs;
         i += (long long)gridDim.x * blockDim.x) {
      const long long r = i / (K / 8), c8 = i % (K / 8);
      const uint4 v = ld16(x + r * ldx + c8 * 8);
      st16(stage + r * K + c8 * 8, v);
      st16(afull + ((long long)c.rank * rpr + r) * K + c8 * 8, v);
    }
    __threadfence();
    __syncthreads();
    int ok = 1;
    if (threadIdx.x == 0) {
      // grid-wide barrier: all CTAs are resident (persistent grid <= #SMs)
      atomicAdd(&cnt[tiles_m], 1u);
      const unsigned long long t0 = globaltimer_ns();
      while (ld_acquire_gpu_u32(&cnt[tiles_m]) < gridDim.x) {
        if (globaltimer_ns() - t0 > c.timeout_ns) {
          ok = 0;
          break;
        }
      }
      if (ok && blockIdx.x == 0) announce_ready(c, epoch());
    }
    return __syncthreads_and(ok) != 0;
  }

  __device__ bool wait_a(int tm) const {
    const int p = tm * BM / rpr;
    if (p != c.rank) {
      const unsigned long long t0 = globaltimer_ns();
      while (ld_acquire_gpu_u32(&cnt[tm]) < (unsigned)cpt) {
        if (globaltimer_ns() - t0 > c.timeout_ns) {
          record_timeout(c, p, op_id, epoch());
          return false;
        }
      }
    }
    fence_proxy_async_global();  // generic-proxy writes -> TMA reads
    return true;
  }

  __device__ void copy_role(int cw, int lane) const {
    const int W = c.world;
    const int tps = rpr / BM;             // M-tiles per shard
    const int per_shard = tps * cpt;
    const int total = (W - 1) * per_shard;
    const int cols = K / cpt;             // multiple of 8
    const int nworkers = gridDim.x * extra;
    const unsigned long long e = epoch();
    unsigned int ready_mask = 0;
    for (int q = blockIdx.x * extra + cw; q < total; q += nworkers) {
      const int d = 1 + q / per_shard;
      const int p = (c.rank + d) % W;
      const int rem = q % per_shard;
      const int lt = rem / cpt, piece = rem % cpt;
      if (!(ready_mask & (1u << p))) {
        int ok = 1;
        if (lane == 0) {
          ok = wait_flag_sys(fused_ready(c, c.rank, p), e, c.timeout_ns);
          if (!ok) record_timeout(c, p, op_id, e);
        }
        if (!__shfl_sync(0xffffffffu, ok, 0)) return;
        ready_mask |= 1u << p;
      }
      const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(c.peer_base[p] + c.stage_off +
                                                                        (unsigned long long)slot() * c.slot_bytes) +
                                 (long long)lt * BM * K + piece * cols;
      __nv_bfloat16* dst = afull + ((long long)p * rpr + (long long)lt * BM) * K + piece * cols;
      const int pr = cols / 8;               // 16-byte packs per row
      const int n = BM * pr;
      int i = lane;
      // 16 loads of 16 bytes in flight per lane (8 KiB per warp): NVLink
      // latency x bandwidth needs ~2 MiB in flight across the GPU.
      constexpr int U = 16;
      for (; i + (U - 1) * 32 < n; i += U * 32) {
        uint4 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int k = i + u * 32;
          v[u] = ld16_volatile(src + (long long)(k / pr) * K + (k % pr) * 8);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int k = i + u * 32;
          st16(dst + (long long)(k / pr) * K + (k % pr) * 8, v[u]);
        }
      }
      for (; i < n; i += 32) st16(dst + (long long)(i / pr) * K + (i % pr) * 8, ld16_volatile(src + (long long)(i / pr) * K + (i % pr) * 8));
      fence_proxy_async_global();
      __threadfence();
      __syncwarp();
      if (lane == 0) atomicAdd(&cnt[p * tps + lt], 1u);
    }
  }

  __device__ void finalize() const {
    __shared__ unsigned int ticket;
    if (threadIdx.x == 0) ticket = atomicAdd(&cnt[tiles_m + 1], 1u);
    __syncthreads();
    if (ticket == gridDim.x - 1) {
      // Last CTA: every other CTA has finished; reset the counters for the next call.
      for (int i = threadIdx.x; i < tiles_m + 2; i += blockDim.x) cnt[i] = 0u;
      __threadfence();
    }
    finish_call(c, s_call());
  }
};

}  // namespace gemm

// ------------------------------------------------------------ launchers
cudaError_t gemm_reduce_scatter(const CommDev& c, const __nv_bfloat16* A, const __nv_bfloat16* B,
                                __nv_bfloat16* out, int M, int N, int K, long long lda, long long ldb,
                                long long ldo, const __nv_bfloat16* bias, float alpha, const CUtensorMap* maps,
                                cudaStream_t s) {
  using namespace gemm;
  if (!maps) return cudaErrorInvalidValue;
  const int W = c.world;
  if (M % (W * BM) != 0 || N % 8 != 0) return cudaErrorInvalidValue;
  const int rpr = M / W;
  const int tiles_n = (N + BN - 1) / BN;
  if ((rpr / BM) * tiles_n > kMaxFusedTiles) return cudaErrorInvalidValue;
  if ((unsigned long long)M * N * 2 > c.slot_bytes) return cudaErrorInvalidValue;
  CUtensorMap dummy;
  cudaError_t e = make_tmap_bf16(&dummy, A, M, K, lda, 32, 64);
  if (e != cudaSuccess) return e;
  EpiPeerRS epi{c, rpr, N, tiles_n, alpha, bias, out, ldo, kOpGemmRs, EPI_WARPS, maps};
  const int m_rotate = ((c.rank + 1) % W) * (rpr / BM);
  return launch_gemm_generic<EpiPeerRS, NoGate, 0>(A, B, M, N, K, lda, ldb, dummy, dummy, m_rotate, epi, NoGate{},
                                                   gemm_sm_count(), s);
}

// fp8 (block-scaled) row-parallel linear fused with reduce-scatter: the fp8
// promotion kernel with the same peer-store epilogue (BM = 128, BN = 256 as
// the bf16 kernel, eight storing warps per tile).
cudaError_t gemm_fp8_reduce_scatter(const CommDev& c, const uint8_t* A, const float* sa, const uint8_t* B,
                                    const float* sb, __nv_bfloat16* out, int M, int N, int K, long long lda,
                                    long long ldb, long long ldo, const __nv_bfloat16* bias, float alpha,
                                    const CUtensorMap* maps, cudaStream_t s) {
  using namespace gemm;
  if (!maps) return cudaErrorInvalidValue;
  static_assert(gemm8::BM == BM && gemm8::BN == BN, "tile geometry shared with EpiPeerRS");
  const int W = c.world;
  if (M % (W * BM) != 0 || N % 8 != 0 || K % 16 != 0) return cudaErrorInvalidValue;
  const int rpr = M / W;
  const int tiles_n = (N + BN - 1) / BN;
  if ((rpr / BM) * tiles_n > kMaxFusedTiles) return cudaErrorInvalidValue;
  if ((unsigned long long)M * N * 2 > c.slot_bytes) return cudaErrorInvalidValue;
  CUtensorMap ta, tb, dummy;
  cudaError_t e = make_tmap_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, A, M, K, lda, gemm8::BM, gemm8::BK);
  if (e != cudaSuccess) return e;
  e = make_tmap_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, B, N, K, ldb, gemm8::BN, gemm8::BK);
  if (e != cudaSuccess) return e;
  dummy = ta;
  EpiPeerRS epi{c, rpr, N, tiles_n, alpha, bias, out, ldo, kOpGemmRs, gemm8::PROMO_WARPS, maps};
  const int m_rotate = ((c.rank + 1) % W) * (rpr / BM);
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(gemm8::k_gemm_fp8<EpiPeerRS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         gemm8::SMEM_BYTES);
    attr_set = true;
  }
  gemm8::k_gemm_fp8<EpiPeerRS><<<gemm_sm_count(), gemm8::THREADS, gemm8::SMEM_BYTES, s>>>(
      ta, tb, dummy, dummy, sa, sb, M, N, K, m_rotate, epi, NoGate{}, gemm_err_word());
  return cudaGetLastError();
}

cudaError_t all_gather_gemm(const CommDev& c, const __nv_bfloat16* x, long long ldx, const __nv_bfloat16* B,
                            __nv_bfloat16* out, __nv_bfloat16* afull, unsigned int* cnt, int M, int N, int K,
                            long long ldb, long long ldo, const __nv_bfloat16* bias, int act, __nv_bfloat16* pre,
                            float alpha, cudaStream_t s) {
  using namespace gemm;
  const int W = c.world;
  if (M % (W * BM) != 0 || K % 64 != 0) return cudaErrorInvalidValue;
  const int rpr = M / W;
  if ((unsigned long long)rpr * K * 2 > c.slot_bytes) return cudaErrorInvalidValue;
  CUtensorMap tout, tpre;
  cudaError_t e = make_tmap_bf16(&tout, out, M, N, ldo, 32, 64);
  if (e != cudaSuccess) return e;
  tpre = tout;
  if (pre) {
    e = make_tmap_bf16(&tpre, pre, M, N, ldo, 32, 64);
    if (e != cudaSuccess) return e;
  }
  int cpt = 8;
  while (cpt > 1 && (K / cpt) % 8 != 0) cpt >>= 1;
  constexpr int kExtra = 2;
  GateAG gate{c, rpr, K, M / BM, x, ldx, afull, cnt, cpt, kExtra, kOpAgGemm};
  EpiStore epi{bias, nullptr, 0, alpha, act, pre != nullptr};
  const int m_rotate = c.rank * (rpr / BM);
  return launch_gemm_generic<EpiStore, GateAG, kExtra>(afull, B, M, N, K, K, ldb, tout, tpre, m_rotate, epi, gate,
                                                       gemm_sm_count(), s);
}

}  // namespace nexar
