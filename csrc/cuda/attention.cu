// Self-attention for head dimension 64 on tcgen05 (sm_100a): forward and
// backward, causal or full, bf16 in / out, fp32 softmax statistics.
//
// Layout (the GPT-2 block): qkv is the row-major [B*T, 3C] output of the QKV
// projection (C = H * 64; columns [0, C) are Q, [C, 2C) K, [2C, 3C) V, head h
// at h*64), y the [B*T, C] attention output, lse the [B, H, T] natural-log
// softmax normaliser of every query row (scores scaled by 1/sqrt(64)).
//
// Forward (k_attn_fwd): one CTA per (128-query block, batch, head).
//   warp 0      TMA loads: the Q tile once, then K and V tiles of 128 keys
//               into a 2-deep ring (every load reads this GPU's memory; no
//               multicast);
//   warp 1      allocates 512 TMEM columns; lane 0 issues S = Q K^T
//               (M = N = 128, K = 64) into one of two S accumulators and
//               O_j = P_j V_j (M = 128, N = 64, K = 128) into one of two
//               O accumulators, one block ahead (S of block j is computed
//               while the softmax of block j - 1 runs);
//   warps 4-7   one query row per thread (TMEM lane = row): online softmax in
//               the exp2 domain, P written as bf16 into 128-byte-swizzled
//               shared memory (the A operand of the next MMA), and the
//               running output kept in registers: O = alpha * O + P_j V_j
//               read back from TMEM one block behind.
// Backward (k_attn_bwd): one CTA per (128-key block, batch, head), looping
// over the query blocks that see it.
//   warp 0      K_j, V_j once; Q_i, dO_i, lse_i, Delta_i per step (2-deep);
//   warp 1      S^T = K Q^T and dP^T = V dO^T (M = N = 128, K = 64), then
//               dV += P^T dO, dK += dS^T Q (M = 128, N = 64, K = 128,
//               accumulated in TMEM over all steps) and dQ_i = dS K into one
//               of two TMEM buffers;
//   warps 4-7   one key row per thread: P^T = exp(S^T * scale - lse),
//               dS^T = P^T (dP^T - Delta), both as bf16 into swizzled shared
//               memory (dS^T doubles as the MN-major A operand of dQ);
//   warps 8-11  drain dQ_i from TMEM into a swizzled shared staging tile and
//               add it to the fp32 dQ accumulator with two tensor bulk
//               reductions (cp.reduce.async.bulk.tensor .add, 128 x 32 fp32
//               boxes) per step.
// Delta = rowsum(dO * O) comes from k_attn_delta; k_attn_dq_out scales the
// fp32 dQ accumulator into the Q columns of dqkv.
//
// Every mbarrier wait is bounded (2 s of %globaltimer); a wait that gives up
// records a code in the GEMM error word (gemm_error_flag), the CTA unwinds and
// TMEM is freed after all issued MMAs have completed.
//
// This file has no counterpart in the reference (ml-rust/nexar has no model
// code); it replaces the cuDNN attention that torch's SDPA would run on the
// GPT-2 training path.
#include "attention_api.h"

#include "common.cuh"
#include "gemm_api.h"
#include "sm100.cuh"

namespace nexar {

unsigned int* gemm_err_word();

namespace attn {

using namespace sm100;

constexpr int HD = 64;                       // head dimension
constexpr int BQ = 128, BKV = 128;           // query / key block
constexpr int TILE = 128 * HD * 2;           // one [128][64] bf16 tile: 16 KB
constexpr uint64_t kWait = 2000000000ull;    // ns per wait
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// Byte offset of 16-byte chunk `ch` (0..7) of row `r` in a [rows][64] bf16
// tile stored with the 128-byte swizzle (the layout TMA writes and the UMMA
// descriptors read: chunk ch of row r lands at ch ^ (r & 7)).
NEXAR_D uint32_t sw128(int r, int ch) { return (uint32_t)(r * 128 + ((ch ^ (r & 7)) << 4)); }

// MN-major operand descriptor whose 64-wide MN blocks are `lbo` bytes apart.
NEXAR_D uint64_t desc_mn(uint32_t addr, uint32_t lbo) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}

NEXAR_D uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Untiled bulk copy global -> shared, completion counted on `bar` (both
// addresses 16-byte aligned, size a multiple of 16).
NEXAR_D void bulk_load(void* smem_dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               :: "r"(smem_u32(smem_dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}
// Tiled bulk reduction shared -> global through a tensor map: the box at
// (x, y) of the mapped fp32 tensor += the (swizzled) box in shared memory.
NEXAR_D void tma_reduce_add_2d(const CUtensorMap* map, const void* smem_src, int x, int y) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];"
               :: "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(smem_src)), "r"(x), "r"(y) : "memory");
}
NEXAR_D void named_sync(int id, int threads) { asm volatile("bar.sync %0, %1;" :: "r"(id), "r"(threads) : "memory"); }
// Named barrier that also ANDs `v` over the participating threads: every
// thread gets the same answer, so a group leaves a loop together.
NEXAR_D bool named_and(int id, int threads, bool v) {
  int r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.s32 %0, 1, 0, q;\n\t}"
      : "=r"(r) : "r"(v ? 1 : 0), "r"(id), "r"(threads) : "memory");
  return r != 0;
}

NEXAR_D uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// Bounded wait by lane 0 of a warp; every lane then observes the completed
// phase itself (acquire) before touching the data the phase publishes.
NEXAR_D bool warp_wait(uint64_t* bar, uint32_t parity, int lane) {
  int ok = 1;
  if (lane == 0) ok = mbar_wait_bounded(bar, parity, kWait) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  if (ok) mbar_try_wait(bar, parity);
  return ok != 0;
}

NEXAR_D void fail(unsigned int* err, volatile int* abort_flag, unsigned int code) {
  atomicExch(err, code);
  *abort_flag = 1;
}

NEXAR_D void tmem_ld_x32(uint32_t taddr, uint32_t* r) {
  tmem_ld_32x32b_x32(taddr, *reinterpret_cast<uint32_t(*)[32]>(r));
}

// ============================================================ forward
constexpr int F_Q = 0, F_K = TILE, F_V = 3 * TILE, F_P = 5 * TILE;  // P: 2 buffers x 32 KB
constexpr int F_BAR = F_P + 4 * TILE;
constexpr int F_SMEM = F_BAR + 256 + 1024;
constexpr int F_THREADS = 256;
// TMEM columns: S accumulators at 0 / 128, O accumulators at 256 / 320.
constexpr uint32_t T_S = 0, T_O = 256;

__global__ void __launch_bounds__(F_THREADS, 1)
k_attn_fwd(const __grid_constant__ CUtensorMap tm_qkv, __nv_bfloat16* __restrict__ y, float* __restrict__ lse, int B,
           int T, int H, int causal, float scale_log2, unsigned int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + F_BAR);
  uint64_t* q_full = bar;
  uint64_t* k_full = bar + 1;     // [2]
  uint64_t* v_full = bar + 3;     // [2]
  uint64_t* kv_empty = bar + 5;   // [2]
  uint64_t* s_full = bar + 7;     // [2]
  uint64_t* p_full = bar + 9;     // [2]
  uint64_t* o_full = bar + 11;    // [2]
  uint64_t* o_empty = bar + 13;   // [2]
  uint64_t* mma_done = bar + 15;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 16);
  __shared__ volatile int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = T / BQ;
  const int BH = B * H;
  const int qb = nq - 1 - (int)(blockIdx.x / BH);  // most key blocks first (causal)
  const int bh = (int)(blockIdx.x % BH);
  const int b = bh / H, h = bh % H;
  const int C = H * HD;
  const int nkv = causal ? qb + 1 : nq;
  const int row0 = b * T;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(k_full + s, 1);
      mbar_init(v_full + s, 1);
      mbar_init(kv_empty + s, 1);
      mbar_init(s_full + s, 1);
      mbar_init(p_full + s, 128);
      mbar_init(o_full + s, 1);
      mbar_init(o_empty + s, 128);
    }
    mbar_init(mma_done, 1);
    s_abort = 0;
    mbar_fence_init();
    tma_prefetch_desc(&tm_qkv);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, TILE);
      tma_load_2d(smem + F_Q, &tm_qkv, q_full, h * HD, row0 + qb * BQ);
      int issued = 0;
      for (int j = 0; j < nkv && !s_abort; ++j) {
        const int s = j & 1;
        if (j >= 2 && !mbar_wait_bounded(kv_empty + s, ((j >> 1) - 1) & 1, kWait)) {
          fail(err, &s_abort, 21u);
          break;
        }
        mbar_arrive_expect_tx(k_full + s, TILE);
        tma_load_2d(smem + F_K + s * TILE, &tm_qkv, k_full + s, C + h * HD, row0 + j * BKV);
        mbar_arrive_expect_tx(v_full + s, TILE);
        tma_load_2d(smem + F_V + s * TILE, &tm_qkv, v_full + s, 2 * C + h * HD, row0 + j * BKV);
        issued = j + 1;
      }
      // No TMA write may still be landing when the CTA exits.
      mbar_wait_bounded(q_full, 0, kWait >> 4);
      for (int j = issued > 2 ? issued - 2 : 0; j < issued; ++j) {
        mbar_wait_bounded(k_full + (j & 1), (j >> 1) & 1, kWait >> 4);
        mbar_wait_bounded(v_full + (j & 1), (j >> 1) & 1, kWait >> 4);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idS = umma_idesc_bf16_f32(BQ, BKV);
      constexpr uint32_t idO = umma_idesc_bf16_f32(BQ, HD, false, true);
      const uint32_t q_addr = smem_u32(smem + F_Q);
      bool ok = mbar_wait_bounded(q_full, 0, kWait);
      if (!ok) fail(err, &s_abort, 22u);
      for (int j = 0; ok && j <= nkv && !s_abort; ++j) {
        if (j < nkv) {
          const int s = j & 1;
          if (!mbar_wait_bounded(k_full + s, (j >> 1) & 1, kWait)) {
            fail(err, &s_abort, 23u);
            break;
          }
          tc_fence_after();
          // S buffer s was read by the softmax of block j - 2, which this
          // thread saw finish (p_full) before issuing O_{j-2}.
          const uint32_t k_addr = smem_u32(smem + F_K + s * TILE);
#pragma unroll
          for (int k = 0; k < HD / 16; ++k)
            umma_f16(tbase + T_S + s * BKV, umma_desc_sw128_kmajor(q_addr + k * 32),
                     umma_desc_sw128_kmajor(k_addr + k * 32), idS, k > 0 ? 1u : 0u);
          umma_commit(s_full + s);
        }
        if (j >= 1) {
          const int jj = j - 1, s = jj & 1;
          const uint32_t u = (uint32_t)(jj >> 1);
          if (!mbar_wait_bounded(p_full + s, u & 1, kWait) || !mbar_wait_bounded(v_full + s, u & 1, kWait) ||
              (jj >= 2 && !mbar_wait_bounded(o_empty + s, (u - 1) & 1, kWait))) {
            fail(err, &s_abort, 24u);
            break;
          }
          tc_fence_after();
          const uint32_t p_addr = smem_u32(smem + F_P + s * 2 * TILE);
          const uint32_t v_addr = smem_u32(smem + F_V + s * TILE);
#pragma unroll
          for (int k = 0; k < BKV / 16; ++k)
            umma_f16(tbase + T_O + s * HD, umma_desc_sw128_kmajor(p_addr + (k >> 2) * TILE + (k & 3) * 32),
                     desc_mn(v_addr + k * 2048, 8192), idO, k > 0 ? 1u : 0u);
          umma_commit(o_full + s);
          umma_commit(kv_empty + s);
        }
      }
      // Every issued MMA has finished before TMEM is released.
      umma_commit(mma_done);
      mbar_wait_bounded(mma_done, 0, kWait);
    }
  } else if (warp >= 4) {
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // query row in the block = TMEM lane
    const uint32_t lane_base = tbase + ((uint32_t)(quarter * 32) << 16);
    const int qrow = qb * BQ + r;
    float m = -INFINITY, l = 0.f, alpha_pend = 0.f;
    float o[HD];
#pragma unroll
    for (int i = 0; i < HD; ++i) o[i] = 0.f;
    bool ok = true;

    auto fold = [&](int jj, float a) -> bool {
      const int s = jj & 1;
      if (!warp_wait(o_full + s, (uint32_t)(jj >> 1) & 1, lane)) return false;
      tc_fence_after();
      uint32_t ot[HD];
      tmem_ld_x32(lane_base + T_O + s * HD, ot);
      tmem_ld_x32(lane_base + T_O + s * HD + 32, ot + 32);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(o_empty + s);
#pragma unroll
      for (int i = 0; i < HD; ++i) o[i] = o[i] * a + __uint_as_float(ot[i]);
      return true;
    };

    for (int j = 0; j < nkv; ++j) {
      const int s = j & 1;
      if (!warp_wait(s_full + s, (uint32_t)(j >> 1) & 1, lane) || s_abort) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t x[BKV];
#pragma unroll
      for (int c0 = 0; c0 < BKV; c0 += 32) tmem_ld_x32(lane_base + T_S + s * BKV + c0, x + c0);
      tmem_ld_wait();
      const bool diag = causal && j == qb;
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < BKV; ++c) {
        float v = __uint_as_float(x[c]) * scale_log2;
        if (diag && c > r) v = -INFINITY;
        x[c] = __float_as_uint(v);
        mx = fmaxf(mx, v);
      }
      const float m_new = fmaxf(m, mx);
      const float alpha = exp2f(m - m_new);
      float sum = 0.f;
      uint8_t* pbuf = smem + F_P + s * 2 * TILE;
#pragma unroll
      for (int ch = 0; ch < BKV / 8; ++ch) {
        float p[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          p[e] = exp2f(__uint_as_float(x[ch * 8 + e]) - m_new);
          sum += p[e];
        }
        uint4 pk;
        pk.x = pack_bf16(p[0], p[1]);
        pk.y = pack_bf16(p[2], p[3]);
        pk.z = pack_bf16(p[4], p[5]);
        pk.w = pack_bf16(p[6], p[7]);
        *reinterpret_cast<uint4*>(pbuf + (ch >> 3) * TILE + sw128(r, ch & 7)) = pk;
      }
      l = l * alpha + sum;
      m = m_new;
      fence_proxy_async_smem();  // P (generic-proxy writes) -> the tensor cores
      tc_fence_before();
      mbar_arrive(p_full + s);
      if (j >= 1 && !fold(j - 1, alpha_pend)) {
        ok = false;
        break;
      }
      alpha_pend = alpha;
    }
    if (ok && nkv > 0) ok = fold(nkv - 1, alpha_pend);
    if (ok) {
      const float inv = 1.f / l;
      __nv_bfloat16* yr = y + (size_t)(row0 + qrow) * C + h * HD;
#pragma unroll
      for (int ch = 0; ch < HD / 8; ++ch) {
        uint4 pk;
        pk.x = pack_bf16(o[ch * 8 + 0] * inv, o[ch * 8 + 1] * inv);
        pk.y = pack_bf16(o[ch * 8 + 2] * inv, o[ch * 8 + 3] * inv);
        pk.z = pack_bf16(o[ch * 8 + 4] * inv, o[ch * 8 + 5] * inv);
        pk.w = pack_bf16(o[ch * 8 + 6] * inv, o[ch * 8 + 7] * inv);
        reinterpret_cast<uint4*>(yr)[ch] = pk;
      }
      lse[(size_t)bh * T + qrow] = (m + log2f(l)) * kLn2;
    } else if (lane == 0) {
      fail(err, &s_abort, 25u);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

// ============================================================ backward
constexpr int G_K = 0, G_V = TILE, G_Q = 2 * TILE, G_DO = 4 * TILE;  // Q / dO: 2 stages each
constexpr int G_PT = 6 * TILE, G_DST = 8 * TILE;                      // two [128][64] halves each
constexpr int G_DQS = 10 * TILE;                                      // fp32 [128][64] staging: 32 KB
constexpr int G_LSE = 12 * TILE, G_DEL = G_LSE + 1024;                // [2][128] fp32 each
constexpr int G_BAR = G_DEL + 1024;
constexpr int G_SMEM = G_BAR + 256 + 1024;
constexpr int G_THREADS = 384;
// TMEM columns: S^T 0, dP^T 128, dV 256, dK 320, dQ buffers 384 / 448.
constexpr uint32_t T_ST = 0, T_DPT = 128, T_DV = 256, T_DK = 320, T_DQ = 384;

__global__ void __launch_bounds__(G_THREADS, 1)
k_attn_bwd(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ CUtensorMap tm_do,
           const __grid_constant__ CUtensorMap tm_dq, const float* __restrict__ lse, const float* __restrict__ delta,
           __nv_bfloat16* __restrict__ dqkv, int B, int T, int H, int causal, float scale, unsigned int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + G_BAR);
  uint64_t* kv_full = bar;
  uint64_t* q_full = bar + 1;     // [2]
  uint64_t* q_empty = bar + 3;    // [2]
  uint64_t* sp_full = bar + 5;
  uint64_t* pds_full = bar + 6;
  uint64_t* pds_empty = bar + 7;
  uint64_t* dq_full = bar + 8;    // [2]
  uint64_t* dq_empty = bar + 10;  // [2]
  uint64_t* acc_full = bar + 12;
  uint64_t* mma_done = bar + 13;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 14);
  __shared__ volatile int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = T / BQ;
  const int BH = B * H;
  const int kb = (int)(blockIdx.x / BH);  // key block; the earliest see the most query blocks
  const int bh = (int)(blockIdx.x % BH);
  const int b = bh / H, h = bh % H;
  const int C = H * HD;
  const int i0 = causal ? kb : 0;
  const int nsteps = nq - i0;
  const int row0 = b * T;
  const float scale_log2 = scale * kLog2e;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(q_full + s, 1);
      mbar_init(q_empty + s, 1);
      mbar_init(dq_full + s, 1);
      mbar_init(dq_empty + s, 128);
    }
    mbar_init(sp_full, 1);
    mbar_init(pds_full, 128);
    mbar_init(pds_empty, 1);
    mbar_init(acc_full, 1);
    mbar_init(mma_done, 1);
    s_abort = 0;
    mbar_fence_init();
    tma_prefetch_desc(&tm_qkv);
    tma_prefetch_desc(&tm_do);
    tma_prefetch_desc(&tm_dq);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(kv_full, 2 * TILE);
      tma_load_2d(smem + G_K, &tm_qkv, kv_full, C + h * HD, row0 + kb * BKV);
      tma_load_2d(smem + G_V, &tm_qkv, kv_full, 2 * C + h * HD, row0 + kb * BKV);
      int issued = 0;
      for (int t = 0; t < nsteps && !s_abort; ++t) {
        const int i = i0 + t, s = t & 1;
        if (t >= 2 && !mbar_wait_bounded(q_empty + s, ((t >> 1) - 1) & 1, kWait)) {
          fail(err, &s_abort, 31u);
          break;
        }
        mbar_arrive_expect_tx(q_full + s, 2 * TILE + 2 * 512);
        tma_load_2d(smem + G_Q + s * TILE, &tm_qkv, q_full + s, h * HD, row0 + i * BQ);
        tma_load_2d(smem + G_DO + s * TILE, &tm_do, q_full + s, h * HD, row0 + i * BQ);
        bulk_load(smem + G_LSE + s * 512, lse + (size_t)bh * T + i * BQ, 512, q_full + s);
        bulk_load(smem + G_DEL + s * 512, delta + (size_t)bh * T + i * BQ, 512, q_full + s);
        issued = t + 1;
      }
      mbar_wait_bounded(kv_full, 0, kWait >> 4);
      for (int t = issued > 2 ? issued - 2 : 0; t < issued; ++t)
        mbar_wait_bounded(q_full + (t & 1), (t >> 1) & 1, kWait >> 4);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idS = umma_idesc_bf16_f32(BKV, BQ);
      constexpr uint32_t idKV = umma_idesc_bf16_f32(BKV, HD, false, true);  // dV, dK: B MN-major
      constexpr uint32_t idQ = umma_idesc_bf16_f32(BQ, HD, true, true);     // dQ: A and B MN-major
      const uint32_t k_addr = smem_u32(smem + G_K), v_addr = smem_u32(smem + G_V);
      const uint32_t pt_addr = smem_u32(smem + G_PT), dst_addr = smem_u32(smem + G_DST);
      bool ok = mbar_wait_bounded(kv_full, 0, kWait);
      if (!ok) fail(err, &s_abort, 32u);
      for (int t = 0; ok && t < nsteps && !s_abort; ++t) {
        const int s = t & 1;
        const uint32_t u = (uint32_t)(t >> 1);
        if (!mbar_wait_bounded(q_full + s, u & 1, kWait)) {
          fail(err, &s_abort, 33u);
          break;
        }
        tc_fence_after();
        // S^T / dP^T of step t - 1 were read before pds_full of t - 1 (waited below).
        const uint32_t q_addr = smem_u32(smem + G_Q + s * TILE), do_addr = smem_u32(smem + G_DO + s * TILE);
#pragma unroll
        for (int k = 0; k < HD / 16; ++k)
          umma_f16(tbase + T_ST, umma_desc_sw128_kmajor(k_addr + k * 32), umma_desc_sw128_kmajor(q_addr + k * 32),
                   idS, k > 0 ? 1u : 0u);
#pragma unroll
        for (int k = 0; k < HD / 16; ++k)
          umma_f16(tbase + T_DPT, umma_desc_sw128_kmajor(v_addr + k * 32), umma_desc_sw128_kmajor(do_addr + k * 32),
                   idS, k > 0 ? 1u : 0u);
        umma_commit(sp_full);
        if (!mbar_wait_bounded(pds_full, (uint32_t)t & 1, kWait) ||
            (t >= 2 && !mbar_wait_bounded(dq_empty + s, (u - 1) & 1, kWait))) {
          fail(err, &s_abort, 34u);
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < BQ / 16; ++k)
          umma_f16(tbase + T_DV, umma_desc_sw128_kmajor(pt_addr + (k >> 2) * TILE + (k & 3) * 32),
                   desc_mn(do_addr + k * 2048, 8192), idKV, (t > 0 || k > 0) ? 1u : 0u);
#pragma unroll
        for (int k = 0; k < BQ / 16; ++k)
          umma_f16(tbase + T_DK, umma_desc_sw128_kmajor(dst_addr + (k >> 2) * TILE + (k & 3) * 32),
                   desc_mn(q_addr + k * 2048, 8192), idKV, (t > 0 || k > 0) ? 1u : 0u);
        // dQ_i = dS K: A = dS^T read MN-major (query blocks of 64 are the two halves, TILE apart).
#pragma unroll
        for (int k = 0; k < BKV / 16; ++k)
          umma_f16(tbase + T_DQ + s * HD, desc_mn(dst_addr + k * 2048, TILE), desc_mn(k_addr + k * 2048, 8192), idQ,
                   k > 0 ? 1u : 0u);
        umma_commit(dq_full + s);
        umma_commit(q_empty + s);
        umma_commit(pds_empty);
      }
      if (ok && !s_abort) umma_commit(acc_full);
      umma_commit(mma_done);
      mbar_wait_bounded(mma_done, 0, kWait);
    }
  } else if (warp >= 4 && warp < 8) {
    // ---- P^T and dS^T, one key row per thread
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // key row in the block = TMEM lane
    const uint32_t lane_base = tbase + ((uint32_t)(quarter * 32) << 16);
    bool ok = true;
    for (int t = 0; t < nsteps; ++t) {
      const int i = i0 + t, s = t & 1;
      if (!warp_wait(sp_full, (uint32_t)t & 1, lane) || !warp_wait(q_full + s, (uint32_t)(t >> 1) & 1, lane) ||
          (t >= 1 && !warp_wait(pds_empty, (uint32_t)(t - 1) & 1, lane)) || s_abort) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float* lse_s = reinterpret_cast<const float*>(smem + G_LSE + s * 512);
      const float* del_s = reinterpret_cast<const float*>(smem + G_DEL + s * 512);
      const bool diag = causal && i == kb;
#pragma unroll 1
      for (int c0 = 0; c0 < BQ; c0 += 32) {
        uint32_t sr[32], dr[32];
        tmem_ld_x32(lane_base + T_ST + c0, sr);
        tmem_ld_x32(lane_base + T_DPT + c0, dr);
        tmem_ld_wait();
        float p[32], ds[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int c = c0 + e;  // query column
          float pv = exp2f(__uint_as_float(sr[e]) * scale_log2 - lse_s[c] * kLog2e);
          if (diag && c < r) pv = 0.f;  // key r is later than query c
          p[e] = pv;
          ds[e] = pv * (__uint_as_float(dr[e]) - del_s[c]);
        }
        const int half = c0 >> 6;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int ch = ((c0 & 63) >> 3) + q;
          uint4 pk, dk;
          pk.x = pack_bf16(p[q * 8 + 0], p[q * 8 + 1]);
          pk.y = pack_bf16(p[q * 8 + 2], p[q * 8 + 3]);
          pk.z = pack_bf16(p[q * 8 + 4], p[q * 8 + 5]);
          pk.w = pack_bf16(p[q * 8 + 6], p[q * 8 + 7]);
          dk.x = pack_bf16(ds[q * 8 + 0], ds[q * 8 + 1]);
          dk.y = pack_bf16(ds[q * 8 + 2], ds[q * 8 + 3]);
          dk.z = pack_bf16(ds[q * 8 + 4], ds[q * 8 + 5]);
          dk.w = pack_bf16(ds[q * 8 + 6], ds[q * 8 + 7]);
          *reinterpret_cast<uint4*>(smem + G_PT + half * TILE + sw128(r, ch)) = pk;
          *reinterpret_cast<uint4*>(smem + G_DST + half * TILE + sw128(r, ch)) = dk;
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(pds_full);
    }
    if (ok && warp_wait(acc_full, 0, lane)) {
      tc_fence_after();
      uint32_t dv[HD], dk[HD];
      tmem_ld_x32(lane_base + T_DV, dv);
      tmem_ld_x32(lane_base + T_DV + 32, dv + 32);
      tmem_ld_x32(lane_base + T_DK, dk);
      tmem_ld_x32(lane_base + T_DK + 32, dk + 32);
      tmem_ld_wait();
      const size_t row = (size_t)(row0 + kb * BKV + r) * (3 * C);
      uint4* gk = reinterpret_cast<uint4*>(dqkv + row + C + h * HD);
      uint4* gv = reinterpret_cast<uint4*>(dqkv + row + 2 * C + h * HD);
#pragma unroll
      for (int ch = 0; ch < HD / 8; ++ch) {
        const float* fk = reinterpret_cast<const float*>(dk + ch * 8);
        const float* fv = reinterpret_cast<const float*>(dv + ch * 8);
        uint4 pk, pv;
        pk.x = pack_bf16(fk[0] * scale, fk[1] * scale);
        pk.y = pack_bf16(fk[2] * scale, fk[3] * scale);
        pk.z = pack_bf16(fk[4] * scale, fk[5] * scale);
        pk.w = pack_bf16(fk[6] * scale, fk[7] * scale);
        pv.x = pack_bf16(fv[0], fv[1]);
        pv.y = pack_bf16(fv[2], fv[3]);
        pv.z = pack_bf16(fv[4], fv[5]);
        pv.w = pack_bf16(fv[6], fv[7]);
        gk[ch] = pk;
        gv[ch] = pv;
      }
    } else if (lane == 0) {
      fail(err, &s_abort, 35u);
    }
  } else if (warp >= 8) {
    // ---- dQ_i: TMEM -> swizzled shared staging -> tensor bulk fp32 adds into the accumulator
    const int quarter = warp & 3;
    const int rq = quarter * 32 + lane;  // query row in the block = TMEM lane
    const uint32_t lane_base = tbase + ((uint32_t)(quarter * 32) << 16);
    const bool issuer = (warp == 8 && lane == 0);
    uint8_t* stage = smem + G_DQS;
    for (int t = 0; t < nsteps; ++t) {
      const int i = i0 + t, s = t & 1;
      const bool ok = warp_wait(dq_full + s, (uint32_t)(t >> 1) & 1, lane) && !s_abort;
      uint32_t v[HD];
      if (ok) {
        tc_fence_after();
        tmem_ld_x32(lane_base + T_DQ + s * HD, v);
        tmem_ld_x32(lane_base + T_DQ + s * HD + 32, v + 32);
        tmem_ld_wait();
        tc_fence_before();
        mbar_arrive(dq_empty + s);
      }
      // The staging tile is free once the previous reduction has read it.
      if (issuer) tma_store_wait_read<0>();
      // All four warps leave together if any of them gave up (no one may
      // wait at the barriers below for a warp that has left).
      if (!named_and(2, 128, ok)) break;
      // Row rq as two 128 x 32 fp32 boxes in the 128-byte-swizzled layout of
      // the dQ tensor map (chunk k of 4 floats lands at k ^ (rq & 7)).
#pragma unroll
      for (int k = 0; k < HD / 4; ++k) {
        float4 f;
        f.x = __uint_as_float(v[k * 4 + 0]);
        f.y = __uint_as_float(v[k * 4 + 1]);
        f.z = __uint_as_float(v[k * 4 + 2]);
        f.w = __uint_as_float(v[k * 4 + 3]);
        *reinterpret_cast<float4*>(stage + (k >> 3) * TILE + sw128(rq, k & 7)) = f;
      }
      fence_proxy_async_smem();
      named_sync(2, 128);
      if (issuer) {
        const int y0 = bh * T + i * BQ;
        tma_reduce_add_2d(&tm_dq, stage, 0, y0);
        tma_reduce_add_2d(&tm_dq, stage + TILE, 32, y0);
        tma_store_commit();
      }
    }
    if (issuer) tma_store_wait_all<0>();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

// Delta[b, h, t] = sum_d dO[b*T + t, h*64 + d] * O[b*T + t, h*64 + d] (fp32).
__global__ void k_attn_delta(const __nv_bfloat16* __restrict__ y, const __nv_bfloat16* __restrict__ dy,
                             float* __restrict__ delta, int BT, int T, int H) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)BT * H) return;
  const int row = (int)(idx / H), h = (int)(idx % H);
  const int C = H * HD;
  const uint4* a = reinterpret_cast<const uint4*>(y + (size_t)row * C + h * HD);
  const uint4* g = reinterpret_cast<const uint4*>(dy + (size_t)row * C + h * HD);
  float acc = 0.f;
#pragma unroll
  for (int ch = 0; ch < HD / 8; ++ch) {
    const uint4 va = a[ch], vg = g[ch];
    const __nv_bfloat162* pa = reinterpret_cast<const __nv_bfloat162*>(&va);
    const __nv_bfloat162* pg = reinterpret_cast<const __nv_bfloat162*>(&vg);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 fa = __bfloat1622float2(pa[e]), fg = __bfloat1622float2(pg[e]);
      acc += fa.x * fg.x + fa.y * fg.y;
    }
  }
  const int bb = row / T, t = row % T;
  delta[((size_t)bb * H + h) * T + t] = acc;
}

// dqkv[b*T + t, h*64 + d] = bf16(scale * dq_acc[b, h, t, d]).
__global__ void k_attn_dq_out(const float* __restrict__ dq_acc, __nv_bfloat16* __restrict__ dqkv, int B, int T,
                              int H, float scale) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;  // one 8-element chunk each
  if (idx >= (long long)B * H * T * (HD / 8)) return;
  const int ch = (int)(idx % (HD / 8));
  const long long rowh = idx / (HD / 8);  // (b*H + h) * T + t
  const int t = (int)(rowh % T);
  const int bh = (int)(rowh / T);
  const int b = bh / H, h = bh % H;
  const float4* src = reinterpret_cast<const float4*>(dq_acc + rowh * HD + ch * 8);
  const float4 f0 = src[0], f1 = src[1];
  uint4 pk;
  pk.x = pack_bf16(f0.x * scale, f0.y * scale);
  pk.y = pack_bf16(f0.z * scale, f0.w * scale);
  pk.z = pack_bf16(f1.x * scale, f1.y * scale);
  pk.w = pack_bf16(f1.z * scale, f1.w * scale);
  const int C = H * HD;
  *reinterpret_cast<uint4*>(dqkv + (size_t)(b * T + t) * (3 * C) + h * HD + ch * 8) = pk;
}

}  // namespace attn

// ------------------------------------------------------------ host
bool attention_supported(int B, int T, int H, int head_dim) {
  return B > 0 && H > 0 && head_dim == attn::HD && T > 0 && T % attn::BQ == 0;
}

size_t attention_bwd_workspace_floats(int B, int T, int H) {
  return (size_t)B * H * T * attn::HD + (size_t)B * H * T;
}

cudaError_t attention_fwd(const __nv_bfloat16* qkv, __nv_bfloat16* y, float* lse, int B, int T, int H, bool causal,
                          cudaStream_t s) {
  using namespace attn;
  if (!attention_supported(B, T, H, HD)) return cudaErrorInvalidValue;
  const int C = H * HD;
  CUtensorMap tm;
  cudaError_t e = make_tmap_bf16(&tm, qkv, (long long)B * T, 3LL * C, 3LL * C, BQ, HD);
  if (e != cudaSuccess) return e;
  static bool attr_set = false;
  if (!attr_set) {
    e = cudaFuncSetAttribute(k_attn_fwd, cudaFuncAttributeMaxDynamicSharedMemorySize, F_SMEM);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  const float scale_log2 = kLog2e / sqrtf((float)HD);
  const unsigned grid = (unsigned)((T / BQ) * B * H);
  k_attn_fwd<<<grid, F_THREADS, F_SMEM, s>>>(tm, y, lse, B, T, H, causal ? 1 : 0, scale_log2, gemm_err_word());
  return cudaGetLastError();
}

cudaError_t attention_bwd(const __nv_bfloat16* qkv, const __nv_bfloat16* y, const __nv_bfloat16* dy,
                          const float* lse, __nv_bfloat16* dqkv, float* ws, int B, int T, int H, bool causal,
                          cudaStream_t s) {
  using namespace attn;
  if (!attention_supported(B, T, H, HD)) return cudaErrorInvalidValue;
  const int C = H * HD;
  float* dq_acc = ws;
  float* delta = ws + (size_t)B * H * T * HD;
  CUtensorMap tq, tdo, tdq;
  cudaError_t e = make_tmap_bf16(&tq, qkv, (long long)B * T, 3LL * C, 3LL * C, BQ, HD);
  if (e != cudaSuccess) return e;
  e = make_tmap_bf16(&tdo, dy, (long long)B * T, C, C, BQ, HD);
  if (e != cudaSuccess) return e;
  // dQ accumulator [B*H*T, 64] fp32, boxes of 128 rows x 32 columns (128 bytes).
  e = make_tmap_2d(&tdq, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, dq_acc, (long long)B * H * T, HD, HD, BQ, 32);
  if (e != cudaSuccess) return e;
  static bool attr_set = false;
  if (!attr_set) {
    e = cudaFuncSetAttribute(k_attn_bwd, cudaFuncAttributeMaxDynamicSharedMemorySize, G_SMEM);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  e = cudaMemsetAsync(dq_acc, 0, (size_t)B * H * T * HD * sizeof(float), s);
  if (e != cudaSuccess) return e;
  const long long rows = (long long)B * T * H;
  k_attn_delta<<<(unsigned)((rows + 255) / 256), 256, 0, s>>>(y, dy, delta, B * T, T, H);
  const float scale = 1.f / sqrtf((float)HD);
  const unsigned grid = (unsigned)((T / BKV) * B * H);
  k_attn_bwd<<<grid, G_THREADS, G_SMEM, s>>>(tq, tdo, tdq, lse, delta, dqkv, B, T, H, causal ? 1 : 0, scale,
                                              gemm_err_word());
  const long long chunks = (long long)B * H * T * (HD / 8);
  k_attn_dq_out<<<(unsigned)((chunks + 255) / 256), 256, 0, s>>>(dq_acc, dqkv, B, T, H, scale);
  return cudaGetLastError();
}

}  // namespace nexar
