// Self-attention for head dimension 64 on tcgen05 (sm_100a): forward and
// backward, causal or full, bf16 in / out, fp32 softmax statistics.
//
// Layout (the GPT-2 block): qkv is the row-major [B*T, 3C] output of the QKV
// projection (C = H * 64; columns [0, C) are Q, [C, 2C) K, [2C, 3C) V, head h
// at h*64), y the [B*T, C] attention output, lse the [B, H, T] natural-log
// softmax normaliser of every query row (scores scaled by 1/sqrt(64)).
//
// Forward (k_attn_fwd): one CTA per (pair of adjacent 128-query tiles A and
// B, batch, head); the tiles share every K / V load.
//   warp 0      TMA loads: both Q tiles once, then K and V tiles of 128 keys
//               into a 3-deep ring (every load reads this GPU's memory; no
//               multicast);
//   warps 1-2   warp 1 allocates 512 TMEM columns; lane 0 of warp 1 (tile A)
//               and of warp 2 (tile B) issues S_t = Q_t K_j^T (M = N = 128,
//               K = 64) for the next key block as soon as the tile's softmax
//               holds the current scores, and O_t += P_t V_j (M = 128,
//               N = 64, K = 128, P read from TMEM) once P_t is written. One
//               issuer per tile: the tensor pipe takes an MMA only as fast as
//               it runs them, so a single issuer would serialise the tiles;
//               O_A and O_B accumulate in TMEM;
//   warps 4-7   softmax of tile A, warps 8-11 of tile B, one query row per
//               thread (TMEM lane = row), in the exp2 domain. The running
//               maximum is raised lazily (only when a block's maximum exceeds
//               it by more than 2^8), so the accumulated output is rescaled
//               in TMEM only on those blocks. A quarter of the exponentials
//               run on the FMA pipe (exp2_poly2), the rest on the MUFU unit.
//               P goes to TMEM as packed bf16 (tcgen05.st), where the next
//               MMA reads it as its A operand.
// Backward (k_attn_bwd): one CTA per (128-key block, batch, head), looping
// over the query blocks that see it, each as two halves of 64 queries.
//   warp 0      K_j, V_j once; Q_i, dO_i, lse_i, Delta_i per block (2-deep);
//   warp 1      S^T = K Q_half^T and dP^T = V dO_half^T (M = 128, N = 64,
//               K = 64) into one of two TMEM half buffers, two halves ahead;
//               dV += P^T dO_half, dK += dS^T Q_half (K = 64, accumulated in
//               TMEM over all steps); after both halves dQ_i = dS K
//               (M = 128, N = 64, K = 128) into one of two TMEM buffers;
//   warps 4-11  one key row per thread, 32 query columns of a half per warp:
//               P^T = exp(S^T * scale - lse), dS^T = P^T (dP^T - Delta), both
//               as bf16 into swizzled shared memory (dS^T doubles as the
//               MN-major A operand of dQ); at the end dV (warps 4-7) and dK
//               (warps 8-11) from TMEM to dqkv;
//   warps 12-15 drain dQ_i from TMEM into a swizzled shared staging tile and
//               add it to the fp32 dQ accumulator with two tensor bulk
//               reductions (cp.reduce.async.bulk.tensor .add, 128 x 32 fp32
//               boxes) per query block.
// k_attn_prep computes Delta = rowsum(dO * O) and clears the dQ accumulator;
// k_attn_dq_out scales the fp32 dQ accumulator into the Q columns of dqkv.
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

// Non-blocking phase test (never suspends the thread).
NEXAR_D bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
  return ok != 0;
}

// Bounded wait by lane 0 of a warp; every lane then observes the completed
// phase itself (acquire) before touching the data the phase publishes.
NEXAR_D bool warp_wait(uint64_t* bar, uint32_t parity, int lane) {
  // Fast path: one warp-wide test (the phase is usually complete already).
  if (mbar_test(bar, parity)) return true;
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

// Event timeline of one CTA (SM clock, %clock64) for tuning the pipelines:
// recorded only when attention_trace_select picked that CTA. Slots: forward
// softmax of tile t at 512 t + 8 j + k, forward MMA at 1024 + 8 j + 4 t + k,
// forward loads at 1536 + j; backward softmax at 2048 + 4 u + k, backward MMA
// at 3072 + 4 u + k.
constexpr int kTraceSlots = 4096;
__device__ unsigned long long g_trace[kTraceSlots];
__device__ int g_trace_cta = -1;
// `on` is this CTA's (blockIdx.x == g_trace_cta), read once at kernel entry.
NEXAR_D void trace(bool on, int slot) {
  if (on && slot >= 0 && slot < kTraceSlots) g_trace[slot] = clock64();
}

NEXAR_D float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
NEXAR_D float ex2(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// Packed fp32 pairs (Blackwell f32x2 pipes): d = a * b + c, a + b, a * b.
NEXAR_D void ffma2(float& d0, float& d1, float a0, float a1, float b0, float b1, float c0, float c1) {
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d0), "=f"(d1) : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}
NEXAR_D void fadd2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d0), "=f"(d1) : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}
NEXAR_D void fmul2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d0), "=f"(d1) : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

// 2^x of two values on the FMA pipe, taking part of the exponentials off the
// MUFU unit (its 16 results per SM clock bound the softmax). Method: the
// Cody-Waite split x = n + f with n = rint(x) (the 1.5 * 2^23 rounding
// constant) and |f| <= 1/2; 2^f by a cubic whose coefficients were fitted for
// this file by Lawson-weighted least squares on [-1/2, 1/2] (maximum relative
// error 7.5e-5, below the bf16 rounding of P); 2^n by adding n to the exponent
// field. Inputs below -125 (the masked -inf among them) give exactly 0.
NEXAR_D void exp2_poly2(float& r0, float& r1, float x0, float x1) {
  constexpr float kRound = 12582912.f;  // 1.5 * 2^23
  constexpr float c0 = 0.9999281764f, c1 = 0.6932609677f, c2 = 0.2426097095f, c3 = 0.0551709794f;
  const float y0 = fmaxf(x0, -125.f), y1 = fmaxf(x1, -125.f);
  float t0, t1, n0, n1, f0, f1, p0, p1;
  fadd2(t0, t1, y0, y1, kRound, kRound);
  fadd2(n0, n1, t0, t1, -kRound, -kRound);
  fadd2(f0, f1, y0, y1, -n0, -n1);
  ffma2(p0, p1, c3, c3, f0, f1, c2, c2);
  ffma2(p0, p1, p0, p1, f0, f1, c1, c1);
  ffma2(p0, p1, p0, p1, f0, f1, c0, c0);
  const int e0 = __float_as_int(p0) + (__float_as_int(t0) << 23);
  const int e1 = __float_as_int(p1) + (__float_as_int(t1) << 23);
  r0 = x0 < -125.f ? 0.f : __int_as_float(e0);
  r1 = x1 < -125.f ? 0.f : __int_as_float(e1);
}

NEXAR_D void tmem_st_x32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
      :: "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
         "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
         "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
         "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
NEXAR_D void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// kind::f16 MMA whose A operand is read from tensor memory (M = 128 rows in
// the 128 lanes, K along the columns, two bf16 per 32-bit column) and B from
// shared memory: no shared-memory traffic for A.
NEXAR_D void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      :: "r"(tmem_d), "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}

// ============================================================ forward
// One CTA per pair of adjacent 128-query tiles (A = 2p, B = 2p + 1) of one
// (batch, head): the two tiles share every K / V load, and their softmax
// warpgroups overlap on the SM (one computes exponentials while the tensor
// cores run the other's MMAs).
constexpr int F_STAGES = 3;
constexpr int F_QA = 0;                             // Q_A, Q_B: 2 tiles
constexpr int F_K = 2 * TILE;                       // K ring
constexpr int F_V = F_K + F_STAGES * TILE;          // V ring
constexpr int F_BAR = F_V + F_STAGES * TILE;
constexpr int F_SMEM = F_BAR + 256 + 1024;
// Warpgroup 0: TMA (warp 0), MMA (warp 1); warpgroup 1: softmax of tile A;
// warpgroup 2: softmax of tile B. 168 registers per thread (3 warps per SM
// sub-partition: 3 x 32 x 168 = 16,128 of its 16,384).
constexpr int F_THREADS = 384;
// TMEM columns: S_A 0, S_B 128 (fp32 scores), O_A 256, O_B 320 (fp32 output
// accumulators), P_A 384, P_B 448 (bf16 probabilities, two per column: the A
// operand of O += P V, read by the tensor cores straight from TMEM).
constexpr uint32_t T_S = 0, T_O = 256, T_P = 384;
// The running maximum is raised only when a block's maximum exceeds it by
// more than 2^8: between raises the probabilities stay below 256 (exact in
// fp32, ample range in bf16) and the output accumulator needs no rescaling.
constexpr float kRescaleLog2 = 8.f;

__global__ void __launch_bounds__(F_THREADS, 1)
k_attn_fwd(const __grid_constant__ CUtensorMap tm_qkv, __nv_bfloat16* __restrict__ y, float* __restrict__ lse, int B,
           int T, int H, int causal, float scale_log2, unsigned int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + F_BAR);
  uint64_t* q_full = bar;
  uint64_t* k_full = bar + 1;     // [F_STAGES]
  uint64_t* v_full = bar + 4;     // [F_STAGES]
  uint64_t* kv_empty = bar + 7;   // [F_STAGES]
  uint64_t* s_full = bar + 10;    // [2] per tile: S = Q K^T complete
  uint64_t* s_free = bar + 12;    // [2] per tile: S read into registers
  uint64_t* p_full = bar + 14;    // [2] per tile: P in shared memory, O rescaled
  uint64_t* o_done = bar + 16;    // [2] per tile: O += P V complete
  uint64_t* mma_done = bar + 18;  // [2] per MMA issuer
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 20);
  __shared__ volatile int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool tron = (int)blockIdx.x == g_trace_cta;
  const int nq = T / BQ;
  const int npair = (nq + 1) / 2;
  const int BH = B * H;
  const int pr = npair - 1 - (int)(blockIdx.x / BH);  // most key blocks first (causal)
  const int bh = (int)(blockIdx.x % BH);
  const int b = bh / H, h = bh % H;
  const int C = H * HD;
  const int row0 = b * T;
  const int ntile = (2 * pr + 1 < nq) ? 2 : 1;
  int nkv[2];
#pragma unroll
  for (int t = 0; t < 2; ++t) nkv[t] = causal ? 2 * pr + t + 1 : nq;
  const int nkv_max = nkv[ntile - 1];

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < F_STAGES; ++s) {
      mbar_init(k_full + s, 1);
      mbar_init(v_full + s, 1);
      mbar_init(kv_empty + s, ntile);  // one commit per tile's MMA issuer
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(s_full + t, 1);
      mbar_init(s_free + t, 128);
      mbar_init(p_full + t, 128);
      mbar_init(o_done + t, 1);
    }
    mbar_init(mma_done, 1);
    mbar_init(mma_done + 1, 1);
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
      mbar_arrive_expect_tx(q_full, ntile * TILE);
      for (int t = 0; t < ntile; ++t)
        tma_load_2d(smem + F_QA + t * TILE, &tm_qkv, q_full, h * HD, row0 + (2 * pr + t) * BQ);
      int issued = 0;
      for (int j = 0; j < nkv_max && !s_abort; ++j) {
        const int st = j % F_STAGES;
        if (j >= F_STAGES && !mbar_wait_bounded(kv_empty + st, ((j / F_STAGES) - 1) & 1, kWait)) {
          fail(err, &s_abort, 21u);
          break;
        }
        mbar_arrive_expect_tx(k_full + st, TILE);
        tma_load_2d(smem + F_K + st * TILE, &tm_qkv, k_full + st, C + h * HD, row0 + j * BKV);
        mbar_arrive_expect_tx(v_full + st, TILE);
        tma_load_2d(smem + F_V + st * TILE, &tm_qkv, v_full + st, 2 * C + h * HD, row0 + j * BKV);
        trace(tron, 1536 + j);
        issued = j + 1;
      }
      // No TMA write may still be landing when the CTA exits.
      mbar_wait_bounded(q_full, 0, kWait >> 4);
      for (int j = issued > F_STAGES ? issued - F_STAGES : 0; j < issued; ++j) {
        mbar_wait_bounded(k_full + j % F_STAGES, (j / F_STAGES) & 1, kWait >> 4);
        mbar_wait_bounded(v_full + j % F_STAGES, (j / F_STAGES) & 1, kWait >> 4);
      }
    }
  } else if (warp == 1 || warp == 2) {
    // One MMA issuer per tile (warp 1: tile A, warp 2: tile B), each in its
    // tile's own order with blocking waits: the tensor pipe interleaves the
    // two tiles' MMAs, so one tile's late softmax never holds back the other.
    const int t = warp - 1;
    if (lane == 0) {
      // Descriptors are computed once: a K step of 16 elements advances a
      // K-major operand by 32 bytes (start-address field + 2) and an
      // MN-major one by 16 rows of 128 bytes (+ 128); stages and tiles are
      // TILE bytes apart (+ TILE / 16).
      constexpr uint32_t idS = umma_idesc_bf16_f32(BQ, BKV);
      constexpr uint32_t idO = umma_idesc_bf16_f32(BQ, HD, false, true);
      constexpr uint64_t kTileStep = TILE >> 4;
      const uint64_t dq = umma_desc_sw128_kmajor(smem_u32(smem + F_QA)) + (uint64_t)t * kTileStep;
      const uint64_t dk0 = umma_desc_sw128_kmajor(smem_u32(smem + F_K));
      const uint64_t dv0 = desc_mn(smem_u32(smem + F_V), 8192);
      const uint32_t d_s = tbase + T_S + t * BKV, d_o = tbase + T_O + t * HD, pa = tbase + T_P + t * 64;
      const int nk = t < ntile ? nkv[t] : 0;
      auto issue_s = [&](int j) {
        const uint64_t db = dk0 + (uint64_t)(j % F_STAGES) * kTileStep;
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) umma_f16(d_s, dq + 2 * k, db + 2 * k, idS, k > 0 ? 1u : 0u);
        umma_commit(s_full + t);
      };
      bool ok = true;
      if (nk > 0) {
        ok = mbar_wait_bounded(q_full, 0, kWait) && mbar_wait_bounded(k_full, 0, kWait);
        if (ok) {
          tc_fence_after();
          issue_s(0);
        } else {
          fail(err, &s_abort, 22u);
        }
      }
      for (int j = 0; ok && j < (t < ntile ? nkv_max : 0) && !s_abort; ++j) {
        if (j < nk) {
          // The next scores as soon as the softmax holds the current ones.
          if (j + 1 < nk) {
            if (!mbar_wait_bounded(s_free + t, j & 1, kWait) ||
                !mbar_wait_bounded(k_full + (j + 1) % F_STAGES, ((j + 1) / F_STAGES) & 1, kWait)) {
              fail(err, &s_abort, 23u);
              ok = false;
              break;
            }
            tc_fence_after();
            issue_s(j + 1);
            trace(tron, 1024 + 8 * j + 4 * t);
          }
          // O_t += P_t V_j (P read from TMEM) once the softmax has written P_t.
          if (!mbar_wait_bounded(p_full + t, j & 1, kWait) ||
              !mbar_wait_bounded(v_full + j % F_STAGES, (j / F_STAGES) & 1, kWait)) {
            fail(err, &s_abort, 24u);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t db = dv0 + (uint64_t)(j % F_STAGES) * kTileStep;
#pragma unroll
          for (int k = 0; k < BKV / 16; ++k)  // K step of 16 = 8 TMEM columns of packed P
            umma_f16_ts(d_o, pa + 8 * k, db + 128 * k, idO, (j > 0 || k > 0) ? 1u : 0u);
          umma_commit(o_done + t);
          trace(tron, 1024 + 8 * j + 4 * t + 1);
        }
        // This tile is done with K_j and V_j (the stage frees after both tiles).
        umma_commit(kv_empty + j % F_STAGES);
      }
      // Every issued MMA has finished before TMEM is released.
      umma_commit(mma_done + t);
      mbar_wait_bounded(mma_done + t, 0, kWait);
    }
  } else if (warp >= 4) {
    const int t = (warp >> 2) - 1;        // tile of this warpgroup
    const int quarter = warp & 3;         // TMEM lane quarter of this warp
    const int r = quarter * 32 + lane;    // query row in the tile = TMEM lane
    if (t < ntile) {
      const uint32_t lane_base = tbase + ((uint32_t)(quarter * 32) << 16);
      const uint32_t s_col = T_S + t * BKV, o_col = T_O + t * HD;
      const int qt = 2 * pr + t;
      const int qrow = qt * BQ + r;
      float m = -INFINITY, l = 0.f;
      bool ok = true;
      const bool tr = tron && r == 0;
      for (int j = 0; j < nkv[t]; ++j) {
        if (!warp_wait(s_full + t, (uint32_t)j & 1, lane) || s_abort) {
          ok = false;
          break;
        }
        if (tr) trace(true, 512 * t + 8 * j);
        tc_fence_after();
        uint32_t x[BKV];
#pragma unroll
        for (int c0 = 0; c0 < BKV; c0 += 32) tmem_ld_x32(lane_base + s_col + c0, x + c0);
        tmem_ld_wait();
        tc_fence_before();
        mbar_arrive(s_free + t);
        if (tr) trace(true, 512 * t + 8 * j + 1);
        if (causal && j == qt) {
#pragma unroll
          for (int c = 0; c < BKV; ++c)
            if (c > r) x[c] = __float_as_uint(-INFINITY);
        }
        float mx0 = __uint_as_float(x[0]), mx1 = __uint_as_float(x[1]);
        float mx2 = __uint_as_float(x[2]), mx3 = __uint_as_float(x[3]);
#pragma unroll
        for (int c = 4; c < BKV; c += 8) {
          mx0 = fmax3(mx0, __uint_as_float(x[c + 0]), __uint_as_float(x[c + 1]));
          mx1 = fmax3(mx1, __uint_as_float(x[c + 2]), __uint_as_float(x[c + 3]));
          mx2 = fmax3(mx2, __uint_as_float(x[c + 4]), __uint_as_float(x[c + 5]));
          mx3 = fmax3(mx3, __uint_as_float(x[c + 6]), __uint_as_float(x[c + 7]));
        }
        const float m_blk = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * scale_log2;
        const bool raise = m_blk > m + kRescaleLog2;
        const float m_new = raise ? m_blk : m;
        const float alpha = raise ? ex2(m - m_new) : 1.f;
        if (tr) trace(true, 512 * t + 8 * j + 2);
        if (j >= 1) {
          // P_t (TMEM) and O_t are free once O_t += P_{j-1} V_{j-1} has completed.
          if (!warp_wait(o_done + t, (uint32_t)(j - 1) & 1, lane)) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
        if (tr) trace(true, 512 * t + 8 * j + 3);
        // Probabilities into the row's P columns of TMEM, 32 columns (64
        // values) at a time: 6 of every 8 exponentials on the MUFU unit, 2 on
        // the FMA pipe (exp2_poly2), which balances the two for this loop.
        const float neg = -m_new;
        float sum0 = 0.f, sum1 = 0.f;
        uint32_t pk[32];
#pragma unroll
        for (int ch = 0; ch < BKV / 8; ++ch) {
          float p[8];
#pragma unroll
          for (int e = 0; e < 8; e += 2)
            ffma2(p[e], p[e + 1], __uint_as_float(x[ch * 8 + e]), __uint_as_float(x[ch * 8 + e + 1]), scale_log2,
                  scale_log2, neg, neg);
#pragma unroll
          for (int e = 0; e < 6; ++e) p[e] = ex2(p[e]);
          exp2_poly2(p[6], p[7], p[6], p[7]);
          sum0 += (p[0] + p[2]) + (p[4] + p[6]);
          sum1 += (p[1] + p[3]) + (p[5] + p[7]);
          const int q = (ch & 7) * 4;
          pk[q + 0] = pack_bf16(p[0], p[1]);
          pk[q + 1] = pack_bf16(p[2], p[3]);
          pk[q + 2] = pack_bf16(p[4], p[5]);
          pk[q + 3] = pack_bf16(p[6], p[7]);
          if ((ch & 7) == 7) tmem_st_x32(lane_base + T_P + t * 64 + (ch >> 3) * 32, pk);
        }
        tmem_st_wait();
        l = l * alpha + (sum0 + sum1);
        m = m_new;
        if (j >= 1 && __any_sync(0xffffffffu, raise)) {
          // The maximum rose: scale the accumulated output to it before P_j V_j is added.
          uint32_t o[HD];
          tmem_ld_x32(lane_base + o_col, o);
          tmem_ld_x32(lane_base + o_col + 32, o + 32);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < HD; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st_x32(lane_base + o_col, o);
          tmem_st_x32(lane_base + o_col + 32, o + 32);
          tmem_st_wait();
        }
        tc_fence_before();  // P (and a rescaled O) in TMEM before the MMA warp reads it
        mbar_arrive(p_full + t);
        if (tr) trace(true, 512 * t + 8 * j + 4);
      }
      if (ok && nkv[t] > 0) ok = warp_wait(o_done + t, (uint32_t)(nkv[t] - 1) & 1, lane);
      if (ok) {
        tc_fence_after();
        uint32_t o[HD];
        tmem_ld_x32(lane_base + o_col, o);
        tmem_ld_x32(lane_base + o_col + 32, o + 32);
        tmem_ld_wait();
        const float inv = 1.f / l;
        __nv_bfloat16* yr = y + (size_t)(row0 + qrow) * C + h * HD;
#pragma unroll
        for (int ch = 0; ch < HD / 8; ++ch) {
          const float* f = reinterpret_cast<const float*>(o + ch * 8);
          uint4 pk;
          pk.x = pack_bf16(f[0] * inv, f[1] * inv);
          pk.y = pack_bf16(f[2] * inv, f[3] * inv);
          pk.z = pack_bf16(f[4] * inv, f[5] * inv);
          pk.w = pack_bf16(f[6] * inv, f[7] * inv);
          reinterpret_cast<uint4*>(yr)[ch] = pk;
        }
        lse[(size_t)bh * T + qrow] = (m + log2f(l)) * kLn2;
      } else if (lane == 0) {
        fail(err, &s_abort, 25u);
      }
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
// One CTA per (128-key block, batch, head), looping over the query blocks
// that see it. Every query block is processed as two halves of 64 queries
// ("half-steps"): the scores S^T and dP^T of a half go to one of two TMEM
// buffers, so the tensor cores compute the next halves' scores and the
// previous half's dV / dK updates while the softmax warps work on this one.
constexpr int G_K = 0, G_V = TILE, G_Q = 2 * TILE, G_DO = 4 * TILE;  // Q / dO: 2 stages each
constexpr int G_PT = 6 * TILE;                                        // P^T: one [128][64] tile per half buffer
constexpr int G_DST = 8 * TILE;                                       // dS^T of the query block: two [128][64] halves
constexpr int G_DQS = 10 * TILE;                                      // fp32 [128][64] dQ staging: 32 KB
constexpr int G_LSE = 12 * TILE, G_DEL = G_LSE + 1024;                // [2][128] fp32 each
constexpr int G_BAR = G_DEL + 1024;
constexpr int G_SMEM = G_BAR + 256 + 1024;
// Warp 0 TMA, 1 MMA, 2-3 idle, 4-11 softmax (warps 4-7: columns 0-31 of a
// half, 8-11: columns 32-63), 12-15 dQ drain. 128 registers per thread.
constexpr int G_THREADS = 512;
// TMEM columns: half buffers b at 128 b (S^T half: +0, dP^T half: +64), dV
// 256, dK 320, dQ buffers 384 / 448.
constexpr uint32_t T_SP = 0, T_DV = 256, T_DK = 320, T_DQ = 384;

__global__ void __launch_bounds__(G_THREADS, 1)
k_attn_bwd(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ CUtensorMap tm_do,
           const __grid_constant__ CUtensorMap tm_dq, const float* __restrict__ lse, const float* __restrict__ delta,
           __nv_bfloat16* __restrict__ dqkv, int B, int T, int H, int causal, float scale, unsigned int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + G_BAR);
  uint64_t* kv_full = bar;
  uint64_t* q_full = bar + 1;     // [2] Q, dO, lse, Delta of a query block
  uint64_t* q_empty = bar + 3;    // [2]
  uint64_t* sp_full = bar + 5;    // [2] per half buffer: S^T, dP^T complete
  uint64_t* sp_free = bar + 7;    // [2] per half buffer: read into registers
  uint64_t* pds_full = bar + 9;   // [2] per half buffer: P^T, dS^T in shared memory
  uint64_t* dq_full = bar + 11;   // [2]
  uint64_t* dq_empty = bar + 13;  // [2]
  uint64_t* dq_read = bar + 15;   // dQ of the query block done (dS^T half 0, P^T buffer 0 free)
  uint64_t* h1_read = bar + 16;   // second half's dV / dK done (dS^T half 1, P^T buffer 1 free)
  uint64_t* acc_full = bar + 17;
  uint64_t* mma_done = bar + 18;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 19);
  __shared__ volatile int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool tron = (int)blockIdx.x == g_trace_cta;
  const int nq = T / BQ;
  const int BH = B * H;
  const int kb = (int)(blockIdx.x / BH);  // key block; the earliest see the most query blocks
  const int bh = (int)(blockIdx.x % BH);
  const int b = bh / H, h = bh % H;
  const int C = H * HD;
  const int i0 = causal ? kb : 0;
  const int nsteps = nq - i0;
  const int U = 2 * nsteps;  // half-steps
  const int row0 = b * T;
  const float scale_log2 = scale * kLog2e;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(q_full + s, 1);
      mbar_init(q_empty + s, 1);
      mbar_init(sp_full + s, 1);
      mbar_init(sp_free + s, 256);
      mbar_init(pds_full + s, 256);
      mbar_init(dq_full + s, 1);
      mbar_init(dq_empty + s, 128);
    }
    mbar_init(dq_read, 1);
    mbar_init(h1_read, 1);
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
      // Descriptors computed once (see the forward kernel): K-major operands
      // advance 2 per K step of 16, MN-major ones 128; tiles TILE / 16 apart.
      constexpr uint32_t idS = umma_idesc_bf16_f32(BKV, 64);                 // S^T / dP^T half: N = 64 queries
      constexpr uint32_t idKV = umma_idesc_bf16_f32(BKV, HD, false, true);  // dV, dK: B MN-major
      constexpr uint32_t idQ = umma_idesc_bf16_f32(BQ, HD, true, true);     // dQ: A and B MN-major
      constexpr uint64_t kTileStep = TILE >> 4, kHalf = 8192 >> 4;
      const uint64_t dk = umma_desc_sw128_kmajor(smem_u32(smem + G_K));
      const uint64_t dv = umma_desc_sw128_kmajor(smem_u32(smem + G_V));
      const uint64_t dq0 = umma_desc_sw128_kmajor(smem_u32(smem + G_Q));
      const uint64_t ddo0 = umma_desc_sw128_kmajor(smem_u32(smem + G_DO));
      const uint64_t dqm0 = desc_mn(smem_u32(smem + G_Q), 8192);    // Q as an MN-major B operand
      const uint64_t ddom0 = desc_mn(smem_u32(smem + G_DO), 8192);  // dO as an MN-major B operand
      const uint64_t dpt = umma_desc_sw128_kmajor(smem_u32(smem + G_PT));
      const uint64_t dst = umma_desc_sw128_kmajor(smem_u32(smem + G_DST));
      const uint64_t dstm = desc_mn(smem_u32(smem + G_DST), TILE);   // dS^T as an MN-major A operand
      const uint64_t dkm = desc_mn(smem_u32(smem + G_K), 8192);      // K as an MN-major B operand
      // S^T and dP^T of half-step u into half buffer u & 1.
      auto issue_sp = [&](int u) -> bool {
        const int t = u >> 1, hh = u & 1, s = t & 1;
        if (!mbar_wait_bounded(q_full + s, (t >> 1) & 1, kWait)) return false;
        tc_fence_after();
        const uint64_t off = (uint64_t)s * kTileStep + (uint64_t)hh * kHalf;
        const uint64_t bq = dq0 + off, bdo = ddo0 + off;
        const uint32_t d = tbase + T_SP + (u & 1) * 128;
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) umma_f16(d, dk + 2 * k, bq + 2 * k, idS, k > 0 ? 1u : 0u);
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) umma_f16(d + 64, dv + 2 * k, bdo + 2 * k, idS, k > 0 ? 1u : 0u);
        umma_commit(sp_full + (u & 1));
        return true;
      };
      bool ok = mbar_wait_bounded(kv_full, 0, kWait);
      if (ok) {
        tc_fence_after();
        ok = issue_sp(0) && (U < 2 || issue_sp(1));
      }
      if (!ok) fail(err, &s_abort, 32u);
      for (int u = 0; ok && u < U && !s_abort; ++u) {
        const int t = u >> 1, hh = u & 1, s = t & 1, bf = u & 1;
        const uint32_t ph = (uint32_t)(u >> 1) & 1;
        // Next scores into this half buffer once the softmax has read it.
        if (u + 2 < U) {
          if (!mbar_wait_bounded(sp_free + bf, ph, kWait) || !issue_sp(u + 2)) {
            fail(err, &s_abort, 33u);
            break;
          }
        }
        trace(tron, 3072 + 4 * u);
        if (!mbar_wait_bounded(pds_full + bf, ph, kWait)) {
          fail(err, &s_abort, 34u);
          break;
        }
        trace(tron, 3072 + 4 * u + 1);
        tc_fence_after();
        if (hh == 1) {
          // dQ_i = dS K first (A = dS^T read MN-major, the two 64-query halves
          // TILE apart): the next block's softmax waits on it to reuse dS^T.
          if (t >= 2 && !mbar_wait_bounded(dq_empty + s, ((t >> 1) - 1) & 1, kWait)) {
            fail(err, &s_abort, 35u);
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int k = 0; k < BKV / 16; ++k)
            umma_f16(tbase + T_DQ + s * HD, dstm + 128 * k, dkm + 128 * k, idQ, k > 0 ? 1u : 0u);
          umma_commit(dq_full + s);
          umma_commit(dq_read);
        }
        // dV += P^T dO_half, dK += dS^T Q_half (K = 64 queries).
        const uint64_t off = (uint64_t)s * kTileStep + (uint64_t)hh * kHalf;
        const uint64_t a_pt = dpt + (uint64_t)bf * kTileStep, a_ds = dst + (uint64_t)hh * kTileStep;
        const uint64_t b_do = ddom0 + off, b_q = dqm0 + off;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_f16(tbase + T_DV, a_pt + 2 * k, b_do + 128 * k, idKV, (u > 0 || k > 0) ? 1u : 0u);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_f16(tbase + T_DK, a_ds + 2 * k, b_q + 128 * k, idKV, (u > 0 || k > 0) ? 1u : 0u);
        if (hh == 1) {
          umma_commit(h1_read);
          umma_commit(q_empty + s);
          trace(tron, 3072 + 4 * u + 2);
        }
      }
      if (ok && !s_abort) umma_commit(acc_full);
      umma_commit(mma_done);
      mbar_wait_bounded(mma_done, 0, kWait);
    }
  } else if (warp >= 4 && warp < 12) {
    // ---- P^T and dS^T: one key row per thread, 32 query columns of each half per warp
    const int wg = (warp >> 2) - 1;     // column group within a half
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // key row in the block = TMEM lane
    const uint32_t lane_base = tbase + ((uint32_t)(quarter * 32) << 16);
    const bool tr = tron && wg == 0 && r == 0;
    bool ok = true;
    for (int u = 0; u < U; ++u) {
      const int t = u >> 1, hh = u & 1, s = t & 1, bf = u & 1;
      const int i = i0 + t;
      if (!warp_wait(sp_full + bf, (uint32_t)(u >> 1) & 1, lane) ||
          (hh == 0 && !warp_wait(q_full + s, (uint32_t)(t >> 1) & 1, lane)) || s_abort) {
        ok = false;
        break;
      }
      if (tr) trace(true, 2048 + 4 * u);
      tc_fence_after();
      uint32_t sr[32], dr[32];
      tmem_ld_x32(lane_base + T_SP + bf * 128 + wg * 32, sr);
      tmem_ld_x32(lane_base + T_SP + bf * 128 + 64 + wg * 32, dr);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(sp_free + bf);
      if (tr) trace(true, 2048 + 4 * u + 1);
      // The previous query block's MMAs must be done with this half's P^T
      // buffer and dS^T half (its dQ for half 0, its second dV / dK for half 1).
      if (t >= 1 && !warp_wait(hh == 0 ? dq_read : h1_read, (uint32_t)(t - 1) & 1, lane)) {
        ok = false;
        break;
      }
      if (tr) trace(true, 2048 + 4 * u + 2);
      const int cbase = hh * 64 + wg * 32;  // first query column of this thread's 32
      const float* lse_s = reinterpret_cast<const float*>(smem + G_LSE + s * 512) + cbase;
      const float* del_s = reinterpret_cast<const float*>(smem + G_DEL + s * 512) + cbase;
      const bool diag = causal && i == kb;
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) {
        const float4 l0 = reinterpret_cast<const float4*>(lse_s)[2 * ch];
        const float4 l1 = reinterpret_cast<const float4*>(lse_s)[2 * ch + 1];
        const float4 d0 = reinterpret_cast<const float4*>(del_s)[2 * ch];
        const float4 d1 = reinterpret_cast<const float4*>(del_s)[2 * ch + 1];
        const float lv[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
        const float dv[8] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
        float p[8], ds[8];
        // p = 2^(s * scale * log2e - lse * log2e), dS = p (dP - Delta), in packed pairs.
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
          const int c = ch * 8 + e;
          float n0, n1;
          fmul2(n0, n1, lv[e], lv[e + 1], -kLog2e, -kLog2e);
          ffma2(p[e], p[e + 1], __uint_as_float(sr[c]), __uint_as_float(sr[c + 1]), scale_log2, scale_log2, n0, n1);
          fadd2(ds[e], ds[e + 1], __uint_as_float(dr[c]), __uint_as_float(dr[c + 1]), -dv[e], -dv[e + 1]);
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          float pv = ex2(p[e]);
          if (diag && cbase + ch * 8 + e < r) pv = 0.f;  // key r is later than query cbase + c
          p[e] = pv;
        }
#pragma unroll
        for (int e = 0; e < 8; e += 2) fmul2(ds[e], ds[e + 1], ds[e], ds[e + 1], p[e], p[e + 1]);
        uint4 pk, dk;
        pk.x = pack_bf16(p[0], p[1]);
        pk.y = pack_bf16(p[2], p[3]);
        pk.z = pack_bf16(p[4], p[5]);
        pk.w = pack_bf16(p[6], p[7]);
        dk.x = pack_bf16(ds[0], ds[1]);
        dk.y = pack_bf16(ds[2], ds[3]);
        dk.z = pack_bf16(ds[4], ds[5]);
        dk.w = pack_bf16(ds[6], ds[7]);
        *reinterpret_cast<uint4*>(smem + G_PT + bf * TILE + sw128(r, wg * 4 + ch)) = pk;
        *reinterpret_cast<uint4*>(smem + G_DST + hh * TILE + sw128(r, wg * 4 + ch)) = dk;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(pds_full + bf);
      if (tr) trace(true, 2048 + 4 * u + 3);
    }
    // dV (warps 4-7) and dK (warps 8-11) out of TMEM once every step is accumulated.
    if (ok && warp_wait(acc_full, 0, lane)) {
      tc_fence_after();
      const float sc = wg == 0 ? 1.f : scale;
      const size_t row = (size_t)(row0 + kb * BKV + r) * (3 * C);
      uint4* g = reinterpret_cast<uint4*>(dqkv + row + (wg == 0 ? 2 * C : C) + h * HD);
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t a[32];
        tmem_ld_x32(lane_base + (wg == 0 ? T_DV : T_DK) + half * 32, a);
        tmem_ld_wait();
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {
          const float* f = reinterpret_cast<const float*>(a + ch * 8);
          uint4 pk;
          pk.x = pack_bf16(f[0] * sc, f[1] * sc);
          pk.y = pack_bf16(f[2] * sc, f[3] * sc);
          pk.z = pack_bf16(f[4] * sc, f[5] * sc);
          pk.w = pack_bf16(f[6] * sc, f[7] * sc);
          g[half * 4 + ch] = pk;
        }
      }
    } else if (lane == 0) {
      fail(err, &s_abort, 36u);
    }
  } else if (warp >= 12) {
    // ---- dQ_i: TMEM -> swizzled shared staging -> tensor bulk fp32 adds into the accumulator
    const int quarter = warp & 3;
    const int rq = quarter * 32 + lane;  // query row in the block = TMEM lane
    const uint32_t lane_base = tbase + ((uint32_t)(quarter * 32) << 16);
    const bool issuer = (warp == 12 && lane == 0);
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

// Delta[b, h, t] = sum_d dO[b*T + t, h*64 + d] * O[b*T + t, h*64 + d] (fp32),
// and the fp32 dQ accumulator row [b, h, t, :] cleared (one launch for both).
__global__ void k_attn_prep(const __nv_bfloat16* __restrict__ y, const __nv_bfloat16* __restrict__ dy,
                            float* __restrict__ delta, float* __restrict__ dq_acc, int BT, int T, int H) {
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
  const size_t rh = ((size_t)bb * H + h) * T + t;
  delta[rh] = acc;
  float4* z = reinterpret_cast<float4*>(dq_acc + rh * HD);
#pragma unroll
  for (int k = 0; k < HD / 4; ++k) z[k] = make_float4(0.f, 0.f, 0.f, 0.f);
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
cudaError_t attention_trace_select(int cta) {
  cudaError_t e = cudaMemcpyToSymbol(attn::g_trace_cta, &cta, sizeof(int));
  if (e != cudaSuccess) return e;
  static const unsigned long long zeros[attn::kTraceSlots] = {};
  return cudaMemcpyToSymbol(attn::g_trace, zeros, sizeof(zeros));
}

cudaError_t attention_trace_read(unsigned long long* host, int n) {
  if (n > attn::kTraceSlots) n = attn::kTraceSlots;
  return cudaMemcpyFromSymbol(host, attn::g_trace, (size_t)n * sizeof(unsigned long long));
}

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
  const unsigned grid = (unsigned)(((T / BQ + 1) / 2) * B * H);
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
  const long long rows = (long long)B * T * H;
  k_attn_prep<<<(unsigned)((rows + 255) / 256), 256, 0, s>>>(y, dy, delta, dq_acc, B * T, T, H);
  const float scale = 1.f / sqrtf((float)HD);
  const unsigned grid = (unsigned)((T / BKV) * B * H);
  k_attn_bwd<<<grid, G_THREADS, G_SMEM, s>>>(tq, tdo, tdq, lse, delta, dqkv, B, T, H, causal ? 1 : 0, scale,
                                              gemm_err_word());
  const long long chunks = (long long)B * H * T * (HD / 8);
  k_attn_dq_out<<<(unsigned)((chunks + 255) / 256), 256, 0, s>>>(dq_acc, dqkv, B, T, H, scale);
  return cudaGetLastError();
}

}  // namespace nexar
