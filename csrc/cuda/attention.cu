// Self-attention for head dimension 64 on tcgen05 (sm_100a): forward and
// backward, causal or full, bf16 in / out, fp32 softmax statistics.
//
// Layout (the GPT-2 block): qkv is the row-major [B*T, 3C] output of the QKV
// projection (C = H * 64; columns [0, C) are Q, [C, 2C) K, [2C, 3C) V, head h
// at h*64), y the [B*T, C] attention output, lse the [B, H, T] natural-log
// softmax normaliser of every query row (scores scaled by 1/sqrt(64)).
//
// Forward (k_attn_fwd): one CTA per (128-query tile, batch, head), two CTAs
// resident per SM (256 TMEM columns, 192 threads each), longest tiles first.
//   warp 0      TMA loads: the Q tile once, then K and V tiles of 128 keys
//               into two 2-deep rings (K_j is released when S_j completes,
//               V_j when O += P_j V_j does; every load reads this GPU's
//               memory, no multicast);
//   warp 1      allocates the TMEM columns; lane 0 issues S = Q K_j^T
//               (M = N = 128, K = 64) for the next key block as soon as the
//               softmax holds the current scores, and O += P V_j (M = 128,
//               N = 64, K = 128, P read from TMEM) once P is written; O
//               accumulates in TMEM;
//   warps 2-5   softmax, one query row per thread (TMEM lane = row, lane
//               quarter = warp % 4), in the exp2 domain. The running maximum
//               is raised lazily (only when a block's maximum exceeds it by
//               more than 2^8), so the accumulated output is rescaled in TMEM
//               only on those blocks. A quarter of the exponentials run on
//               the FMA pipe (exp2_poly2), the rest on the MUFU unit. P goes
//               to TMEM as packed bf16 (tcgen05.st), where the next MMA reads
//               it as its A operand.
//   The two resident CTAs overlap: one computes exponentials while the
//   tensor cores run the other's MMAs, and one's start (barrier setup, first
//   loads) hides behind the other's work.
// Backward (k_attn_bwd): persistent, one CTA per SM walking (128-key block,
// batch, head) items in snake order of decreasing length; each item loops
// over the query blocks that see its key block, each as two halves of 64
// queries.
//   warp 0      K_j, V_j per item (2 slots: the next item's load overlaps
//               this one); Q_i, dO_i, lse_i, Delta_i per block (2-deep);
//   warp 1      S^T = K Q_half^T and dP^T = V dO_half^T (M = 128, N = 64,
//               K = 64) into one of two TMEM half buffers; dV += P^T dO_half
//               and dK += dS^T Q_half (K = 64, A read from TMEM, accumulated
//               over all steps), then the next scores of the same buffer;
//               after both halves dQ_i = dS K (M = 128, N = 64, K = 128) into
//               one of two TMEM buffers;
//   warps 4-11  one key row per thread, 32 query columns of a half per warp:
//               P^T = exp(S^T * scale - lse), dS^T = P^T (dP^T - Delta), both
//               packed bf16 back into TMEM over the scores just read, dS^T
//               also into swizzled shared memory (two stages: the MN-major A
//               operand of dQ); at the end dV (warps 4-7) and dK (warps 8-11)
//               from TMEM to dqkv;
//   warps 12-15 drain dQ_i from TMEM through a swizzled 128 x 32 fp32
//               staging box into the fp32 dQ accumulator with two tensor bulk
//               reductions (cp.reduce.async.bulk.tensor .add) per query block.
// k_attn_prep computes Delta = rowsum(dO * O) (a memset clears the dQ accumulator);
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
int gemm_sm_count();

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

// Bounded wait that polls with test_wait. The waits of these pipelines sit
// on their critical path, and a thread suspended in try_wait was measured to
// resume hundreds of cycles after the phase completed; polling costs one
// issue slot per probe of the one thread (or warp) that waits.
NEXAR_D bool mbar_spin(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
  if (mbar_test(bar, parity)) return true;
  uint64_t t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 256; ++i)
      if (mbar_test(bar, parity)) return true;
    uint64_t t1;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t1));
    if (t1 - t0 > limit_ns) return false;
  }
}

// Bounded wait by lane 0 of a warp; every lane then observes the completed
// phase itself (acquire) before touching the data the phase publishes.
NEXAR_D bool warp_wait(uint64_t* bar, uint32_t parity, int lane) {
  // Fast path: one warp-wide test (the phase is usually complete already).
  if (mbar_test(bar, parity)) return true;
  int ok = 1;
  if (lane == 0) ok = mbar_spin(bar, parity, kWait) ? 1 : 0;
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
// softmax at 8 j + k, forward MMA at 1024 + 8 j + k (k = 0: next S issued,
// 1: P V issued, 2: S read, 3: P written), forward loads at 1536 + j;
// backward softmax at 2048 + 4 u + k, backward MMA at 3072 + 4 u + k (u
// counts half-steps over the CTA's items; k = 0: step start, 1: P^T / dS^T
// written, 2: dQ / dV / dK issued, 3: the next scores issued).
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
NEXAR_D void tmem_st_x16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
      :: "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
         "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
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
// One CTA per 128-query tile of one (batch, head), two CTAs resident per SM:
// while one CTA's softmax computes exponentials the tensor cores run the
// other's MMAs, and one CTA's start (barrier setup, first loads) overlaps
// the other's work. The tiles are scheduled longest first (most key blocks).
constexpr int F_STAGES = 2;                  // K ring and V ring, released separately
constexpr int F_Q = 0;
constexpr int F_K = TILE;                    // K ring
constexpr int F_V = F_K + F_STAGES * TILE;   // V ring
constexpr int F_BAR = F_V + F_STAGES * TILE;
constexpr int F_SMEM = F_BAR + 128 + 1024;
// Warp 0 TMA, warp 1 TMEM allocation + MMA issue, warps 2-5 softmax (TMEM
// lane quarter = warp % 4). 2 x 192 threads x 168 registers fit the SM.
constexpr int F_THREADS = 192;
// TMEM columns (256 per CTA, two CTAs per SM): S 0 (fp32 scores), O 128
// (fp32 output accumulator), P 192 (bf16 probabilities, two per column: the
// A operand of O += P V, read by the tensor cores straight from TMEM).
constexpr uint32_t T_S = 0, T_O = 128, T_P = 192;
constexpr uint32_t F_TMEM_COLS = 256;
// The running maximum is raised only when a block's maximum exceeds it by
// more than 2^8: between raises the probabilities stay below 256 (exact in
// fp32, ample range in bf16) and the output accumulator needs no rescaling.
constexpr float kRescaleLog2 = 8.f;

__global__ void __launch_bounds__(F_THREADS, 2)
k_attn_fwd(const __grid_constant__ CUtensorMap tm_qkv, __nv_bfloat16* __restrict__ y, float* __restrict__ lse, int B,
           int T, int H, int causal, float scale_log2, unsigned int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + F_BAR);
  uint64_t* q_full = bar;
  uint64_t* k_full = bar + 1;                // [F_STAGES]
  uint64_t* v_full = bar + 1 + F_STAGES;     // [F_STAGES]
  uint64_t* k_empty = bar + 1 + 2 * F_STAGES;
  uint64_t* v_empty = bar + 1 + 3 * F_STAGES;
  uint64_t* s_full = bar + 1 + 4 * F_STAGES;  // S = Q K^T complete
  uint64_t* s_free = s_full + 1;              // S read into registers
  uint64_t* p_full = s_full + 2;              // P in TMEM, O rescaled
  uint64_t* o_done = s_full + 3;              // O += P V complete
  uint64_t* mma_done = s_full + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_full + 5);
  __shared__ volatile int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool tron = (int)blockIdx.x == g_trace_cta;
  const int nq = T / BQ;
  const int BH = B * H;
  const int qt = nq - 1 - (int)(blockIdx.x / BH);  // most key blocks first (causal)
  const int bh = (int)(blockIdx.x % BH);
  const int b = bh / H, h = bh % H;
  const int C = H * HD;
  const int row0 = b * T;
  const int nkv = causal ? qt + 1 : nq;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < F_STAGES; ++s) {
      mbar_init(k_full + s, 1);
      mbar_init(v_full + s, 1);
      mbar_init(k_empty + s, 1);
      mbar_init(v_empty + s, 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 128);
    mbar_init(p_full, 128);
    mbar_init(o_done, 1);
    mbar_init(mma_done, 1);
    s_abort = 0;
    mbar_fence_init();
    tma_prefetch_desc(&tm_qkv);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, F_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, TILE);
      tma_load_2d(smem + F_Q, &tm_qkv, q_full, h * HD, row0 + qt * BQ);
      // K_j may load once S_{j-2} has completed, V_j once O += P_{j-2} V_{j-2} has.
      int issued = 0;
      for (int j = 0; j < nkv && !s_abort; ++j) {
        const int st = j % F_STAGES;
        const uint32_t ph = ((j / F_STAGES) - 1) & 1;
        if (j >= F_STAGES && !mbar_spin(k_empty + st, ph, kWait)) {
          fail(err, &s_abort, 21u);
          break;
        }
        mbar_arrive_expect_tx(k_full + st, TILE);
        tma_load_2d(smem + F_K + st * TILE, &tm_qkv, k_full + st, C + h * HD, row0 + j * BKV);
        if (j >= F_STAGES && !mbar_spin(v_empty + st, ph, kWait)) {
          fail(err, &s_abort, 21u);
          issued = -(j + 1);  // K_j was issued, V_j was not
          break;
        }
        mbar_arrive_expect_tx(v_full + st, TILE);
        tma_load_2d(smem + F_V + st * TILE, &tm_qkv, v_full + st, 2 * C + h * HD, row0 + j * BKV);
        trace(tron, 1536 + j);
        issued = j + 1;
      }
      // No TMA write may still be landing when the CTA exits.
      mbar_wait_bounded(q_full, 0, kWait >> 4);
      const int nk = issued < 0 ? -issued : issued, nv = issued < 0 ? -issued - 1 : issued;
      for (int j = nk > F_STAGES ? nk - F_STAGES : 0; j < nk; ++j)
        mbar_wait_bounded(k_full + j % F_STAGES, (j / F_STAGES) & 1, kWait >> 4);
      for (int j = nv > F_STAGES ? nv - F_STAGES : 0; j < nv; ++j)
        mbar_wait_bounded(v_full + j % F_STAGES, (j / F_STAGES) & 1, kWait >> 4);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // Descriptors are computed once: a K step of 16 elements advances a
      // K-major operand by 32 bytes (start-address field + 2) and an
      // MN-major one by 16 rows of 128 bytes (+ 128); stages are TILE bytes
      // apart (+ TILE / 16).
      constexpr uint32_t idS = umma_idesc_bf16_f32(BQ, BKV);
      constexpr uint32_t idO = umma_idesc_bf16_f32(BQ, HD, false, true);
      constexpr uint64_t kTileStep = TILE >> 4;
      const uint64_t dq = umma_desc_sw128_kmajor(smem_u32(smem + F_Q));
      const uint64_t dk0 = umma_desc_sw128_kmajor(smem_u32(smem + F_K));
      const uint64_t dv0 = desc_mn(smem_u32(smem + F_V), 8192);
      const uint32_t d_s = tbase + T_S, d_o = tbase + T_O, pa = tbase + T_P;
      auto issue_s = [&](int j) {
        const uint64_t db = dk0 + (uint64_t)(j % F_STAGES) * kTileStep;
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) umma_f16(d_s, dq + 2 * k, db + 2 * k, idS, k > 0 ? 1u : 0u);
        umma_commit(s_full);
        umma_commit(k_empty + j % F_STAGES);
      };
      bool ok = mbar_spin(q_full, 0, kWait) && mbar_spin(k_full, 0, kWait);
      if (ok) {
        tc_fence_after();
        issue_s(0);
      } else {
        fail(err, &s_abort, 22u);
      }
      for (int j = 0; ok && j < nkv && !s_abort; ++j) {
        // The next scores as soon as the softmax holds the current ones.
        if (j + 1 < nkv) {
          if (!mbar_spin(s_free, j & 1, kWait) ||
              !mbar_spin(k_full + (j + 1) % F_STAGES, ((j + 1) / F_STAGES) & 1, kWait)) {
            fail(err, &s_abort, 23u);
            break;
          }
          trace(tron, 1024 + 8 * j + 2);
          tc_fence_after();
          issue_s(j + 1);
          trace(tron, 1024 + 8 * j);
        }
        // O += P V_j (P read from TMEM) once the softmax has written P.
        if (!mbar_spin(p_full, j & 1, kWait) ||
            !mbar_spin(v_full + j % F_STAGES, (j / F_STAGES) & 1, kWait)) {
          fail(err, &s_abort, 24u);
          break;
        }
        trace(tron, 1024 + 8 * j + 3);
        tc_fence_after();
        const uint64_t db = dv0 + (uint64_t)(j % F_STAGES) * kTileStep;
#pragma unroll
        for (int k = 0; k < BKV / 16; ++k)  // K step of 16 = 8 TMEM columns of packed P
          umma_f16_ts(d_o, pa + 8 * k, db + 128 * k, idO, (j > 0 || k > 0) ? 1u : 0u);
        umma_commit(o_done);
        umma_commit(v_empty + j % F_STAGES);
        trace(tron, 1024 + 8 * j + 1);
      }
      // Every issued MMA has finished before TMEM is released.
      umma_commit(mma_done);
      mbar_spin(mma_done, 0, kWait);
    }
  } else {
    const int quarter = warp & 3;         // TMEM lane quarter of this warp
    const int r = quarter * 32 + lane;    // query row in the tile = TMEM lane
    const uint32_t lane_base = tbase + ((uint32_t)(quarter * 32) << 16);
    const int qrow = qt * BQ + r;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    const bool tr = tron && r == 0;
    for (int j = 0; j < nkv; ++j) {
      if (!warp_wait(s_full, (uint32_t)j & 1, lane) || s_abort) {
        ok = false;
        break;
      }
      if (tr) trace(true, 8 * j);
      tc_fence_after();
      uint32_t x[BKV];
#pragma unroll
      for (int c0 = 0; c0 < BKV; c0 += 32) tmem_ld_x32(lane_base + T_S + c0, x + c0);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(s_free);
      if (tr) trace(true, 8 * j + 1);
      if (causal && j == qt) {
#pragma unroll
        for (int c = 0; c < BKV; ++c)
          if (c > r) x[c] = __float_as_uint(-INFINITY);
      }
      // Row maximum: x[0..3] seed four chains, 15 steps of 8 cover x[4..123],
      // x[124..127] close them (no read past the 128 scores).
      float mx0 = __uint_as_float(x[0]), mx1 = __uint_as_float(x[1]);
      float mx2 = __uint_as_float(x[2]), mx3 = __uint_as_float(x[3]);
#pragma unroll
      for (int c = 4; c < BKV - 4; c += 8) {
        mx0 = fmax3(mx0, __uint_as_float(x[c + 0]), __uint_as_float(x[c + 1]));
        mx1 = fmax3(mx1, __uint_as_float(x[c + 2]), __uint_as_float(x[c + 3]));
        mx2 = fmax3(mx2, __uint_as_float(x[c + 4]), __uint_as_float(x[c + 5]));
        mx3 = fmax3(mx3, __uint_as_float(x[c + 6]), __uint_as_float(x[c + 7]));
      }
      mx0 = fmaxf(mx0, __uint_as_float(x[BKV - 4]));
      mx1 = fmaxf(mx1, __uint_as_float(x[BKV - 3]));
      mx2 = fmaxf(mx2, __uint_as_float(x[BKV - 2]));
      mx3 = fmaxf(mx3, __uint_as_float(x[BKV - 1]));
      const float m_blk = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * scale_log2;
      const bool raise = m_blk > m + kRescaleLog2;
      const float m_new = raise ? m_blk : m;
      const float alpha = raise ? ex2(m - m_new) : 1.f;
      if (tr) trace(true, 8 * j + 2);
      if (j >= 1) {
        // P (TMEM) and O are free once O += P_{j-1} V_{j-1} has completed.
        if (!warp_wait(o_done, (uint32_t)(j - 1) & 1, lane)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      if (tr) trace(true, 8 * j + 3);
      // Probabilities into the row's P columns of TMEM, 32 columns (64
      // values) at a time: 6 of every 8 exponentials on the MUFU unit, 2 on
      // the FMA pipe (exp2_poly2); 4 + 4 measured slower (44.4 against
      // 41.5 us per GPT-2 layer).
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
        if ((ch & 7) == 7) tmem_st_x32(lane_base + T_P + (ch >> 3) * 32, pk);
      }
      tmem_st_wait();
      l = l * alpha + (sum0 + sum1);
      m = m_new;
      if (j >= 1 && __any_sync(0xffffffffu, raise)) {
        // The maximum rose: scale the accumulated output to it before P_j V_j is added.
        uint32_t o[HD];
        tmem_ld_x32(lane_base + T_O, o);
        tmem_ld_x32(lane_base + T_O + 32, o + 32);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < HD; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
        tmem_st_x32(lane_base + T_O, o);
        tmem_st_x32(lane_base + T_O + 32, o + 32);
        tmem_st_wait();
      }
      tc_fence_before();  // P (and a rescaled O) in TMEM before the MMA warp reads it
      mbar_arrive(p_full);
      if (tr) trace(true, 8 * j + 4);
    }
    if (ok && nkv > 0) ok = warp_wait(o_done, (uint32_t)(nkv - 1) & 1, lane);
    if (ok) {
      tc_fence_after();
      uint32_t o[HD];
      tmem_ld_x32(lane_base + T_O, o);
      tmem_ld_x32(lane_base + T_O + 32, o + 32);
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
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, F_TMEM_COLS);
  }
}

// ============================================================ backward
// Persistent: one CTA per SM walks a list of (128-key block, batch, head)
// items, each looping over the query blocks that see its key block. The
// items are dealt in snake order of decreasing length (row r of the deal
// goes to CTAs 0..P-1, row r + 1 to P-1..0), which balances the causal work
// to within one query block per SM. K and V are double-buffered across
// items, so the next item's scores start while this item's dV / dK drain.
// Every query block is processed as two halves of 64 queries ("half-steps"):
// the scores S^T and dP^T of a half go to one of two TMEM buffers, so the
// tensor cores compute the next halves' scores and the previous half's
// dV / dK updates while the softmax warps work on this one.
constexpr int G_KV = 0;                      // [slot][K, V]: 2 slots of two tiles
constexpr int G_Q = 4 * TILE, G_DO = 6 * TILE;  // Q / dO: 2 stages each
constexpr int G_DST = 8 * TILE;  // dS^T of a query block, two stages: [stage][half] [128 keys][64 queries]
constexpr int G_DQS = 12 * TILE;                                      // fp32 [128][32] dQ staging box: 16 KB
constexpr int G_LSE = 13 * TILE, G_DEL = G_LSE + 1024;                // [2][128] fp32 each
constexpr int G_BAR = G_DEL + 1024;
constexpr int G_SMEM = G_BAR + 256 + 1024;
// Warp 0 TMA, 1 MMA, 2-3 idle, 4-11 softmax (warps 4-7: columns 0-31 of a
// half, 8-11: columns 32-63), 12-15 dQ drain. 128 registers per thread.
constexpr int G_THREADS = 512;
// TMEM columns: half buffers b at 128 b (S^T half: +0, dP^T half: +64), dV
// 256, dK 320, dQ buffers 384 / 448. The softmax warps write P^T and dS^T
// (packed bf16) back over the scores they have read: warp group g's 32
// query columns of S^T (dP^T) become 16 columns of P^T (dS^T) at +32 g, the
// A operands of the dV and dK MMAs. The next scores overwrite the buffer only
// after those MMAs: tcgen05.mma operations issued by one thread run in order.
constexpr uint32_t T_SP = 0, T_DV = 256, T_DK = 320, T_DQ = 384;

// Item k of CTA c (of P) in the snake deal: its position in the list of
// items ordered by decreasing length, or -1 past the end.
NEXAR_D int bwd_item(int k, int c, int P, int nitems) {
  const int pos = k * P + ((k & 1) ? P - 1 - c : c);
  return pos < nitems ? pos : -1;
}

__global__ void __launch_bounds__(G_THREADS, 1)
k_attn_bwd(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ CUtensorMap tm_do,
           const __grid_constant__ CUtensorMap tm_dq, const float* __restrict__ lse, const float* __restrict__ delta,
           __nv_bfloat16* __restrict__ dqkv, int B, int T, int H, int causal, float scale, unsigned int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + G_BAR);
  uint64_t* kv_full = bar;        // [2] per K / V slot
  uint64_t* kv_empty = bar + 2;   // [2]
  uint64_t* q_full = bar + 4;     // [2] Q, dO, lse, Delta of a query block
  uint64_t* q_empty = bar + 6;    // [2]
  uint64_t* sp_full = bar + 8;    // [2] per half buffer: S^T, dP^T complete
  uint64_t* pds_full = bar + 10;  // [2] per half buffer: P^T, dS^T in TMEM (dS^T also in shared memory)
  uint64_t* dq_full = bar + 12;   // [2]
  uint64_t* dq_empty = bar + 14;  // [2]
  uint64_t* dq_read = bar + 16;   // [2] dQ of a query block done: its dS^T stage is free
  uint64_t* acc_full = bar + 18;  // an item's dV / dK complete
  uint64_t* acc_empty = bar + 19; // an item's dV / dK drained from TMEM
  uint64_t* mma_done = bar + 20;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 21);
  __shared__ volatile int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool tron = (int)blockIdx.x == g_trace_cta;
  const int nq = T / BQ;
  const int BH = B * H;
  const int nitems = nq * BH;
  const int P = (int)gridDim.x, cta = (int)blockIdx.x;
  const int C = H * HD;
  const float scale_log2 = scale * kLog2e;
  // Item at list position `pos`: key block (the earliest see the most query
  // blocks), batch-head, first query block and number of query blocks.
  auto item = [&](int pos, int& kb, int& bh, int& i0, int& nsteps) {
    kb = pos / BH;
    bh = pos % BH;
    i0 = causal ? kb : 0;
    nsteps = nq - i0;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(kv_full + s, 1);
      mbar_init(kv_empty + s, 1);
      mbar_init(q_full + s, 1);
      mbar_init(q_empty + s, 1);
      mbar_init(sp_full + s, 1);
      mbar_init(pds_full + s, 256);
      mbar_init(dq_full + s, 1);
      mbar_init(dq_empty + s, 128);
      mbar_init(dq_read + s, 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 256);
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
      // Runs ahead of the MMAs by up to one item (K / V) and two query
      // blocks (Q, dO, lse, Delta); gt counts query blocks over all items.
      int gt = 0, it = 0;
      bool ok = true;
      for (int pos; ok && (pos = bwd_item(it, cta, P, nitems)) >= 0 && !s_abort; ++it) {
        int kb, bh, i0, nsteps;
        item(pos, kb, bh, i0, nsteps);
        const int row0 = (bh / H) * T, h = bh % H, ks = it & 1;
        if (it >= 2 && !mbar_spin(kv_empty + ks, ((it >> 1) - 1) & 1, kWait)) {
          fail(err, &s_abort, 31u);
          break;
        }
        mbar_arrive_expect_tx(kv_full + ks, 2 * TILE);
        tma_load_2d(smem + G_KV + ks * 2 * TILE, &tm_qkv, kv_full + ks, C + h * HD, row0 + kb * BKV);
        tma_load_2d(smem + G_KV + ks * 2 * TILE + TILE, &tm_qkv, kv_full + ks, 2 * C + h * HD, row0 + kb * BKV);
        for (int t = 0; t < nsteps; ++t, ++gt) {
          const int i = i0 + t, s = gt & 1;
          if (gt >= 2 && !mbar_spin(q_empty + s, ((gt >> 1) - 1) & 1, kWait)) {
            fail(err, &s_abort, 31u);
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(q_full + s, 2 * TILE + 2 * 512);
          tma_load_2d(smem + G_Q + s * TILE, &tm_qkv, q_full + s, h * HD, row0 + i * BQ);
          tma_load_2d(smem + G_DO + s * TILE, &tm_do, q_full + s, h * HD, row0 + i * BQ);
          bulk_load(smem + G_LSE + s * 512, lse + (size_t)bh * T + i * BQ, 512, q_full + s);
          bulk_load(smem + G_DEL + s * 512, delta + (size_t)bh * T + i * BQ, 512, q_full + s);
        }
      }
      // No TMA write may still be landing when the CTA exits: wait for the
      // last two K / V loads and the last two query blocks issued.
      for (int k = it > 2 ? it - 2 : 0; k < it; ++k)
        mbar_wait_bounded(kv_full + (k & 1), (k >> 1) & 1, kWait >> 4);
      for (int k = gt > 2 ? gt - 2 : 0; k < gt; ++k)
        mbar_wait_bounded(q_full + (k & 1), (k >> 1) & 1, kWait >> 4);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // K-major operands advance 2 per K step of 16, MN-major ones 128;
      // tiles TILE / 16 apart.
      constexpr uint32_t idS = umma_idesc_bf16_f32(BKV, 64);                 // S^T / dP^T half: N = 64 queries
      constexpr uint32_t idKV = umma_idesc_bf16_f32(BKV, HD, false, true);  // dV, dK: B MN-major
      constexpr uint32_t idQ = umma_idesc_bf16_f32(BQ, HD, true, true);     // dQ: A and B MN-major
      constexpr uint64_t kTileStep = TILE >> 4, kHalf = 8192 >> 4;
      const uint64_t dk0 = umma_desc_sw128_kmajor(smem_u32(smem + G_KV));
      const uint64_t dkm0 = desc_mn(smem_u32(smem + G_KV), 8192);     // K as an MN-major B operand
      const uint64_t dq0 = umma_desc_sw128_kmajor(smem_u32(smem + G_Q));
      const uint64_t ddo0 = umma_desc_sw128_kmajor(smem_u32(smem + G_DO));
      const uint64_t dqm0 = desc_mn(smem_u32(smem + G_Q), 8192);    // Q as an MN-major B operand
      const uint64_t ddom0 = desc_mn(smem_u32(smem + G_DO), 8192);  // dO as an MN-major B operand
      const uint64_t dstm = desc_mn(smem_u32(smem + G_DST), TILE);  // dS^T as an MN-major A operand
      int gt = 0, it = 0;
      bool ok = true;
      for (int pos; ok && (pos = bwd_item(it, cta, P, nitems)) >= 0 && !s_abort; ++it) {
        int kb, bh, i0, nsteps;
        item(pos, kb, bh, i0, nsteps);
        const int ks = it & 1, U = 2 * nsteps;
        const uint64_t dk = dk0 + (uint64_t)ks * 2 * kTileStep, dv = dk + kTileStep;
        const uint64_t dkm = dkm0 + (uint64_t)ks * 2 * kTileStep;
        // S^T and dP^T of this item's half-step u into half buffer (2 gt + u) & 1.
        auto issue_sp = [&](int u) -> bool {
          const int tb = gt + (u >> 1), hh = u & 1, s = tb & 1;
          if (!mbar_spin(q_full + s, (tb >> 1) & 1, kWait)) return false;
          tc_fence_after();
          const uint64_t off = (uint64_t)s * kTileStep + (uint64_t)hh * kHalf;
          const uint64_t bq = dq0 + off, bdo = ddo0 + off;
          const int bf = u & 1;  // (2 gt + u) & 1
          const uint32_t d = tbase + T_SP + bf * 128;
#pragma unroll
          for (int k = 0; k < HD / 16; ++k) umma_f16(d, dk + 2 * k, bq + 2 * k, idS, k > 0 ? 1u : 0u);
#pragma unroll
          for (int k = 0; k < HD / 16; ++k) umma_f16(d + 64, dv + 2 * k, bdo + 2 * k, idS, k > 0 ? 1u : 0u);
          umma_commit(sp_full + bf);
          return true;
        };
        ok = mbar_spin(kv_full + ks, (it >> 1) & 1, kWait);
        if (ok) {
          tc_fence_after();
          ok = issue_sp(0) && (U < 2 || issue_sp(1));
        }
        if (!ok) {
          fail(err, &s_abort, 32u);
          break;
        }
        for (int u = 0; u < U; ++u) {
          const int gu = 2 * gt + u, tb = gt + (u >> 1), hh = u & 1, s = tb & 1, bf = gu & 1;
          trace(tron, 3072 + 4 * gu);
          if (!mbar_spin(pds_full + bf, (uint32_t)(gu >> 1) & 1, kWait)) {
            fail(err, &s_abort, 34u);
            ok = false;
            break;
          }
          trace(tron, 3072 + 4 * gu + 1);
          tc_fence_after();
          if (hh == 1) {
            // dQ_i = dS K (A = dS^T of both halves, read MN-major from shared
            // memory; the halves are TILE apart) into dQ buffer s once the
            // drain warps have emptied it.
            if (tb >= 2 && !mbar_spin(dq_empty + s, ((tb >> 1) - 1) & 1, kWait)) {
              fail(err, &s_abort, 35u);
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t a_ds = dstm + (uint64_t)s * 2 * kTileStep;
#pragma unroll
            for (int k = 0; k < BKV / 16; ++k)
              umma_f16(tbase + T_DQ + s * HD, a_ds + 128 * k, dkm + 128 * k, idQ, k > 0 ? 1u : 0u);
            umma_commit(dq_full + s);
            umma_commit(dq_read + s);
          }
          // The previous item's dV / dK must have left TMEM before this
          // item's first update overwrites them.
          if (u == 0 && it >= 1) {
            if (!mbar_spin(acc_empty, (uint32_t)(it - 1) & 1, kWait)) {
              fail(err, &s_abort, 37u);
              ok = false;
              break;
            }
            tc_fence_after();
          }
          // dV += P^T dO_half, dK += dS^T Q_half (K = 64 queries), A from TMEM:
          // K step k (queries 16k .. 16k + 15) sits at column 32 (k / 2) + 8 (k % 2).
          const uint64_t off = (uint64_t)s * kTileStep + (uint64_t)hh * kHalf;
          const uint64_t b_do = ddom0 + off, b_q = dqm0 + off;
          const uint32_t a_p = tbase + T_SP + bf * 128;
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_f16_ts(tbase + T_DV, a_p + 32 * (k >> 1) + 8 * (k & 1), b_do + 128 * k, idKV,
                        (u > 0 || k > 0) ? 1u : 0u);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_f16_ts(tbase + T_DK, a_p + 64 + 32 * (k >> 1) + 8 * (k & 1), b_q + 128 * k, idKV,
                        (u > 0 || k > 0) ? 1u : 0u);
          if (hh == 1) umma_commit(q_empty + s);
          trace(tron, 3072 + 4 * gu + 2);
          // The next scores of this half buffer, behind the MMAs that read it.
          if (u + 2 < U && !issue_sp(u + 2)) {
            fail(err, &s_abort, 33u);
            ok = false;
            break;
          }
          trace(tron, 3072 + 4 * gu + 3);
        }
        if (!ok) break;
        umma_commit(acc_full);
        umma_commit(kv_empty + ks);
        gt += nsteps;
      }
      // Every issued MMA has finished before TMEM is released.
      umma_commit(mma_done);
      mbar_spin(mma_done, 0, kWait);
    }
  } else if (warp >= 4 && warp < 12) {
    // ---- P^T and dS^T: one key row per thread, 32 query columns of each half per warp
    const int wg = (warp >> 2) - 1;     // column group within a half
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // key row in the block = TMEM lane
    const uint32_t lane_base = tbase + ((uint32_t)(quarter * 32) << 16);
    const bool tr = tron && wg == 0 && r == 0;
    bool ok = true;
    int gt = 0, it = 0;
    for (int pos; ok && (pos = bwd_item(it, cta, P, nitems)) >= 0; ++it) {
      int kb, bh, i0, nsteps;
      item(pos, kb, bh, i0, nsteps);
      for (int u = 0; u < 2 * nsteps; ++u) {
        const int gu = 2 * gt + u, t = u >> 1, tb = gt + t, hh = u & 1, s = tb & 1, bf = gu & 1;
        const int i = i0 + t;
        if (!warp_wait(sp_full + bf, (uint32_t)(gu >> 1) & 1, lane) ||
            (hh == 0 && !warp_wait(q_full + s, (uint32_t)(tb >> 1) & 1, lane)) || s_abort) {
          ok = false;
          break;
        }
        if (tr) trace(true, 2048 + 4 * gu);
        tc_fence_after();
        uint32_t sr[32], dr[32];
        const uint32_t col_s = lane_base + T_SP + bf * 128 + wg * 32;  // this warp's S^T columns; dP^T at + 64
        tmem_ld_x32(col_s, sr);
        tmem_ld_x32(col_s + 64, dr);
        tmem_ld_wait();
        if (tr) trace(true, 2048 + 4 * gu + 1);
        // dS^T goes to shared memory stage s as well (the A operand of dQ):
        // the stage is free once the dQ of query block tb - 2 has completed.
        if (hh == 0 && tb >= 2 && !warp_wait(dq_read + s, (uint32_t)((tb >> 1) - 1) & 1, lane)) {
          ok = false;
          break;
        }
        if (tr) trace(true, 2048 + 4 * gu + 2);
        const int cbase = hh * 64 + wg * 32;  // first query column of this thread's 32
        const float* lse_s = reinterpret_cast<const float*>(smem + G_LSE + s * 512) + cbase;
        const float* del_s = reinterpret_cast<const float*>(smem + G_DEL + s * 512) + cbase;
        uint8_t* dst_s = smem + G_DST + (s * 2 + hh) * TILE;
        const bool diag = causal && i == kb;
        uint32_t ppk[16], dpk[16];
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
            ffma2(p[e], p[e + 1], __uint_as_float(sr[c]), __uint_as_float(sr[c + 1]), scale_log2, scale_log2, n0,
                  n1);
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
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            ppk[ch * 4 + e] = pack_bf16(p[2 * e], p[2 * e + 1]);
            dpk[ch * 4 + e] = pack_bf16(ds[2 * e], ds[2 * e + 1]);
          }
          uint4 dk;
          dk.x = dpk[ch * 4 + 0];
          dk.y = dpk[ch * 4 + 1];
          dk.z = dpk[ch * 4 + 2];
          dk.w = dpk[ch * 4 + 3];
          *reinterpret_cast<uint4*>(dst_s + sw128(r, wg * 4 + ch)) = dk;
        }
        // P^T and dS^T over this warp's own (already read) score columns.
        tmem_st_x16(col_s, ppk);
        tmem_st_x16(col_s + 64, dpk);
        tmem_st_wait();
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(pds_full + bf);
        if (tr) trace(true, 2048 + 4 * gu + 3);
      }
      // dV (warps 4-7) and dK (warps 8-11) of this item out of TMEM once
      // every step is accumulated; then the MMA warp may start the next item's.
      if (ok && warp_wait(acc_full, (uint32_t)it & 1, lane)) {
        tc_fence_after();
        const float sc = wg == 0 ? 1.f : scale;
        const size_t row = (size_t)((bh / H) * T + kb * BKV + r) * (3 * C);
        uint4* g = reinterpret_cast<uint4*>(dqkv + row + (wg == 0 ? 2 * C : C) + (bh % H) * HD);
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
        tc_fence_before();
        mbar_arrive(acc_empty);
      } else {
        ok = false;
      }
      gt += nsteps;
    }
    if (!ok && lane == 0) fail(err, &s_abort, 36u);
  } else if (warp >= 12) {
    // ---- dQ_i: TMEM -> swizzled shared staging -> tensor bulk fp32 adds into the accumulator
    const int quarter = warp & 3;
    const int rq = quarter * 32 + lane;  // query row in the block = TMEM lane
    const uint32_t lane_base = tbase + ((uint32_t)(quarter * 32) << 16);
    const bool issuer = (warp == 12 && lane == 0);
    uint8_t* stage = smem + G_DQS;
    bool ok = true;
    int gt = 0, it = 0;
    for (int pos; ok && (pos = bwd_item(it, cta, P, nitems)) >= 0; ++it) {
      int kb, bh, i0, nsteps;
      item(pos, kb, bh, i0, nsteps);
      for (int t = 0; t < nsteps; ++t) {
        const int tb = gt + t, i = i0 + t, s = tb & 1;
        ok = warp_wait(dq_full + s, (uint32_t)(tb >> 1) & 1, lane) && !s_abort;
        uint32_t v[HD];
        if (ok) {
          tc_fence_after();
          tmem_ld_x32(lane_base + T_DQ + s * HD, v);
          tmem_ld_x32(lane_base + T_DQ + s * HD + 32, v + 32);
          tmem_ld_wait();
          tc_fence_before();
          mbar_arrive(dq_empty + s);
        }
        // Row rq as two 128 x 32 fp32 boxes through one staging box in the
        // 128-byte-swizzled layout of the dQ tensor map (chunk k of 4 floats
        // lands at k ^ (rq & 7)); the box is rewritten once the previous
        // reduction has read it. All four warps leave together if any of
        // them gave up (no one may wait at the barriers below for a warp
        // that has left).
        const int y0 = bh * T + i * BQ;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          if (issuer) tma_store_wait_read<0>();
          if (!named_and(2, 128, ok)) {
            ok = false;
            break;
          }
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            float4 f;
            f.x = __uint_as_float(v[half * 32 + k * 4 + 0]);
            f.y = __uint_as_float(v[half * 32 + k * 4 + 1]);
            f.z = __uint_as_float(v[half * 32 + k * 4 + 2]);
            f.w = __uint_as_float(v[half * 32 + k * 4 + 3]);
            *reinterpret_cast<float4*>(stage + sw128(rq, k)) = f;
          }
          fence_proxy_async_smem();
          named_sync(2, 128);
          if (issuer) {
            tma_reduce_add_2d(&tm_dq, stage, half * 32, y0);
            tma_store_commit();
          }
        }
        if (!ok) break;
      }
      gt += nsteps;
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
__global__ void k_attn_prep(const __nv_bfloat16* __restrict__ y, const __nv_bfloat16* __restrict__ dy,
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
  const size_t rh = ((size_t)bb * H + h) * T + t;
  delta[rh] = acc;
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
  const long long rows = (long long)B * T * H;
  // The dQ accumulator is cleared as one contiguous range: cleared row by row
  // from the prep kernel (rows 256 KB apart across neighbouring threads) the
  // prep took 19.8 us per GPT-2 layer.
  e = cudaMemsetAsync(dq_acc, 0, (size_t)B * H * T * HD * sizeof(float), s);
  if (e != cudaSuccess) return e;
  k_attn_prep<<<(unsigned)((rows + 255) / 256), 256, 0, s>>>(y, dy, delta, B * T, T, H);
  const float scale = 1.f / sqrtf((float)HD);
  const int items = (T / BKV) * B * H;
  const unsigned grid = (unsigned)(items < gemm_sm_count() ? items : gemm_sm_count());
  k_attn_bwd<<<grid, G_THREADS, G_SMEM, s>>>(tq, tdo, tdq, lse, delta, dqkv, B, T, H, causal ? 1 : 0, scale,
                                              gemm_err_word());
  const long long chunks = (long long)B * H * T * (HD / 8);
  k_attn_dq_out<<<(unsigned)((chunks + 255) / 256), 256, 0, s>>>(dq_acc, dqkv, B, T, H, scale);
  return cudaGetLastError();
}

}  // namespace nexar
