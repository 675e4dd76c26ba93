// Host API of the tcgen05 GEMMs (plain and fused with collectives).
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace nexar {

// C[M,N] = act(alpha * A[M,K] . B[N,K]^T + bias) (+ residual), bf16 in/out,
// fp32 accumulation in TMEM. `pre_act` (optional) receives the value before
// the activation. Leading dimensions in elements; all must be multiples of 8.
cudaError_t gemm_bf16(const __nv_bfloat16* A, const __nv_bfloat16* B, __nv_bfloat16* C, int M, int N, int K,
                      long long lda, long long ldb, long long ldc, const __nv_bfloat16* bias,
                      const __nv_bfloat16* residual, long long ldr, __nv_bfloat16* pre_act, int act, float alpha,
                      cudaStream_t s);

// General form. a_mn: A is stored MN-major as row-major [K, M] (lda >= M);
// b_mn: B is stored as row-major [K, N]. accumulate: C += result.
// splits: 1 = no split-K, 0 = choose (uses ws), > 1 = forced (needs ws of
// gemm_split_workspace_bytes; falls back to 1 when ws is too small).
cudaError_t gemm_bf16_ex(const __nv_bfloat16* A, const __nv_bfloat16* B, __nv_bfloat16* C, int M, int N, int K,
                         long long lda, long long ldb, long long ldc, bool a_mn, bool b_mn,
                         const __nv_bfloat16* bias, const __nv_bfloat16* residual, long long ldr,
                         __nv_bfloat16* pre_act, int act, float alpha, bool accumulate, int splits, float* ws,
                         size_t ws_bytes, cudaStream_t s);
int gemm_choose_splits(int M, int N, int K);
// Plain GEMMs may run on the 2-SM (CTA pair, 256x256 tile) kernel (default
// on; NEXAR_GEMM_2SM=0 or gemm_set_2sm(0) keeps every GEMM on the 1-SM kernel).
void gemm_set_2sm(int on);
int gemm_get_2sm();
// Which step of the last failing gemm_bf16_ex call on this thread failed.
const char* gemm_last_failure();
// Name of a CUDA error that an unrelated earlier call left on this host thread
// and that the last gemm_bf16_ex call cleared before launching ("" if none).
const char* gemm_stale_error();
size_t gemm_split_workspace_bytes(int M, int N, int splits);

// Nonzero if any GEMM launch on this device gave up on a bounded wait.
unsigned int gemm_error_flag();

cudaError_t make_tmap_bf16(CUtensorMap* map, const void* base, long long rows, long long cols, long long ld,
                           int box_rows, int box_cols);
cudaError_t make_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, int esize, const void* base, long long rows,
                         long long cols, long long ld, int box_rows, int box_cols);

// ---- fp8 (e4m3) block-scaled GEMM: C[M,N] = epi( sum_kb sa[m,kb] sb[n/128,kb] (A_kb . B_kb^T) )
// A [M, K] e4m3 with 1x128 scales sa [M, ceil(K/128)] (fp32, row-major);
// B [N, K] e4m3 with 128x128 block scales sb [ceil(N/128), ceil(K/128)].
// K-major operands; lda / ldb in elements (bytes), multiples of 16. `pre`
// must be null (the fp8 kernel keeps no pre-activation copy).
cudaError_t gemm_fp8_blockscaled(const uint8_t* A, const float* sa, const uint8_t* B, const float* sb,
                                 __nv_bfloat16* C, int M, int N, int K, long long lda, long long ldb, long long ldc,
                                 const __nv_bfloat16* bias, int act, __nv_bfloat16* pre, float alpha, cudaStream_t s);
// gu [R, 2F] bf16 (gate | up) -> h = silu(gate) * up quantised: q e4m3 [R, F], s [R, ceil(F/128)].
cudaError_t swiglu_quant_fp8_1x128(const __nv_bfloat16* gu, uint8_t* q, float* s, int R, int F, cudaStream_t st);
// x [R, K] bf16 -> q e4m3 [R, K] and s [R, ceil(K/128)] with s = amax(block)/448 (1x128 blocks).
cudaError_t quant_fp8_1x128(const __nv_bfloat16* x, long long ldx, uint8_t* q, long long ldq, float* s, int R, int K,
                            cudaStream_t st);
// w [N, K] bf16 -> q e4m3 [N, K] and s [ceil(N/128), ceil(K/128)] (128x128 blocks).
cudaError_t quant_fp8_128x128(const __nv_bfloat16* w, long long ldw, uint8_t* q, long long ldq, float* s, int N, int K,
                              cudaStream_t st);

}  // namespace nexar

namespace nexar {
struct CommDev;
// Row-parallel linear fused with reduce-scatter: out[M/W, N] on rank r =
// sum over ranks of (A_r . B_r^T)[rows of r] (+ bias). M % (W*128) == 0.
// `maps`: device array of 2 x kMaxRanks tensor maps over every owner's staging
// slot ([M, N] bf16, boxes 32 x 64; DeviceComm::rs_maps): the epilogue writes
// each finished tile into its owner's slot with a TMA store.
cudaError_t gemm_reduce_scatter(const CommDev& c, const __nv_bfloat16* A, const __nv_bfloat16* B,
                                __nv_bfloat16* out, int M, int N, int K, long long lda, long long ldb,
                                long long ldo, const __nv_bfloat16* bias, float alpha, const CUtensorMap* maps,
                                cudaStream_t s);
// Column-parallel linear fused with all-gather: out[M, N] = act(AG(x) . B^T + bias)
// with x the local [M/W, K] shard; afull [M, K] is a local gather workspace and
// cnt a zeroed uint32 array of M/128 + 2 entries (left zeroed on exit).
// fp8 block-scaled variant of gemm_reduce_scatter (A / B e4m3 with 1x128 /
// 128x128 scales as gemm_fp8_blockscaled).
cudaError_t gemm_fp8_reduce_scatter(const CommDev& c, const uint8_t* A, const float* sa, const uint8_t* B,
                                    const float* sb, __nv_bfloat16* out, int M, int N, int K, long long lda,
                                    long long ldb, long long ldo, const __nv_bfloat16* bias, float alpha,
                                    const CUtensorMap* maps, cudaStream_t s);
cudaError_t all_gather_gemm(const CommDev& c, const __nv_bfloat16* x, long long ldx, const __nv_bfloat16* B,
                            __nv_bfloat16* out, __nv_bfloat16* afull, unsigned int* cnt, int M, int N, int K,
                            long long ldb, long long ldo, const __nv_bfloat16* bias, int act, __nv_bfloat16* pre,
                            float alpha, cudaStream_t s);
}  // namespace nexar
