// Host side of the block-scaled fp8 GEMM, plus the 1x128 / 128x128 e4m3
// quantisers that produce its operands.
#include <cuda_fp8.h>

#include "gemm_fp8.cuh"
#include "gemm_api.h"

namespace nexar {

unsigned int* gemm_err_word();
int gemm_sm_count();

namespace {

constexpr float kE4M3Max = 448.f;

__device__ __forceinline__ uint8_t to_e4m3(float v) {
  return (uint8_t)__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
}

// One warp per (row, 128-column block): lane l owns columns 4l..4l+3.
__global__ void __launch_bounds__(256) k_quant_1x128(const __nv_bfloat16* __restrict__ x, long long ldx,
                                                     uint8_t* __restrict__ q, long long ldq, float* __restrict__ s,
                                                     int R, int K) {
  const int kb_count = (K + 127) / 128;
  const long long w = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (w >= (long long)R * kb_count) return;
  const int lane = threadIdx.x & 31;
  const int r = (int)(w / kb_count), kb = (int)(w % kb_count);
  const int c = kb * 128 + lane * 4;
  float v[4] = {0.f, 0.f, 0.f, 0.f};
  const __nv_bfloat16* xr = x + (long long)r * ldx;
  if (c + 3 < K) {
    const uint2 u = *reinterpret_cast<const uint2*>(xr + c);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
    const float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
  } else {
#pragma unroll
    for (int e = 0; e < 4; ++e)
      if (c + e < K) v[e] = __bfloat162float(xr[c + e]);
  }
  float m = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const float scale = m > 0.f ? m / kE4M3Max : 1.f;
  const float inv = 1.f / scale;
  uint8_t* qr = q + (long long)r * ldq;
  if (c + 3 < K) {
    uchar4 o4 = make_uchar4(to_e4m3(v[0] * inv), to_e4m3(v[1] * inv), to_e4m3(v[2] * inv), to_e4m3(v[3] * inv));
    *reinterpret_cast<uchar4*>(qr + c) = o4;
  } else {
#pragma unroll
    for (int e = 0; e < 4; ++e)
      if (c + e < K) qr[c + e] = to_e4m3(v[e] * inv);
  }
  if (lane == 0) s[(long long)r * kb_count + kb] = scale;
}

// SwiGLU fused with the 1x128 quantiser: one warp per (row, 128-column block).
__global__ void __launch_bounds__(256) k_swiglu_quant_1x128(const __nv_bfloat16* __restrict__ gu,
                                                            uint8_t* __restrict__ q, float* __restrict__ s, int R,
                                                            int F) {
  const int kb_count = (F + 127) / 128;
  const long long w = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (w >= (long long)R * kb_count) return;
  const int lane = threadIdx.x & 31;
  const int r = (int)(w / kb_count), kb = (int)(w % kb_count);
  const int c = kb * 128 + lane * 4;
  const __nv_bfloat16* g = gu + (long long)r * 2 * F;
  float h[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    if (c + e < F) {
      const float a = __bfloat162float(g[c + e]), u = __bfloat162float(g[F + c + e]);
      // the bf16 path rounds h to bf16 before the down projection: do the same
      h[e] = __bfloat162float(__float2bfloat16_rn(a / (1.f + __expf(-a)) * u));
    }
  }
  float m = fmaxf(fmaxf(fabsf(h[0]), fabsf(h[1])), fmaxf(fabsf(h[2]), fabsf(h[3])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const float scale = m > 0.f ? m / kE4M3Max : 1.f;
  const float inv = 1.f / scale;
  uint8_t* qr = q + (long long)r * F;
#pragma unroll
  for (int e = 0; e < 4; ++e)
    if (c + e < F) qr[c + e] = to_e4m3(h[e] * inv);
  if (lane == 0) s[(long long)r * kb_count + kb] = scale;
}

// One CTA per 128x128 block: 256 threads, amax over the block, then quantise.
__global__ void __launch_bounds__(256) k_quant_128x128(const __nv_bfloat16* __restrict__ w, long long ldw,
                                                       uint8_t* __restrict__ q, long long ldq, float* __restrict__ s,
                                                       int N, int K) {
  const int kb = blockIdx.x, nb = blockIdx.y;
  const int r0 = nb * 128, c0 = kb * 128;
  __shared__ float red[8];
  float m = 0.f;
  for (int i = threadIdx.x; i < 128 * 128; i += 256) {
    const int r = r0 + i / 128, c = c0 + i % 128;
    if (r < N && c < K) m = fmaxf(m, fabsf(__bfloat162float(w[(long long)r * ldw + c])));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  m = red[0];
#pragma unroll
  for (int j = 1; j < 8; ++j) m = fmaxf(m, red[j]);
  const float scale = m > 0.f ? m / kE4M3Max : 1.f;
  const float inv = 1.f / scale;
  for (int i = threadIdx.x; i < 128 * 128; i += 256) {
    const int r = r0 + i / 128, c = c0 + i % 128;
    if (r < N && c < K) q[(long long)r * ldq + c] = to_e4m3(__bfloat162float(w[(long long)r * ldw + c]) * inv);
  }
  if (threadIdx.x == 0) s[(long long)nb * gridDim.x + kb] = scale;
}

}  // namespace

cudaError_t quant_fp8_1x128(const __nv_bfloat16* x, long long ldx, uint8_t* q, long long ldq, float* s, int R, int K,
                            cudaStream_t st) {
  if (R <= 0 || K <= 0) return cudaSuccess;
  if ((ldx % 4) || (ldq % 4) || (reinterpret_cast<uintptr_t>(x) & 7u) || (reinterpret_cast<uintptr_t>(q) & 3u))
    return cudaErrorInvalidValue;
  const long long warps = (long long)R * ((K + 127) / 128);
  k_quant_1x128<<<(unsigned)((warps + 7) / 8), 256, 0, st>>>(x, ldx, q, ldq, s, R, K);
  return cudaGetLastError();
}

cudaError_t swiglu_quant_fp8_1x128(const __nv_bfloat16* gu, uint8_t* q, float* s, int R, int F, cudaStream_t st) {
  if (R <= 0 || F <= 0) return cudaSuccess;
  const long long warps = (long long)R * ((F + 127) / 128);
  k_swiglu_quant_1x128<<<(unsigned)((warps + 7) / 8), 256, 0, st>>>(gu, q, s, R, F);
  return cudaGetLastError();
}

cudaError_t quant_fp8_128x128(const __nv_bfloat16* w, long long ldw, uint8_t* q, long long ldq, float* s, int N, int K,
                              cudaStream_t st) {
  if (N <= 0 || K <= 0) return cudaSuccess;
  dim3 grid((K + 127) / 128, (N + 127) / 128);
  k_quant_128x128<<<grid, 256, 0, st>>>(w, ldw, q, ldq, s, N, K);
  return cudaGetLastError();
}

cudaError_t gemm_fp8_blockscaled(const uint8_t* A, const float* sa, const uint8_t* B, const float* sb,
                                 __nv_bfloat16* C, int M, int N, int K, long long lda, long long ldb, long long ldc,
                                 const __nv_bfloat16* bias, int act, __nv_bfloat16* pre, float alpha, cudaStream_t s) {
  using namespace gemm8;
  if (M <= 0 || N <= 0 || K <= 0) return cudaSuccess;
  CUtensorMap ta, tb, tout, tpre;
  cudaError_t e = make_tmap_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, A, M, K, lda, BM, BK);
  if (e != cudaSuccess) return e;
  e = make_tmap_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, B, N, K, ldb, BN, BK);
  if (e != cudaSuccess) return e;
  e = make_tmap_bf16(&tout, C, M, N, ldc, 32, 64);
  if (e != cudaSuccess) return e;
  tpre = tout;
  if (pre) return cudaErrorInvalidValue;  // no pre-activation output from the fp8 kernel
  gemm::EpiStore epi{bias, nullptr, 0, alpha, act, 0};
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(k_gemm_fp8<gemm::EpiStore>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    attr_set = true;
  }
  const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  int grid = gemm_sm_count();
  if (tiles < grid) grid = tiles;
  k_gemm_fp8<gemm::EpiStore><<<grid, THREADS, SMEM_BYTES, s>>>(ta, tb, tout, tpre, sa, sb, M, N, K, 0, epi,
                                                               gemm::NoGate{}, gemm_err_word());
  return cudaGetLastError();
}

}  // namespace nexar
