// Host side of the tcgen05 GEMM: tensor-map creation and launch.
#include <mutex>

#include "gemm_launch.cuh"

namespace nexar {

namespace {
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}
}  // namespace

unsigned int* gemm_err_word() {
  static unsigned int* w = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    if (cudaMalloc(&w, sizeof(unsigned int) * 64) == cudaSuccess) cudaMemset(w, 0, sizeof(unsigned int) * 64);
  });
  return w;
}

int gemm_sm_count() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

// 2D bf16 tensor map over a row-major [rows, cols] matrix with leading
// dimension ld (elements), box = [box_rows, box_cols], 128-byte swizzle.
cudaError_t make_tmap_bf16(CUtensorMap* map, const void* base, long long rows, long long cols, long long ld,
                           int box_rows, int box_cols) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) || (ld * 2) % 16) return cudaErrorInvalidValue;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t gemm_bf16(const __nv_bfloat16* A, const __nv_bfloat16* B, __nv_bfloat16* C, int M, int N, int K,
                      long long lda, long long ldb, long long ldc, const __nv_bfloat16* bias,
                      const __nv_bfloat16* residual, long long ldr, __nv_bfloat16* pre_act, int act, float alpha,
                      cudaStream_t s) {
  CUtensorMap tout, tpre;
  cudaError_t e = make_tmap_bf16(&tout, C, M, N, ldc, 32, 64);
  if (e != cudaSuccess) return e;
  tpre = tout;
  if (pre_act) {
    e = make_tmap_bf16(&tpre, pre_act, M, N, ldc, 32, 64);
    if (e != cudaSuccess) return e;
  }
  gemm::EpiStore epi{bias, residual, ldr, alpha, act, pre_act != nullptr};
  return launch_gemm_generic<gemm::EpiStore, gemm::NoGate, 0>(A, B, M, N, K, lda, ldb, tout, tpre, 0, epi,
                                                                gemm::NoGate{}, 0, s);
}

unsigned int gemm_error_flag() {
  unsigned int v = 0;
  if (unsigned int* w = gemm_err_word()) cudaMemcpy(&v, w, sizeof(v), cudaMemcpyDeviceToHost);
  return v;
}

}  // namespace nexar
