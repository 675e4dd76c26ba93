// Launch helper shared by the plain and the fused (collective) GEMMs.
#pragma once
#include "gemm.cuh"
#include "gemm_api.h"

namespace nexar {

unsigned int* gemm_err_word();
int gemm_sm_count();

// A is [M, K] (K-major, AMN = 0) or [K, M] (MN-major); B is [N, K] or [K, N].
template <class Epi, class Gate, int EXTRA, int AMN = 0, int BMN = 0, int TBN = 256>
cudaError_t launch_gemm_generic(const void* A, const void* B, int M, int N, int K, long long lda, long long ldb,
                                const CUtensorMap& tout, const CUtensorMap& tpre, int m_rotate, const Epi& epi,
                                const Gate& gate, int grid_override, cudaStream_t s, int splits = 1) {
  using namespace gemm;
  if (M <= 0 || N <= 0 || K <= 0) return cudaSuccess;
  CUtensorMap ta, tb;
  cudaError_t e = AMN ? make_tmap_bf16(&ta, A, K, M, lda, 64, 64) : make_tmap_bf16(&ta, A, M, K, lda, BM, BK);
  if (e != cudaSuccess) return e;
  e = BMN ? make_tmap_bf16(&tb, B, K, N, ldb, 64, 64) : make_tmap_bf16(&tb, B, N, K, ldb, TBN, BK);
  if (e != cudaSuccess) return e;
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(k_gemm_bf16<Epi, Gate, EXTRA, AMN, BMN, TBN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         smem_bytes_for(TBN));
    attr_set = true;
  }
  const int tiles = ((M + BM - 1) / BM) * ((N + TBN - 1) / TBN) * splits;
  int grid = gemm_sm_count();
  if (grid_override > 0) {
    grid = grid_override;  // fused kernels: every CTA also has collective work
  } else if (tiles < grid) {
    grid = tiles;
  }
  k_gemm_bf16<Epi, Gate, EXTRA, AMN, BMN, TBN><<<grid, THREADS + 32 * EXTRA, smem_bytes_for(TBN), s>>>(
      ta, tb, tout, tpre, M, N, K, m_rotate, splits, epi, gate, gemm_err_word());
  return cudaGetLastError();
}

}  // namespace nexar
