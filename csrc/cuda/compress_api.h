// Host API of the top-k / fp8 gradient compression kernels.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstddef>

namespace nexar {
// Workspace for topk_fp8_compress over n elements (bytes).
size_t compress_workspace_bytes(unsigned long long n, int* nblk_out);
// Blob bytes for k selected elements: [scale f32 | pad][k u32 idx][k e4m3].
size_t compress_blob_bytes(unsigned long long k);
// residual += grad; select the k largest |residual|; quantise them to e4m3
// with one per-tensor scale into `blob`; residual keeps what was not sent.
cudaError_t topk_fp8_compress(const __nv_bfloat16* grad, float* residual, unsigned long long n, unsigned long long k,
                              unsigned char* blob, void* ws, cudaStream_t s);
// out[idx] += out_scale * dequant(value) for every entry of one blob.
cudaError_t decompress_accumulate(const unsigned char* blob, unsigned long long k, __nv_bfloat16* out, float out_scale,
                                  cudaStream_t s);
int compress_kernel_launches();
}  // namespace nexar
