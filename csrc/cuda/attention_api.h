// Host API of the tcgen05 self-attention kernels (head dimension 64).
//
// qkv: row-major [B*T, 3C] bf16 (C = H * 64; Q, K, V column blocks, head h at
// h*64), y: [B*T, C] bf16, lse: [B, H, T] fp32 natural-log softmax
// normalisers of the scaled scores (scale 1/8). T must be a multiple of 128.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstddef>

namespace nexar {

bool attention_supported(int B, int T, int H, int head_dim);
cudaError_t attention_fwd(const __nv_bfloat16* qkv, __nv_bfloat16* y, float* lse, int B, int T, int H, bool causal,
                          cudaStream_t s);
// fp32 workspace of the backward pass: the dQ accumulator [B, H, T, 64] and
// Delta = rowsum(dy * y) [B, H, T].
size_t attention_bwd_workspace_floats(int B, int T, int H);
// dqkv: [B*T, 3C] bf16 gradient of qkv (every element written).
cudaError_t attention_bwd(const __nv_bfloat16* qkv, const __nv_bfloat16* y, const __nv_bfloat16* dy,
                          const float* lse, __nv_bfloat16* dqkv, float* ws, int B, int T, int H, bool causal,
                          cudaStream_t s);

// Tuning aid: record the event timeline (SM clock) of CTA `cta` of the
// following launches (-1: off), and read the 4096 recorded slots back.
cudaError_t attention_trace_select(int cta);
cudaError_t attention_trace_read(unsigned long long* host, int n);

}  // namespace nexar
