// Host API of the expert-parallel MoE kernels.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace nexar {
struct CommDev;
// Top-2 routing: slot 2t+k of token t goes to slot_expert with gate slot_gate
// and local position slot_pos (atomic order within the expert); counts[E]
// must be zeroed by the caller.
cudaError_t moe_route(const void* logits, bool logits_bf16, int T, int E, int* slot_expert, int* slot_pos,
                      float* slot_gate, int* counts, cudaStream_t s);
// Fused all-to-all dispatch + permutation into the experts' receive buffers
// (heap offset recv_off, capacity rows of d bf16). counts_all: [W][E] all
// ranks' counts. Rewrites slot_pos to the global row (or -1 if dropped).
// ticket: one zeroed uint32 (left zeroed).
cudaError_t moe_dispatch(const CommDev& c, const __nv_bfloat16* x, int T, int d, const int* slot_expert,
                         int* slot_pos, const int* counts_all, unsigned long long recv_off, int capacity,
                         unsigned int* ticket, cudaStream_t s);
// Backward of combine: slot 2t+k stores slot_scale[slot] * g[t] (scale 1 if
// null) into global row slot_pos[slot] (as rewritten by moe_dispatch; -1 =
// dropped) of expert slot_expert[slot]'s buffer at heap offset dst_off.
cudaError_t moe_dispatch_rows(const CommDev& c, const __nv_bfloat16* g, int T, int d, const int* slot_expert,
                              const int* slot_pos, const float* slot_scale, unsigned long long dst_off, int capacity,
                              unsigned int* ticket, cudaStream_t s);
// Fused combine: out[t] = sum_k gate_k * expert_out[expert_k][row_k] pulled from peers.
cudaError_t moe_combine(const CommDev& c, __nv_bfloat16* out, int T, int d, const int* slot_expert,
                        const int* slot_pos, const float* slot_gate, unsigned long long eout_off, cudaStream_t s);
}  // namespace nexar
