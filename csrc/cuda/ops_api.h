// Launch API of the model-side kernels (GPT-2 / Llama-MLP / MoE building
// blocks). All tensors are contiguous row-major device buffers.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>

namespace nexar {

// LayerNorm over the last dim C of R rows. If `res` is non-null the kernel
// first forms s = x + res, writes it to `sum_out`, and normalizes s.
cudaError_t ln_fwd(const __nv_bfloat16* x, const __nv_bfloat16* res, __nv_bfloat16* sum_out,
                   const __nv_bfloat16* w, const __nv_bfloat16* b, __nv_bfloat16* y, float* mean,
                   float* rstd, int R, int C, float eps, cudaStream_t s);
// As ln_fwd with the residual branch's bias folded in: s = x + res + rb.
cudaError_t ln_fwd_ex(const __nv_bfloat16* x, const __nv_bfloat16* res, const __nv_bfloat16* rb,
                      __nv_bfloat16* sum_out, const __nv_bfloat16* w, const __nv_bfloat16* b, __nv_bfloat16* y,
                      float* mean, float* rstd, int R, int C, float eps, cudaStream_t s);
// LayerNorm backward. dx = dLN/dx (+ dres if non-null). dw/db receive the
// column sums; `scratch` holds ln_bwd_scratch_floats(C, blocks) floats;
// `counter` is unused (kept for the C ABI). Two launches: rows, then a
// column reduction of the per-CTA partials.
int ln_bwd_blocks(int R);
size_t ln_bwd_scratch_floats(int C, int blocks);
cudaError_t ln_bwd(const __nv_bfloat16* dy, const __nv_bfloat16* x, const float* mean,
                   const float* rstd, const __nv_bfloat16* w, const __nv_bfloat16* dres,
                   __nv_bfloat16* dx, __nv_bfloat16* dw, __nv_bfloat16* db, float* scratch,
                   unsigned int* counter, int R, int C, int blocks, cudaStream_t s);
// As ln_bwd, plus (if dsum is non-null) the column sums of dx: the bias
// gradient of the layer whose output was added into the residual stream.
// scratch: ln_bwd_scratch_floats_ex(C, blocks, dsum != nullptr) floats.
size_t ln_bwd_scratch_floats_ex(int C, int blocks, bool dsum);
cudaError_t ln_bwd_ex(const __nv_bfloat16* dy, const __nv_bfloat16* x, const float* mean, const float* rstd,
                      const __nv_bfloat16* w, const __nv_bfloat16* dres, __nv_bfloat16* dx, __nv_bfloat16* dw,
                      __nv_bfloat16* db, __nv_bfloat16* dsum, float* scratch, int R, int C, int blocks,
                      cudaStream_t s);
// out[c] (+)= sum_r x[r, c] for a bf16 [R, C] matrix (row stride ldx), fp32
// accumulation in a fixed order; scratch holds colsum_slabs(R) * C floats.
int colsum_slabs(int R);
cudaError_t colsum_bf16(const __nv_bfloat16* x, long long ldx, int R, int C, __nv_bfloat16* out, bool accumulate,
                        float* scratch, cudaStream_t s);

// GELU (tanh approximation, as GPT-2) forward and backward, bf16.
cudaError_t gelu_fwd(const __nv_bfloat16* x, __nv_bfloat16* y, long long n, cudaStream_t s);
cudaError_t gelu_bwd(const __nv_bfloat16* x, const __nv_bfloat16* dy, __nv_bfloat16* dx, long long n,
                     cudaStream_t s);
// SwiGLU: y = silu(g) * u with gu = [R, 2F] (gate | up halves per row).
cudaError_t swiglu_fwd(const __nv_bfloat16* gu, __nv_bfloat16* y, int R, int F, cudaStream_t s);
cudaError_t swiglu_bwd(const __nv_bfloat16* gu, const __nv_bfloat16* dy, __nv_bfloat16* dgu, int R, int F,
                       cudaStream_t s);

// Fused softmax cross-entropy over rows of `logits` [R, Vp] (Vp >= V, the
// padded columns are ignored). Writes per-row loss and, if `dlogits` is
// non-null, (softmax - onehot) * grad_scale into it (may alias logits).
cudaError_t xent_fwd_bwd(const __nv_bfloat16* logits, const int64_t* targets, float* losses,
                         __nv_bfloat16* dlogits, int R, int V, int Vp, float grad_scale,
                         cudaStream_t s);

// Token + position embedding: out[r] = wte[tok[r]] + wpe[r % T].
cudaError_t embed_fwd(const int64_t* tok, const __nv_bfloat16* wte, const __nv_bfloat16* wpe,
                      __nv_bfloat16* out, int R, int T, int C, cudaStream_t s);
// dwte[tok[r]] += dout[r] (atomic); dwpe[t] = sum_b dout[b*T + t] (overwrites).
cudaError_t embed_bwd(const int64_t* tok, const __nv_bfloat16* dout, __nv_bfloat16* dwte,
                      __nv_bfloat16* dwpe, int B, int T, int C, cudaStream_t s);

// Sum of squares of a bf16 buffer -> clip coefficient min(1, max_norm/(norm+1e-6))
// written to *coef (and the norm to *norm_out). `scratch`: grad_norm_blocks()
// floats; `counter`: one zero-initialised uint32.
int grad_norm_blocks(long long n);
cudaError_t grad_norm_clip(const __nv_bfloat16* g, long long n, float max_norm, float* scratch,
                           unsigned int* counter, float* norm_out, float* coef, int blocks,
                           cudaStream_t s);

// AdamW on flat buffers: fp32 master p, m, v; bf16 grad g (times *gscale if
// non-null); bf16 copy of the updated parameters written to p_bf16.
// Elements [0, decay_end) get weight decay; the rest do not. If `step_dev`
// / `lr_dev` are non-null they override `step` / `lr` (graph replay safe).
cudaError_t adamw_step(float* p, float* m, float* v, const __nv_bfloat16* g, __nv_bfloat16* p_bf16,
                       long long n, long long decay_end, float lr, float beta1, float beta2,
                       float eps, float weight_decay, int step, const float* gscale,
                       const int* step_dev, const float* lr_dev, cudaStream_t s);

}  // namespace nexar
