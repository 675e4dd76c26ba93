// LayerNorm backward that allocates no device memory.
//
// This entry point has no counterpart in the reference (ml-rust/nexar has no
// LayerNorm and no device kernels at all). It exists for callers that may not
// allocate device memory at the point where they run the backward pass: code
// running inside a memory pool owned by another framework or runtime (which
// owns every byte of the device and does not expect a library to take more),
// or a latency-critical path where cudaMalloc (which can synchronize the whole
// device) is not acceptable. Such callers still pass every input and output
// buffer; the kernel's temporary storage (per-block partial column sums of
// dgamma and dbeta) comes from a fixed static device array instead of a
// caller-provided or freshly allocated scratch buffer.
//
// Limits and behaviour:
//   * The static array holds NEXAR_LN_NOALLOC_SCRATCH_BYTES (2.5 MiB) on every
//     GPU that loads this library, until the process exits.
//   * Shapes: bf16 rows of width C with C % 8 == 0 and C <= 2048 (the widest
//     row whose partial sums fit the array); larger C is rejected with
//     NEXAR_LN_NOALLOC_TOO_LARGE and nothing is launched.
//   * The first call on each device resolves the array's device address
//     (cudaGetSymbolAddress) with that device current. Make that first call
//     before any CUDA stream capture begins.
//   * All calls on a device share the one array and it keeps the last call's
//     contents. Nothing in it needs clearing: the first launch writes every
//     partial sum that the second launch reads. Calls that can overlap on the
//     GPU (different streams without ordering between them) race on the array
//     and must not be issued.
#pragma once

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NEXAR_LN_NOALLOC_SCRATCH_BYTES (2621440u)
#define NEXAR_LN_NOALLOC_MAX_C 2048

enum NexarNoallocStatus {
  NEXAR_LN_NOALLOC_OK = 0,
  NEXAR_LN_NOALLOC_TOO_LARGE = 1,   // needs more scratch than the static array holds
  NEXAR_LN_NOALLOC_BAD_ARGUMENT = 2,
  NEXAR_LN_NOALLOC_SETUP_FAILED = 3,  // cudaGetSymbolAddress / cudaGetDevice failed
  NEXAR_LN_NOALLOC_LAUNCH_FAILED = 4,
};

// dy, x, w, dres, dx, dw, db: bf16 (__nv_bfloat16) device buffers; x is the
// LayerNorm input [R, C], mean / rstd its saved fp32 row statistics [R],
// w the [C] weight. dres (may be NULL) is added to dx. dw / db receive the
// column sums. Runs on `stream`; returns a NexarNoallocStatus.
__attribute__((visibility("default"))) int nexar_ln_bwd_noalloc(
    const void* dy, const void* x, const float* mean, const float* rstd, const void* w,
    const void* dres, void* dx, void* dw, void* db, int R, int C, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
