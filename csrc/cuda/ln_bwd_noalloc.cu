// LayerNorm backward with its scratch in a static device array (no
// allocation). See ln_bwd_noalloc.h for who needs this and its limits.
#include "ln_bwd_noalloc.h"

#include <mutex>

#include "ops_api.h"

namespace {

// fp32 partial column sums: [blocks][2][C] (dgamma, dbeta per row block).
static __device__ __align__(256) unsigned char g_ln_noalloc_scratch[NEXAR_LN_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mu;
void* g_scratch_addr[kMaxDevices] = {nullptr};

// Resolve the array's device address once per device, with that device
// current (the caller's current device is the one the stream belongs to).
int scratch_address(int device, unsigned char** out) {
  if (device < 0 || device >= kMaxDevices) return NEXAR_LN_NOALLOC_SETUP_FAILED;
  std::lock_guard<std::mutex> g(g_setup_mu);
  if (g_scratch_addr[device] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_ln_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) return NEXAR_LN_NOALLOC_SETUP_FAILED;
    g_scratch_addr[device] = p;
  }
  *out = static_cast<unsigned char*>(g_scratch_addr[device]);
  return NEXAR_LN_NOALLOC_OK;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int nexar_ln_bwd_noalloc(
    const void* dy, const void* x, const float* mean, const float* rstd, const void* w,
    const void* dres, void* dx, void* dw, void* db, int R, int C, cudaStream_t stream) {
  if (!dy || !x || !mean || !rstd || !w || !dx || !dw || !db || R <= 0 || C <= 0 || C % 8 != 0)
    return NEXAR_LN_NOALLOC_BAD_ARGUMENT;
  if (C > NEXAR_LN_NOALLOC_MAX_C) return NEXAR_LN_NOALLOC_TOO_LARGE;
  const int blocks = nexar::ln_bwd_blocks(R);
  const size_t need = nexar::ln_bwd_scratch_floats(C, blocks) * sizeof(float);
  if (need > NEXAR_LN_NOALLOC_SCRATCH_BYTES) return NEXAR_LN_NOALLOC_TOO_LARGE;
  int device = -1;
  if (cudaGetDevice(&device) != cudaSuccess) return NEXAR_LN_NOALLOC_SETUP_FAILED;
  unsigned char* base = nullptr;
  const int st = scratch_address(device, &base);
  if (st != NEXAR_LN_NOALLOC_OK) return st;
  float* partials = reinterpret_cast<float*>(base);
  using bf = __nv_bfloat16;
  const cudaError_t e = nexar::ln_bwd(static_cast<const bf*>(dy), static_cast<const bf*>(x), mean, rstd,
                                      static_cast<const bf*>(w), static_cast<const bf*>(dres),
                                      static_cast<bf*>(dx), static_cast<bf*>(dw), static_cast<bf*>(db),
                                      partials, nullptr, R, C, blocks, stream);
  return e == cudaSuccess ? NEXAR_LN_NOALLOC_OK : NEXAR_LN_NOALLOC_LAUNCH_FAILED;
}
