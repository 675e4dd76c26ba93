// Fused softmax cross-entropy forward + backward (sm_100a).
//
// One block per row. Pass 1 streams the row once with an online max / sum of
// exponentials (fp32); pass 2 writes (softmax - onehot) * grad_scale over the
// logits in place, so the full-vocabulary probabilities are never stored.
#include "common.cuh"
#include "ops_api.h"

namespace nexar {

namespace {
constexpr int kXentThreads = 512;

NEXAR_D void online_merge(float& m, float& s, float m2, float s2) {
  const float mn = fmaxf(m, m2);
  s = (m == -INFINITY ? 0.f : s * __expf(m - mn)) + (m2 == -INFINITY ? 0.f : s2 * __expf(m2 - mn));
  m = mn;
}

__global__ void __launch_bounds__(kXentThreads) k_xent(const __nv_bfloat16* logits,
                                                       const int64_t* __restrict__ targets,
                                                       float* __restrict__ losses,
                                                       __nv_bfloat16* dlogits, int V, int Vp,
                                                       float grad_scale) {
  const int row = blockIdx.x;
  const __nv_bfloat16* x = logits + (size_t)row * Vp;
  float m = -INFINITY, s = 0.f;
  const int nv8 = V / 8;  // full 8-wide packs inside the valid range
  for (int i = threadIdx.x; i < nv8; i += blockDim.x) {
    uint4 r = *reinterpret_cast<const uint4*>(x + i * 8);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&r);
    float v[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float2 t = __bfloat1622float2(h[k]);
      v[2 * k] = t.x;
      v[2 * k + 1] = t.y;
    }
    float pm = v[0];
#pragma unroll
    for (int e = 1; e < 8; ++e) pm = fmaxf(pm, v[e]);
    float ps = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) ps += __expf(v[e] - pm);
    online_merge(m, s, pm, ps);
  }
  for (int j = nv8 * 8 + threadIdx.x; j < V; j += blockDim.x) {
    online_merge(m, s, __bfloat162float(x[j]), 1.f);
  }
  // Block reduce (m, s).
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    online_merge(m, s, m2, s2);
  }
  __shared__ float sm[kXentThreads / 32], ss[kXentThreads / 32];
  __shared__ float lse_sh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sm[warp] = m;
    ss[warp] = s;
  }
  __syncthreads();
  if (warp == 0) {
    m = lane < kXentThreads / 32 ? sm[lane] : -INFINITY;
    s = lane < kXentThreads / 32 ? ss[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      online_merge(m, s, m2, s2);
    }
    if (lane == 0) lse_sh = m + __logf(s);
  }
  __syncthreads();
  const float lse = lse_sh;
  const int64_t t = targets[row];
  if (threadIdx.x == 0) losses[row] = lse - __bfloat162float(x[t]);
  if (dlogits == nullptr) return;
  __syncthreads();  // every thread has read x[t] before it may be overwritten
  __nv_bfloat16* d = dlogits + (size_t)row * Vp;
  const int np8 = Vp / 8;
  for (int i = threadIdx.x; i < np8; i += blockDim.x) {
    uint4 r = *reinterpret_cast<const uint4*>(x + i * 8);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&r);
    float g[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float2 tt = __bfloat1622float2(h[k]);
      g[2 * k] = tt.x;
      g[2 * k + 1] = tt.y;
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int j = i * 8 + e;
      float p = j < V ? __expf(g[e] - lse) : 0.f;
      if (j == t) p -= 1.f;
      g[e] = p * grad_scale;
    }
    uint4 o;
    __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int k = 0; k < 4; ++k) oh[k] = __floats2bfloat162_rn(g[2 * k], g[2 * k + 1]);
    *reinterpret_cast<uint4*>(d + i * 8) = o;
  }
  for (int j = np8 * 8 + threadIdx.x; j < Vp; j += blockDim.x) {
    float p = j < V ? __expf(__bfloat162float(x[j]) - lse) : 0.f;
    if (j == t) p -= 1.f;
    d[j] = __float2bfloat16_rn(p * grad_scale);
  }
}
}  // namespace

cudaError_t xent_fwd_bwd(const __nv_bfloat16* logits, const int64_t* targets, float* losses,
                         __nv_bfloat16* dlogits, int R, int V, int Vp, float grad_scale,
                         cudaStream_t s) {
  if (Vp % 8 != 0 || V > Vp) return cudaErrorInvalidValue;
  k_xent<<<R, kXentThreads, 0, s>>>(logits, targets, losses, dlogits, V, Vp, grad_scale);
  return cudaGetLastError();
}

}  // namespace nexar
