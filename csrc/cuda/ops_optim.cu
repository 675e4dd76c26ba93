// Optimizer kernels: global gradient-norm clip coefficient and fused AdamW
// over flat parameter buffers (sm_100a).
#include "common.cuh"
#include "ops_api.h"

namespace nexar {

namespace {
constexpr int kOptThreads = 512;

__global__ void __launch_bounds__(kOptThreads) k_grad_norm(const __nv_bfloat16* __restrict__ g,
                                                           long long n, float max_norm,
                                                           float* __restrict__ scratch,
                                                           unsigned int* counter, float* norm_out,
                                                           float* coef) {
  float acc = 0.f;
  const long long n8 = n / 8;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n8;
       i += (long long)gridDim.x * blockDim.x) {
    uint4 r = *reinterpret_cast<const uint4*>(g + i * 8);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&r);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float2 t = __bfloat1622float2(h[k]);
      acc += t.x * t.x + t.y * t.y;
    }
  }
  for (long long j = n8 * 8 + blockIdx.x * (long long)blockDim.x + threadIdx.x; j < n;
       j += (long long)gridDim.x * blockDim.x) {
    const float v = __bfloat162float(g[j]);
    acc += v * v;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  __shared__ float red[kOptThreads / 32];
  __shared__ unsigned int ticket;
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float b = 0.f;
    for (int w = 0; w < kOptThreads / 32; ++w) b += red[w];
    scratch[blockIdx.x] = b;
    __threadfence();
    ticket = atomicAdd(counter, 1u);
  }
  __syncthreads();
  if (ticket != gridDim.x - 1) return;
  __threadfence();
  if (threadIdx.x < 32) {
    float t = 0.f;
    for (unsigned int b = threadIdx.x; b < gridDim.x; b += 32) t += __ldcg(scratch + b);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) {
      const float norm = sqrtf(t);
      if (norm_out) *norm_out = norm;
      if (coef) *coef = (max_norm > 0.f) ? fminf(1.f, max_norm / (norm + 1e-6f)) : 1.f;
      *counter = 0u;
    }
  }
}

__global__ void __launch_bounds__(kOptThreads) k_adamw(float* __restrict__ p, float* __restrict__ m,
                                                       float* __restrict__ v,
                                                       const __nv_bfloat16* __restrict__ g,
                                                       __nv_bfloat16* __restrict__ pb, long long n,
                                                       long long decay_end, float lr, float b1,
                                                       float b2, float eps, float wd, float bc1,
                                                       float bc2, const float* gscale,
                                                       const int* step_dev, const float* lr_dev) {
  const float gs = gscale ? *gscale : 1.f;
  if (step_dev) {
    // Step count and learning rate live on the device so a captured CUDA
    // graph replays with the current values.
    const float st = (float)*step_dev;
    bc1 = 1.f - powf(b1, st);
    bc2 = 1.f - powf(b2, st);
  }
  if (lr_dev) lr = *lr_dev;
  const long long n4 = n / 4;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4;
       i += (long long)gridDim.x * blockDim.x) {
    float4 pp = reinterpret_cast<float4*>(p)[i];
    float4 mm = reinterpret_cast<float4*>(m)[i];
    float4 vv = reinterpret_cast<float4*>(v)[i];
    const uint2 gr = reinterpret_cast<const uint2*>(g)[i];
    const __nv_bfloat162* gh = reinterpret_cast<const __nv_bfloat162*>(&gr);
    const float2 g01 = __bfloat1622float2(gh[0]);
    const float2 g23 = __bfloat1622float2(gh[1]);
    float gg[4] = {g01.x * gs, g01.y * gs, g23.x * gs, g23.y * gs};
    float* P = &pp.x;
    float* M = &mm.x;
    float* Vv = &vv.x;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const long long idx = i * 4 + e;
      M[e] = b1 * M[e] + (1.f - b1) * gg[e];
      Vv[e] = b2 * Vv[e] + (1.f - b2) * gg[e] * gg[e];
      const float mh = M[e] / bc1;
      const float vh = Vv[e] / bc2;
      const float decay = idx < decay_end ? wd : 0.f;
      P[e] = P[e] - lr * (mh / (sqrtf(vh) + eps) + decay * P[e]);
    }
    reinterpret_cast<float4*>(p)[i] = pp;
    reinterpret_cast<float4*>(m)[i] = mm;
    reinterpret_cast<float4*>(v)[i] = vv;
    uint2 o;
    __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
    oh[0] = __floats2bfloat162_rn(pp.x, pp.y);
    oh[1] = __floats2bfloat162_rn(pp.z, pp.w);
    reinterpret_cast<uint2*>(pb)[i] = o;
  }
  for (long long j = n4 * 4 + blockIdx.x * (long long)blockDim.x + threadIdx.x; j < n;
       j += (long long)gridDim.x * blockDim.x) {
    const float gg = __bfloat162float(g[j]) * gs;
    m[j] = b1 * m[j] + (1.f - b1) * gg;
    v[j] = b2 * v[j] + (1.f - b2) * gg * gg;
    const float decay = j < decay_end ? wd : 0.f;
    p[j] = p[j] - lr * ((m[j] / bc1) / (sqrtf(v[j] / bc2) + eps) + decay * p[j]);
    pb[j] = __float2bfloat16_rn(p[j]);
  }
}
}  // namespace

int grad_norm_blocks(long long n) {
  long long b = (n / 8 + kOptThreads - 1) / kOptThreads;
  if (b > 148 * 2) b = 148 * 2;
  return (int)(b < 1 ? 1 : b);
}

cudaError_t grad_norm_clip(const __nv_bfloat16* g, long long n, float max_norm, float* scratch,
                           unsigned int* counter, float* norm_out, float* coef, int blocks,
                           cudaStream_t s) {
  k_grad_norm<<<blocks, kOptThreads, 0, s>>>(g, n, max_norm, scratch, counter, norm_out, coef);
  return cudaGetLastError();
}

cudaError_t adamw_step(float* p, float* m, float* v, const __nv_bfloat16* g, __nv_bfloat16* p_bf16,
                       long long n, long long decay_end, float lr, float beta1, float beta2,
                       float eps, float weight_decay, int step, const float* gscale,
                       const int* step_dev, const float* lr_dev, cudaStream_t s) {
  if ((reinterpret_cast<uintptr_t>(p) | reinterpret_cast<uintptr_t>(m) | reinterpret_cast<uintptr_t>(v)) & 15u)
    return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(g) | reinterpret_cast<uintptr_t>(p_bf16)) & 7u) return cudaErrorInvalidValue;
  const float bc1 = 1.f - powf(beta1, (float)step);
  const float bc2 = 1.f - powf(beta2, (float)step);
  long long blocks = (n / 4 + kOptThreads - 1) / kOptThreads;
  if (blocks > 148 * 4) blocks = 148 * 4;
  if (blocks < 1) blocks = 1;
  k_adamw<<<(int)blocks, kOptThreads, 0, s>>>(p, m, v, g, p_bf16, n, decay_end, lr, beta1, beta2, eps,
                                             weight_decay, bc1, bc2, gscale, step_dev, lr_dev);
  return cudaGetLastError();
}

}  // namespace nexar
