// Elementwise model kernels: GELU, SwiGLU, token/position embedding (sm_100a).
// 16-byte vectorised bf16 I/O with fp32 math.
#include "common.cuh"
#include "ops_api.h"

namespace nexar {

namespace {
constexpr int kEwThreads = 256;

NEXAR_D void ld8f(const __nv_bfloat16* p, float* f) {
  uint4 r = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&r);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    float2 t = __bfloat1622float2(h[k]);
    f[2 * k] = t.x;
    f[2 * k + 1] = t.y;
  }
}
NEXAR_D void st8f(__nv_bfloat16* p, const float* f) {
  uint4 r;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&r);
#pragma unroll
  for (int k = 0; k < 4; ++k) h[k] = __floats2bfloat162_rn(f[2 * k], f[2 * k + 1]);
  *reinterpret_cast<uint4*>(p) = r;
}

// GELU, tanh form: 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))).
constexpr float kGeluC = 0.7978845608028654f;  // sqrt(2/pi)
constexpr float kGeluA = 0.044715f;
NEXAR_D float gelu_f(float x) {
  const float u = kGeluC * (x + kGeluA * x * x * x);
  return 0.5f * x * (1.f + tanhf(u));
}
NEXAR_D float gelu_grad(float x) {
  const float u = kGeluC * (x + kGeluA * x * x * x);
  const float t = tanhf(u);
  const float du = kGeluC * (1.f + 3.f * kGeluA * x * x);
  return 0.5f * (1.f + t) + 0.5f * x * (1.f - t * t) * du;
}

__global__ void __launch_bounds__(kEwThreads) k_gelu_fwd(const __nv_bfloat16* __restrict__ x,
                                                         __nv_bfloat16* __restrict__ y, long long n8) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n8;
       i += (long long)gridDim.x * blockDim.x) {
    float v[8];
    ld8f(x + i * 8, v);
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = gelu_f(v[e]);
    st8f(y + i * 8, v);
  }
}

__global__ void __launch_bounds__(kEwThreads) k_gelu_bwd(const __nv_bfloat16* __restrict__ x,
                                                         const __nv_bfloat16* __restrict__ dy,
                                                         __nv_bfloat16* __restrict__ dx, long long n8) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n8;
       i += (long long)gridDim.x * blockDim.x) {
    float v[8], g[8];
    ld8f(x + i * 8, v);
    ld8f(dy + i * 8, g);
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = g[e] * gelu_grad(v[e]);
    st8f(dx + i * 8, v);
  }
}

NEXAR_D float silu_f(float x) { return x / (1.f + __expf(-x)); }

__global__ void __launch_bounds__(kEwThreads) k_swiglu_fwd(const __nv_bfloat16* __restrict__ gu,
                                                           __nv_bfloat16* __restrict__ y, int R, int F) {
  const long long n8 = (long long)R * F / 8;
  const int f8 = F / 8;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n8;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / f8, c = (i % f8) * 8;
    float g[8], u[8];
    ld8f(gu + r * 2 * F + c, g);
    ld8f(gu + r * 2 * F + F + c, u);
#pragma unroll
    for (int e = 0; e < 8; ++e) g[e] = silu_f(g[e]) * u[e];
    st8f(y + r * F + c, g);
  }
}

__global__ void __launch_bounds__(kEwThreads) k_swiglu_bwd(const __nv_bfloat16* __restrict__ gu,
                                                           const __nv_bfloat16* __restrict__ dy,
                                                           __nv_bfloat16* __restrict__ dgu, int R, int F) {
  const long long n8 = (long long)R * F / 8;
  const int f8 = F / 8;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n8;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / f8, c = (i % f8) * 8;
    float g[8], u[8], d[8], dg[8], du[8];
    ld8f(gu + r * 2 * F + c, g);
    ld8f(gu + r * 2 * F + F + c, u);
    ld8f(dy + r * F + c, d);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float sg = 1.f / (1.f + __expf(-g[e]));
      const float si = g[e] * sg;
      du[e] = d[e] * si;
      dg[e] = d[e] * u[e] * (sg * (1.f + g[e] * (1.f - sg)));
    }
    st8f(dgu + r * 2 * F + c, dg);
    st8f(dgu + r * 2 * F + F + c, du);
  }
}

__global__ void __launch_bounds__(kEwThreads) k_embed_fwd(const int64_t* __restrict__ tok,
                                                          const __nv_bfloat16* __restrict__ wte,
                                                          const __nv_bfloat16* __restrict__ wpe,
                                                          __nv_bfloat16* __restrict__ out, int R, int T,
                                                          int C) {
  const int c8 = C / 8;
  const long long n8 = (long long)R * c8;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n8;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / c8;
    const int c = (int)(i % c8) * 8;
    const long long t = tok[r];
    float a[8], b[8];
    ld8f(wte + t * C + c, a);
    ld8f(wpe + (r % T) * C + c, b);
#pragma unroll
    for (int e = 0; e < 8; ++e) a[e] += b[e];
    st8f(out + r * C + c, a);
  }
}

// dwte scatter-add: one thread per (row, bf16 pair).
__global__ void __launch_bounds__(kEwThreads) k_embed_bwd_wte(const int64_t* __restrict__ tok,
                                                              const __nv_bfloat16* __restrict__ dout,
                                                              __nv_bfloat16* __restrict__ dwte, int R,
                                                              int C) {
  const int c2 = C / 2;
  const long long n2 = (long long)R * c2;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n2;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / c2;
    const int c = (int)(i % c2) * 2;
    const __nv_bfloat162 g = *reinterpret_cast<const __nv_bfloat162*>(dout + r * C + c);
    atomicAdd(reinterpret_cast<__nv_bfloat162*>(dwte + tok[r] * C + c), g);
  }
}

// dwpe[t] = sum over the batch of dout[b*T + t]; deterministic (no atomics).
__global__ void __launch_bounds__(kEwThreads) k_embed_bwd_wpe(const __nv_bfloat16* __restrict__ dout,
                                                              __nv_bfloat16* __restrict__ dwpe, int B,
                                                              int T, int C) {
  const int c8 = C / 8;
  const long long n8 = (long long)T * c8;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n8;
       i += (long long)gridDim.x * blockDim.x) {
    const long long t = i / c8;
    const int c = (int)(i % c8) * 8;
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int b = 0; b < B; ++b) {
      float v[8];
      ld8f(dout + ((long long)b * T + t) * C + c, v);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += v[e];
    }
    st8f(dwpe + t * C + c, acc);
  }
}

inline int ew_grid(long long work) {
  long long g = (work + kEwThreads - 1) / kEwThreads;
  if (g > 148 * 16) g = 148 * 16;
  return (int)(g < 1 ? 1 : g);
}
}  // namespace

cudaError_t gelu_fwd(const __nv_bfloat16* x, __nv_bfloat16* y, long long n, cudaStream_t s) {
  if (n % 8) return cudaErrorInvalidValue;
  k_gelu_fwd<<<ew_grid(n / 8), kEwThreads, 0, s>>>(x, y, n / 8);
  return cudaGetLastError();
}
cudaError_t gelu_bwd(const __nv_bfloat16* x, const __nv_bfloat16* dy, __nv_bfloat16* dx, long long n,
                     cudaStream_t s) {
  if (n % 8) return cudaErrorInvalidValue;
  k_gelu_bwd<<<ew_grid(n / 8), kEwThreads, 0, s>>>(x, dy, dx, n / 8);
  return cudaGetLastError();
}
cudaError_t swiglu_fwd(const __nv_bfloat16* gu, __nv_bfloat16* y, int R, int F, cudaStream_t s) {
  if (F % 8) return cudaErrorInvalidValue;
  k_swiglu_fwd<<<ew_grid((long long)R * F / 8), kEwThreads, 0, s>>>(gu, y, R, F);
  return cudaGetLastError();
}
cudaError_t swiglu_bwd(const __nv_bfloat16* gu, const __nv_bfloat16* dy, __nv_bfloat16* dgu, int R, int F,
                       cudaStream_t s) {
  if (F % 8) return cudaErrorInvalidValue;
  k_swiglu_bwd<<<ew_grid((long long)R * F / 8), kEwThreads, 0, s>>>(gu, dy, dgu, R, F);
  return cudaGetLastError();
}
cudaError_t embed_fwd(const int64_t* tok, const __nv_bfloat16* wte, const __nv_bfloat16* wpe,
                      __nv_bfloat16* out, int R, int T, int C, cudaStream_t s) {
  if (C % 8) return cudaErrorInvalidValue;
  k_embed_fwd<<<ew_grid((long long)R * C / 8), kEwThreads, 0, s>>>(tok, wte, wpe, out, R, T, C);
  return cudaGetLastError();
}
cudaError_t embed_bwd(const int64_t* tok, const __nv_bfloat16* dout, __nv_bfloat16* dwte,
                      __nv_bfloat16* dwpe, int B, int T, int C, cudaStream_t s) {
  if (C % 8) return cudaErrorInvalidValue;
  const int R = B * T;
  k_embed_bwd_wte<<<ew_grid((long long)R * C / 2), kEwThreads, 0, s>>>(tok, dout, dwte, R, C);
  k_embed_bwd_wpe<<<ew_grid((long long)T * C / 8), kEwThreads, 0, s>>>(dout, dwpe, B, T, C);
  return cudaGetLastError();
}

}  // namespace nexar
