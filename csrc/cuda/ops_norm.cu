// LayerNorm forward/backward for bf16 activations (sm_100a).
//
// One warp per row; each lane owns fixed 8-element column packs, so in the
// backward pass the dgamma/dbeta partial sums stay in registers across all
// rows a warp visits. Block partials go to a scratch buffer and the last
// block to finish reduces them (ticket counter), so the whole backward is one
// launch. Statistics are computed in fp32 from the bf16 inputs.
#include "common.cuh"
#include "ops_api.h"

namespace nexar {

namespace {
constexpr int kLnWarps = 8;

NEXAR_D float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

NEXAR_D void load8(const __nv_bfloat16* p, float* f) {
  uint4 r = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&r);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    float2 t = __bfloat1622float2(h[k]);
    f[2 * k] = t.x;
    f[2 * k + 1] = t.y;
  }
}
NEXAR_D void store8(__nv_bfloat16* p, const float* f) {
  uint4 r;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&r);
#pragma unroll
  for (int k = 0; k < 4; ++k) h[k] = __floats2bfloat162_rn(f[2 * k], f[2 * k + 1]);
  *reinterpret_cast<uint4*>(p) = r;
}

template <int NP>
__global__ void __launch_bounds__(kLnWarps * 32) k_ln_fwd(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ res,
    __nv_bfloat16* __restrict__ sum_out, const __nv_bfloat16* __restrict__ w,
    const __nv_bfloat16* __restrict__ b, __nv_bfloat16* __restrict__ y, float* __restrict__ mean,
    float* __restrict__ rstd, int R, int C, float eps) {
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * kLnWarps + (threadIdx.x >> 5);
  if (row >= R) return;
  const size_t base = (size_t)row * C;
  float v[NP][8];
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < NP; ++k) {
    const int col = (lane + 32 * k) * 8;
    if (col < C) {
      load8(x + base + col, v[k]);
      if (res) {
        float r[8];
        load8(res + base + col, r);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[k][e] += r[e];
        // The residual stream is kept in bf16: round before normalising so
        // the statistics match the stored sum exactly.
#pragma unroll
        for (int e = 0; e < 8; ++e) v[k][e] = __bfloat162float(__float2bfloat16_rn(v[k][e]));
        store8(sum_out + base + col, v[k]);
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) s += v[k][e];
    }
  }
  const float mu = warp_sum(s) / C;
  float q = 0.f;
#pragma unroll
  for (int k = 0; k < NP; ++k) {
    const int col = (lane + 32 * k) * 8;
    if (col < C) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float d = v[k][e] - mu;
        q += d * d;
      }
    }
  }
  const float rs = rsqrtf(warp_sum(q) / C + eps);
#pragma unroll
  for (int k = 0; k < NP; ++k) {
    const int col = (lane + 32 * k) * 8;
    if (col < C) {
      float wf[8], bf[8], o[8];
      load8(w + col, wf);
      load8(b + col, bf);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = (v[k][e] - mu) * rs * wf[e] + bf[e];
      store8(y + base + col, o);
    }
  }
  if (lane == 0) {
    mean[row] = mu;
    rstd[row] = rs;
  }
}

template <int NP>
__global__ void __launch_bounds__(kLnWarps * 32) k_ln_bwd(
    const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
    const float* __restrict__ mean, const float* __restrict__ rstd,
    const __nv_bfloat16* __restrict__ w, const __nv_bfloat16* __restrict__ dres,
    __nv_bfloat16* __restrict__ dx, __nv_bfloat16* __restrict__ dw, __nv_bfloat16* __restrict__ db,
    float* __restrict__ scratch, unsigned int* counter, int R, int C) {
  extern __shared__ float smem[];  // [2][C]
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < 2 * C; i += blockDim.x) smem[i] = 0.f;
  float aw[NP][8], ab[NP][8], wf[NP][8];
#pragma unroll
  for (int k = 0; k < NP; ++k) {
    const int col = (lane + 32 * k) * 8;
#pragma unroll
    for (int e = 0; e < 8; ++e) aw[k][e] = ab[k][e] = 0.f;
    if (col < C) load8(w + col, wf[k]);
  }
  __syncthreads();
  const int wstride = gridDim.x * kLnWarps;
  for (int row = blockIdx.x * kLnWarps + warp; row < R; row += wstride) {
    const size_t base = (size_t)row * C;
    const float mu = mean[row], rs = rstd[row];
    float g[NP][8], xh[NP][8];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int k = 0; k < NP; ++k) {
      const int col = (lane + 32 * k) * 8;
      if (col < C) {
        float xv[8];
        load8(dy + base + col, g[k]);
        load8(x + base + col, xv);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          xh[k][e] = (xv[e] - mu) * rs;
          aw[k][e] += g[k][e] * xh[k][e];
          ab[k][e] += g[k][e];
          const float gw = g[k][e] * wf[k][e];
          s1 += gw;
          s2 += gw * xh[k][e];
        }
      }
    }
    s1 = warp_sum(s1) / C;
    s2 = warp_sum(s2) / C;
#pragma unroll
    for (int k = 0; k < NP; ++k) {
      const int col = (lane + 32 * k) * 8;
      if (col < C) {
        float o[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = rs * (g[k][e] * wf[k][e] - s1 - xh[k][e] * s2);
        if (dres) {
          float r[8];
          load8(dres + base + col, r);
#pragma unroll
          for (int e = 0; e < 8; ++e) o[e] += r[e];
        }
        store8(dx + base + col, o);
      }
    }
  }
  // Block partials: warps add their register sums into shared memory.
#pragma unroll
  for (int k = 0; k < NP; ++k) {
    const int col = (lane + 32 * k) * 8;
    if (col < C) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        atomicAdd(&smem[col + e], aw[k][e]);
        atomicAdd(&smem[C + col + e], ab[k][e]);
      }
    }
  }
  __syncthreads();
  float* part = scratch + (size_t)blockIdx.x * 2 * C;
  for (int i = threadIdx.x; i < 2 * C; i += blockDim.x) part[i] = smem[i];
  __threadfence();
  __shared__ unsigned int ticket;
  __syncthreads();
  if (threadIdx.x == 0) ticket = atomicAdd(counter, 1u);
  __syncthreads();
  if (ticket != gridDim.x - 1) return;
  // Last block: reduce all partials column-wise (coalesced over columns).
  __threadfence();
  for (int i = threadIdx.x; i < 2 * C; i += blockDim.x) {
    float acc = 0.f;
    for (unsigned int bb = 0; bb < gridDim.x; ++bb) acc += __ldcg(scratch + (size_t)bb * 2 * C + i);
    if (i < C) dw[i] = __float2bfloat16_rn(acc);
    else db[i - C] = __float2bfloat16_rn(acc);
  }
  if (threadIdx.x == 0) *counter = 0u;
}
}  // namespace

#define LN_DISPATCH(C, ...)                                       \
  {                                                               \
    const int np_ = ((C) + 255) / 256;                            \
    if (np_ <= 1) { constexpr int NP = 1; __VA_ARGS__; }          \
    else if (np_ <= 2) { constexpr int NP = 2; __VA_ARGS__; }     \
    else if (np_ <= 3) { constexpr int NP = 3; __VA_ARGS__; }     \
    else if (np_ <= 4) { constexpr int NP = 4; __VA_ARGS__; }     \
    else if (np_ <= 8) { constexpr int NP = 8; __VA_ARGS__; }     \
    else return cudaErrorInvalidValue;                            \
  }

cudaError_t ln_fwd(const __nv_bfloat16* x, const __nv_bfloat16* res, __nv_bfloat16* sum_out,
                   const __nv_bfloat16* w, const __nv_bfloat16* b, __nv_bfloat16* y, float* mean,
                   float* rstd, int R, int C, float eps, cudaStream_t s) {
  if (C % 8 != 0) return cudaErrorInvalidValue;
  const int grid = (R + kLnWarps - 1) / kLnWarps;
  LN_DISPATCH(C, k_ln_fwd<NP><<<grid, kLnWarps * 32, 0, s>>>(x, res, sum_out, w, b, y, mean, rstd, R, C, eps));
  return cudaGetLastError();
}

int ln_bwd_blocks(int R) {
  int b = (R + kLnWarps * 4 - 1) / (kLnWarps * 4);
  return b < 1 ? 1 : (b > 148 ? 148 : b);
}
size_t ln_bwd_scratch_floats(int C, int blocks) { return (size_t)blocks * 2 * C; }

cudaError_t ln_bwd(const __nv_bfloat16* dy, const __nv_bfloat16* x, const float* mean,
                   const float* rstd, const __nv_bfloat16* w, const __nv_bfloat16* dres,
                   __nv_bfloat16* dx, __nv_bfloat16* dw, __nv_bfloat16* db, float* scratch,
                   unsigned int* counter, int R, int C, int blocks, cudaStream_t s) {
  if (C % 8 != 0) return cudaErrorInvalidValue;
  const size_t shm = 2 * C * sizeof(float);
  LN_DISPATCH(C, k_ln_bwd<NP><<<blocks, kLnWarps * 32, shm, s>>>(dy, x, mean, rstd, w, dres, dx, dw, db, scratch, counter, R, C));
  return cudaGetLastError();
}

}  // namespace nexar
