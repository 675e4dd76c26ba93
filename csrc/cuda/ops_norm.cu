// LayerNorm forward/backward for bf16 activations (sm_100a).
//
// One warp per row; each lane owns fixed 8-element column packs, so in the
// backward pass the dgamma/dbeta partial sums stay in registers across all
// rows a warp visits. CTA partials go to a scratch buffer and a second,
// column-parallel launch reduces them in a fixed order (deterministic).
// Statistics are computed in fp32 from the bf16 inputs. The forward can fold
// the residual branch's bias into the residual add (s = x + r + rb), and the
// backward then returns that bias's gradient (column sums of ds) for free.
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
    const __nv_bfloat16* __restrict__ b, const __nv_bfloat16* __restrict__ rb, __nv_bfloat16* __restrict__ y,
    float* __restrict__ mean, float* __restrict__ rstd, int R, int C, float eps) {
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
        if (rb) {
          load8(rb + col, r);
#pragma unroll
          for (int e = 0; e < 8; ++e) v[k][e] += r[e];
        }
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

// Backward rows pass. Each warp walks rows with a one-row software
// prefetch (the next row's dy / x / dres are in flight while the current one
// is reduced); per-lane dgamma / dbeta (and, with DSUM, the column sums of
// dx, which are the bias gradient of the layer that produced the residual
// branch) accumulate in registers, then in shared memory per CTA, and each
// CTA writes one row of partials: part[blockIdx][K * C].
template <int NP, bool DSUM>
__global__ void __launch_bounds__(kLnWarps * 32) k_ln_bwd(
    const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
    const float* __restrict__ mean, const float* __restrict__ rstd,
    const __nv_bfloat16* __restrict__ w, const __nv_bfloat16* __restrict__ dres,
    __nv_bfloat16* __restrict__ dx, float* __restrict__ part, int R, int C) {
  constexpr int K = DSUM ? 3 : 2;
  constexpr bool kPref = NP <= 3;  // wider rows have no registers left for a prefetch
  extern __shared__ float smem[];  // [K][C]
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < K * C; i += blockDim.x) smem[i] = 0.f;
  float aw[NP][8], ab[NP][8], ad[DSUM ? NP : 1][8], wf[NP][8];
#pragma unroll
  for (int k = 0; k < NP; ++k) {
    const int col = (lane + 32 * k) * 8;
#pragma unroll
    for (int e = 0; e < 8; ++e) aw[k][e] = ab[k][e] = 0.f;
    if constexpr (DSUM) {
#pragma unroll
      for (int e = 0; e < 8; ++e) ad[k][e] = 0.f;
    }
    if (col < C) load8(w + col, wf[k]);
  }
  __syncthreads();
  const int wstride = gridDim.x * kLnWarps;
  int row = blockIdx.x * kLnWarps + warp;
  const uint4 z = make_uint4(0, 0, 0, 0);
  uint4 cdy[NP], cx[NP], cr[NP];
#pragma unroll
  for (int k = 0; k < NP; ++k) {
    const int col = (lane + 32 * k) * 8;
    const bool ok = row < R && col < C;
    const size_t off = (size_t)row * C + col;
    cdy[k] = ok ? __ldcs(reinterpret_cast<const uint4*>(dy + off)) : z;
    cx[k] = ok ? __ldcs(reinterpret_cast<const uint4*>(x + off)) : z;
    cr[k] = (ok && dres) ? __ldcs(reinterpret_cast<const uint4*>(dres + off)) : z;
  }
  for (; row < R; row += wstride) {
    const int nrow = row + wstride;
    uint4 ndy[kPref ? NP : 1], nx[kPref ? NP : 1], nr[kPref ? NP : 1];
    if constexpr (kPref) {
#pragma unroll
      for (int k = 0; k < NP; ++k) {
        const int col = (lane + 32 * k) * 8;
        const bool ok = nrow < R && col < C;
        const size_t off = (size_t)nrow * C + col;
        ndy[k] = ok ? __ldcs(reinterpret_cast<const uint4*>(dy + off)) : z;
        nx[k] = ok ? __ldcs(reinterpret_cast<const uint4*>(x + off)) : z;
        nr[k] = (ok && dres) ? __ldcs(reinterpret_cast<const uint4*>(dres + off)) : z;
      }
    }
    const size_t base = (size_t)row * C;
    const float mu = mean[row], rs = rstd[row];
    float g[NP][8], xh[NP][8];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int k = 0; k < NP; ++k) {
      const __nv_bfloat162* hg = reinterpret_cast<const __nv_bfloat162*>(&cdy[k]);
      const __nv_bfloat162* hx = reinterpret_cast<const __nv_bfloat162*>(&cx[k]);
#pragma unroll
      for (int e2 = 0; e2 < 4; ++e2) {
        const float2 gg = __bfloat1622float2(hg[e2]);
        const float2 xx = __bfloat1622float2(hx[e2]);
        g[k][2 * e2] = gg.x;
        g[k][2 * e2 + 1] = gg.y;
        xh[k][2 * e2] = (xx.x - mu) * rs;
        xh[k][2 * e2 + 1] = (xx.y - mu) * rs;
      }
      const int col = (lane + 32 * k) * 8;
      if (col < C) {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
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
          const __nv_bfloat162* hr = reinterpret_cast<const __nv_bfloat162*>(&cr[k]);
#pragma unroll
          for (int e2 = 0; e2 < 4; ++e2) {
            const float2 rr = __bfloat1622float2(hr[e2]);
            o[2 * e2] += rr.x;
            o[2 * e2 + 1] += rr.y;
          }
        }
        // Round to the stored bf16 first so the bias gradient sums exactly
        // what the producing layer receives.
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = __bfloat162float(__float2bfloat16_rn(o[e]));
        if constexpr (DSUM) {
#pragma unroll
          for (int e = 0; e < 8; ++e) ad[k][e] += o[e];
        }
        store8(dx + base + col, o);
      }
      if constexpr (kPref) {
        cdy[k] = ndy[k];
        cx[k] = nx[k];
        cr[k] = nr[k];
      }
    }
    if constexpr (!kPref) {
#pragma unroll
      for (int k = 0; k < NP; ++k) {
        const int col = (lane + 32 * k) * 8;
        const bool ok = nrow < R && col < C;
        const size_t off = (size_t)nrow * C + col;
        cdy[k] = ok ? __ldcs(reinterpret_cast<const uint4*>(dy + off)) : z;
        cx[k] = ok ? __ldcs(reinterpret_cast<const uint4*>(x + off)) : z;
        cr[k] = (ok && dres) ? __ldcs(reinterpret_cast<const uint4*>(dres + off)) : z;
      }
    }
  }
  // CTA partials: warps add their register sums into shared memory.
#pragma unroll
  for (int k = 0; k < NP; ++k) {
    const int col = (lane + 32 * k) * 8;
    if (col < C) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        atomicAdd(&smem[col + e], aw[k][e]);
        atomicAdd(&smem[C + col + e], ab[k][e]);
        if constexpr (DSUM) atomicAdd(&smem[2 * C + col + e], ad[k][e]);
      }
    }
  }
  __syncthreads();
  float* mine = part + (size_t)blockIdx.x * K * C;
  for (int i = threadIdx.x; i < K * C; i += blockDim.x) mine[i] = smem[i];
}

// out_j[c] = sum over P partial rows of part[p][j * C + c] (j < nout), fixed
// order. 256 threads = 32 column groups of 4 x 8 row lanes, shared-memory
// combine of the 8 lanes; one CTA per 128 columns of the K * C partial row.
__global__ void __launch_bounds__(256) k_partials_reduce(const float* __restrict__ part, int P, int W, int C,
                                                         __nv_bfloat16* o0, __nv_bfloat16* o1, __nv_bfloat16* o2,
                                                         int accumulate) {
  __shared__ float4 red[8][32];
  const int cg = threadIdx.x & 31, sl = threadIdx.x >> 5;
  const int col = blockIdx.x * 128 + cg * 4;
  float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
  if (col < W) {
    for (int p = sl; p < P; p += 8) {
      const float4 v = *reinterpret_cast<const float4*>(part + (size_t)p * W + col);
      a.x += v.x; a.y += v.y; a.z += v.z; a.w += v.w;
    }
  }
  red[sl][cg] = a;
  __syncthreads();
  if (sl == 0 && col < W) {
    for (int j = 1; j < 8; ++j) {
      const float4 v = red[j][cg];
      a.x += v.x; a.y += v.y; a.z += v.z; a.w += v.w;
    }
    const int which = col / C, c = col % C;  // C % 4 == 0: a group never straddles outputs
    __nv_bfloat16* o = which == 0 ? o0 : (which == 1 ? o1 : o2);
    if (o) {
      float f[4] = {a.x, a.y, a.z, a.w};
      if (accumulate) {
#pragma unroll
        for (int e = 0; e < 4; ++e) f[e] += __bfloat162float(o[c + e]);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) o[c + e] = __float2bfloat16_rn(f[e]);
    }
  }
}

// Column sums of a bf16 [R, C] matrix, pass 1: CTA (chunk, slab) sums rows of
// its slab for 256 columns (32 groups of 8 columns x 8 row lanes) into
// part[slab][C].
__global__ void __launch_bounds__(256) k_colsum_partial(const __nv_bfloat16* __restrict__ x, long long ldx, int R,
                                                        int C, int rows_per_slab, float* __restrict__ part) {
  __shared__ float red[8][256 + 4];
  const int cg = threadIdx.x & 31, sl = threadIdx.x >> 5;
  const int col = blockIdx.x * 256 + cg * 8;
  const int r0 = blockIdx.y * rows_per_slab;
  const int r1 = min(R, r0 + rows_per_slab);
  float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (col < C) {
#pragma unroll 4
    for (int r = r0 + sl; r < r1; r += 8) {
      float v[8];
      load8(x + (size_t)r * ldx + col, v);
#pragma unroll
      for (int e = 0; e < 8; ++e) a[e] += v[e];
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) red[sl][cg * 8 + e] = a[e];
  __syncthreads();
  const int c = blockIdx.x * 256 + threadIdx.x;
  if (c < C) {
    float t = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) t += red[j][threadIdx.x];
    part[(size_t)blockIdx.y * C + c] = t;
  }
}

inline int reduce_grid(int W) { return (W + 127) / 128; }
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

cudaError_t ln_fwd_ex(const __nv_bfloat16* x, const __nv_bfloat16* res, const __nv_bfloat16* rb,
                      __nv_bfloat16* sum_out, const __nv_bfloat16* w, const __nv_bfloat16* b, __nv_bfloat16* y,
                      float* mean, float* rstd, int R, int C, float eps, cudaStream_t s) {
  if (C % 8 != 0 || (rb && !res)) return cudaErrorInvalidValue;
  const int grid = (R + kLnWarps - 1) / kLnWarps;
  LN_DISPATCH(C, k_ln_fwd<NP><<<grid, kLnWarps * 32, 0, s>>>(x, res, sum_out, w, b, rb, y, mean, rstd, R, C, eps));
  return cudaGetLastError();
}

cudaError_t ln_fwd(const __nv_bfloat16* x, const __nv_bfloat16* res, __nv_bfloat16* sum_out,
                   const __nv_bfloat16* w, const __nv_bfloat16* b, __nv_bfloat16* y, float* mean,
                   float* rstd, int R, int C, float eps, cudaStream_t s) {
  return ln_fwd_ex(x, res, nullptr, sum_out, w, b, y, mean, rstd, R, C, eps, s);
}

int ln_bwd_blocks(int R) {
  int b = (R + kLnWarps * 4 - 1) / (kLnWarps * 4);
  return b < 1 ? 1 : (b > 148 ? 148 : b);
}
size_t ln_bwd_scratch_floats(int C, int blocks) { return (size_t)blocks * 2 * C; }
size_t ln_bwd_scratch_floats_ex(int C, int blocks, bool dsum) { return (size_t)blocks * (dsum ? 3 : 2) * C; }

cudaError_t ln_bwd_ex(const __nv_bfloat16* dy, const __nv_bfloat16* x, const float* mean, const float* rstd,
                      const __nv_bfloat16* w, const __nv_bfloat16* dres, __nv_bfloat16* dx, __nv_bfloat16* dw,
                      __nv_bfloat16* db, __nv_bfloat16* dsum, float* scratch, int R, int C, int blocks,
                      cudaStream_t s) {
  if (C % 8 != 0) return cudaErrorInvalidValue;
  const int K = dsum ? 3 : 2;
  const size_t shm = (size_t)K * C * sizeof(float);
  if (dsum) {
    LN_DISPATCH(C, k_ln_bwd<NP, true><<<blocks, kLnWarps * 32, shm, s>>>(dy, x, mean, rstd, w, dres, dx, scratch, R, C));
  } else {
    LN_DISPATCH(C, k_ln_bwd<NP, false><<<blocks, kLnWarps * 32, shm, s>>>(dy, x, mean, rstd, w, dres, dx, scratch, R, C));
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  k_partials_reduce<<<reduce_grid(K * C), 256, 0, s>>>(scratch, blocks, K * C, C, dw, db, dsum, 0);
  return cudaGetLastError();
}

cudaError_t ln_bwd(const __nv_bfloat16* dy, const __nv_bfloat16* x, const float* mean,
                   const float* rstd, const __nv_bfloat16* w, const __nv_bfloat16* dres,
                   __nv_bfloat16* dx, __nv_bfloat16* dw, __nv_bfloat16* db, float* scratch,
                   unsigned int* counter, int R, int C, int blocks, cudaStream_t s) {
  (void)counter;  // kept for the C ABI; the reduction is a second launch now
  return ln_bwd_ex(dy, x, mean, rstd, w, dres, dx, dw, db, nullptr, scratch, R, C, blocks, s);
}

int colsum_slabs(int R) {
  int sl = (R + 127) / 128;
  return sl < 1 ? 1 : (sl > 64 ? 64 : sl);
}

cudaError_t colsum_bf16(const __nv_bfloat16* x, long long ldx, int R, int C, __nv_bfloat16* out, bool accumulate,
                        float* scratch, cudaStream_t s) {
  if (C % 8 != 0 || (ldx % 8) != 0) return cudaErrorInvalidValue;
  const int slabs = colsum_slabs(R);
  const int rps = (R + slabs - 1) / slabs;
  dim3 grid((C + 255) / 256, slabs);
  k_colsum_partial<<<grid, 256, 0, s>>>(x, ldx, R, C, rps, scratch);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  k_partials_reduce<<<reduce_grid(C), 256, 0, s>>>(scratch, slabs, C, C, out, nullptr, nullptr, accumulate ? 1 : 0);
  return cudaGetLastError();
}

}  // namespace nexar
