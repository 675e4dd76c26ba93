// Gradient compression for the all-reduce (sm_100a): error feedback, top-k
// selection by magnitude, fp8 (e4m3) quantisation, and decompress-accumulate.
//
// Pipeline for one call (all kernels stream over the dense gradient; nothing
// is sorted):
//   1. hist1   r = residual + grad (fp32, never stored); 4096-bin histogram of
//              the top 12 bits of |r|'s fp32 bit pattern (warp-aggregated
//              shared atomics), and the max |r|.
//   2. pick    single block: the bin where the count from the top reaches k.
//   3. hist2   same for the next 12 bits inside that bin.
//   4. pick    the 24-bit key prefix P of the k-th largest magnitude.
//   5. count   per 64 Ki-element block: elements with prefix > P ("above") and
//              == P ("tie").
//   6. scan    single block: output offsets per block; ties are taken in index
//              order until exactly k elements are selected.
//   7. compact per block, order-preserving (one block-wide scan per 4096
//              elements, 8 consecutive elements per thread): selected (index, e4m3(r/scale))
//              pairs land in the blob in ascending index order; the residual
//              keeps r minus what was sent (the quantisation error included)
//              and all of r elsewhere.
// The blob is [scale f32 | pad to 16 B][k x u32 index][k x e4m3 value]. Blobs
// of all ranks are exchanged with the device all-gather (all blobs have the
// same k) and decompress_accumulate adds them into the dense output in rank
// order (deterministic). Selection is exact up to elements whose magnitudes
// agree in the top 24 bits of the fp32 pattern (relative difference < 2^-15):
// among those the lower index wins, like the reference's tie rule
// (nexar/src/compression/topk.rs keeps the k largest |residual|).
#include "common.cuh"
#include "compress_api.h"

namespace nexar {

namespace {
constexpr int kCThreads = 512;
constexpr int kBins = 4096;
constexpr int kGroup = 8;                          // contiguous elements per thread per step
constexpr int kTile = kCThreads * kGroup;          // 4096 elements per block step
constexpr unsigned long long kPerBlock = 1ull << 16;  // elements per count / compact block

struct SelState {
  unsigned int maxkey;      // max fp32 bit pattern of |r|
  unsigned int bin1, bin2;  // chosen bins
  unsigned long long above1;  // elements in bins above bin1
  unsigned long long above;   // elements with 24-bit prefix above P
  unsigned long long need_tie;  // ties to take (in index order)
};

NEXAR_D unsigned int key_of(float r) { return __float_as_uint(fabsf(r)); }
NEXAR_D unsigned int prefix_of(float r) { return key_of(r) >> 8; }

// r = residual + grad for the 8 elements starting at i; lanes past n read 0
// (callers test the index). VEC: g and res are 16-byte aligned and i is a
// multiple of 8, so a full group is one 16-byte and two 16-byte loads.
template <bool VEC>
NEXAR_D void load_group(const __nv_bfloat16* __restrict__ g, const float* res, unsigned long long i,
                        unsigned long long n, float (&r)[kGroup]) {
  if (VEC && i + kGroup <= n) {
    const uint4 gv = ld16_nc(g + i);
    const float4 a = *reinterpret_cast<const float4*>(res + i);
    const float4 b = *reinterpret_cast<const float4*>(res + i + 4);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&gv);
    const float2 g0 = __bfloat1622float2(h[0]), g1 = __bfloat1622float2(h[1]);
    const float2 g2 = __bfloat1622float2(h[2]), g3 = __bfloat1622float2(h[3]);
    r[0] = a.x + g0.x; r[1] = a.y + g0.y; r[2] = a.z + g1.x; r[3] = a.w + g1.y;
    r[4] = b.x + g2.x; r[5] = b.y + g2.y; r[6] = b.z + g3.x; r[7] = b.w + g3.y;
  } else {
#pragma unroll
    for (int j = 0; j < kGroup; ++j) r[j] = i + j < n ? res[i + j] + __bfloat162float(g[i + j]) : 0.f;
  }
}

template <bool VEC>
NEXAR_D void store_group(float* res, unsigned long long i, unsigned long long n, const float (&r)[kGroup]) {
  if (VEC && i + kGroup <= n) {
    *reinterpret_cast<float4*>(res + i) = make_float4(r[0], r[1], r[2], r[3]);
    *reinterpret_cast<float4*>(res + i + 4) = make_float4(r[4], r[5], r[6], r[7]);
  } else {
#pragma unroll
    for (int j = 0; j < kGroup; ++j)
      if (i + j < n) res[i + j] = r[j];
  }
}

// Warp-aggregated shared histogram add: lanes holding the same bin elect one
// leader that adds the group's count (gradients with many equal values, e.g.
// zero rows of an embedding, would otherwise serialise 32-way on one bin).
// Called by all 32 lanes; `valid` false lanes add nothing.
NEXAR_D void warp_hist_add(unsigned int* h, unsigned int bin, bool valid) {
  const unsigned int key = valid ? bin : 0xFFFFFFFFu;
  const unsigned int peers = __match_any_sync(0xffffffffu, key);
  if (valid && (__ffs(peers) - 1) == (int)(threadIdx.x & 31)) atomicAdd(&h[bin], (unsigned int)__popc(peers));
}

// Histogram of the top 12 bits of |r| (stage 1) or of the next 12 bits of the
// elements in bin1 (stage 2). The grid-stride loop is warp-uniform so every
// lane reaches the warp-aggregated add; each thread keeps two groups in flight.
template <bool VEC, int STAGE>
__global__ void __launch_bounds__(kCThreads) k_hist(const __nv_bfloat16* __restrict__ g, const float* __restrict__ res,
                                                    unsigned long long n, unsigned int* __restrict__ hist,
                                                    SelState* st) {
  __shared__ unsigned int h[kBins];
  __shared__ unsigned int smax;
  for (int i = threadIdx.x; i < kBins; i += blockDim.x) h[i] = 0;
  if (threadIdx.x == 0) smax = 0;
  __syncthreads();
  const unsigned int b1 = STAGE == 2 ? st->bin1 : 0u;
  const unsigned long long ngroups = (n + kGroup - 1) / kGroup;
  const unsigned long long stride = (unsigned long long)gridDim.x * blockDim.x;
  const unsigned int lane = threadIdx.x & 31;
  unsigned int lmax = 0;
  for (unsigned long long w0 = blockIdx.x * (unsigned long long)blockDim.x + (threadIdx.x & ~31u); w0 < ngroups;
       w0 += 2 * stride) {
    float r[2][kGroup];
    unsigned long long gi[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      gi[u] = w0 + u * stride + lane;
      if (gi[u] < ngroups) load_group<VEC>(g, res, gi[u] * kGroup, n, r[u]);
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
#pragma unroll
      for (int j = 0; j < kGroup; ++j) {
        const bool in_range = gi[u] < ngroups && gi[u] * kGroup + j < n;
        const unsigned int k = in_range ? key_of(r[u][j]) : 0u;
        if (STAGE == 1) {
          lmax = max(lmax, k);
          warp_hist_add(h, k >> 20, in_range);
        } else {
          const bool in = in_range && (k >> 20) == b1;
          if (__ballot_sync(0xffffffffu, in)) warp_hist_add(h, (k >> 8) & 0xFFFu, in);
        }
      }
    }
  }
  if (STAGE == 1) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) lmax = max(lmax, __shfl_xor_sync(0xffffffffu, lmax, o));
    if (lane == 0) atomicMax(&smax, lmax);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < kBins; i += blockDim.x)
    if (h[i]) atomicAdd(&hist[i], h[i]);
  if (STAGE == 1 && threadIdx.x == 0) atomicMax(&st->maxkey, smax);
}

// Single block: walk bins from the top until the running count reaches `need`.
__global__ void __launch_bounds__(1024) k_pick(const unsigned int* __restrict__ hist, SelState* st,
                                               unsigned long long k, int stage) {
  __shared__ unsigned long long chunk_sum[1024];
  // each thread sums 4 consecutive bins, counted from the top
  const int t = threadIdx.x;
  unsigned long long s = 0;
  for (int j = 0; j < 4; ++j) s += hist[kBins - 1 - (t * 4 + j)];
  chunk_sum[t] = s;
  __syncthreads();
  if (t == 0) {
    const unsigned long long need = stage == 1 ? k : k - st->above1;
    unsigned long long run = 0;
    int bin = 0;
    for (int c = 0; c < 1024; ++c) {
      if (run + chunk_sum[c] >= need) {
        for (int j = 0; j < 4; ++j) {
          const int b = kBins - 1 - (c * 4 + j);
          if (run + hist[b] >= need) {
            bin = b;
            break;
          }
          run += hist[b];
        }
        break;
      }
      run += chunk_sum[c];
    }
    if (stage == 1) {
      st->bin1 = bin;
      st->above1 = run;
    } else {
      st->bin2 = bin;
      st->above = st->above1 + run;
      st->need_tie = k - st->above;
    }
  }
}

// Per-block counts of "above" and "tie" elements over a contiguous range of
// kPerBlock elements (thread t of a step owns 8 consecutive elements).
template <bool VEC>
__global__ void __launch_bounds__(kCThreads) k_count(const __nv_bfloat16* __restrict__ g, const float* __restrict__ res,
                                                     unsigned long long n, const SelState* st,
                                                     unsigned int* __restrict__ blk_above,
                                                     unsigned int* __restrict__ blk_tie) {
  const unsigned int P = (st->bin1 << 12) | st->bin2;
  const unsigned long long lo = blockIdx.x * kPerBlock, hi = min(n, lo + kPerBlock);
  unsigned int a = 0, t = 0;
  for (unsigned long long t0 = lo; t0 < hi; t0 += 2 * kTile) {
    float r[2][kGroup];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const unsigned long long i = t0 + u * kTile + threadIdx.x * kGroup;
      if (i < hi) load_group<VEC>(g, res, i, hi, r[u]);
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const unsigned long long i = t0 + u * kTile + threadIdx.x * kGroup;
#pragma unroll
      for (int j = 0; j < kGroup; ++j) {
        if (i + j < hi) {
          const unsigned int p = prefix_of(r[u][j]);
          a += p > P;
          t += p == P;
        }
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a += __shfl_xor_sync(0xffffffffu, a, o);
    t += __shfl_xor_sync(0xffffffffu, t, o);
  }
  __shared__ unsigned int sa[kCThreads / 32], stt[kCThreads / 32];
  if ((threadIdx.x & 31) == 0) {
    sa[threadIdx.x >> 5] = a;
    stt[threadIdx.x >> 5] = t;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned int A = 0, T = 0;
    for (int w = 0; w < kCThreads / 32; ++w) {
      A += sa[w];
      T += stt[w];
    }
    blk_above[blockIdx.x] = A;
    blk_tie[blockIdx.x] = T;
  }
}

// Single block: output offset per compaction block and the ties it takes.
// Ties are taken in index order, so with T ties before a block and `need` in
// total, the block takes min(need, T + tie_b) - min(need, T) of its own and
// starts at above_before + min(need, T). Thread t owns a contiguous chunk of
// blocks; one block-wide exclusive scan of (above, tie) sums links the chunks.
__global__ void __launch_bounds__(1024) k_scan_blocks(const unsigned int* __restrict__ blk_above,
                                                      const unsigned int* __restrict__ blk_tie, int nblk,
                                                      const SelState* st, unsigned long long* __restrict__ blk_off,
                                                      unsigned int* __restrict__ blk_take) {
  __shared__ unsigned long long wa[32], wt[32];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int per = (nblk + blockDim.x - 1) / blockDim.x;
  const int b0 = min(nblk, t * per), b1 = min(nblk, b0 + per);
  unsigned long long A = 0, T = 0;
  for (int b = b0; b < b1; ++b) {
    A += blk_above[b];
    T += blk_tie[b];
  }
  // inclusive warp scan, then scan of the warp totals
  unsigned long long ia = A, it = T;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long xa = __shfl_up_sync(0xffffffffu, ia, o);
    const unsigned long long xt = __shfl_up_sync(0xffffffffu, it, o);
    if (lane >= o) {
      ia += xa;
      it += xt;
    }
  }
  if (lane == 31) {
    wa[warp] = ia;
    wt[warp] = it;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    unsigned long long va = lane < nw ? wa[lane] : 0, vt = lane < nw ? wt[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned long long xa = __shfl_up_sync(0xffffffffu, va, o);
      const unsigned long long xt = __shfl_up_sync(0xffffffffu, vt, o);
      if (lane >= o) {
        va += xa;
        vt += xt;
      }
    }
    if (lane < nw) {
      wa[lane] = va - (lane < nw ? wa[lane] : 0);  // exclusive
      wt[lane] = vt - (lane < nw ? wt[lane] : 0);
    }
  }
  __syncthreads();
  unsigned long long a_before = wa[warp] + ia - A, t_before = wt[warp] + it - T;
  const unsigned long long need = st->need_tie;
  for (int b = b0; b < b1; ++b) {
    const unsigned long long lo = min(need, t_before), hi = min(need, t_before + blk_tie[b]);
    blk_off[b] = a_before + lo;
    blk_take[b] = (unsigned int)(hi - lo);
    a_before += blk_above[b];
    t_before += blk_tie[b];
  }
}

// Order-preserving compaction of one kPerBlock range; writes the residual for
// every element. Each 4096-element step: thread t classifies its 8
// consecutive elements, one block-wide exclusive scan of the packed counts
// (ties << 16 | above; at most 4096 each) gives the thread's first output slot
// base + above_before + min(ties_left, ties_before), and the thread writes its
// selections in index order. The next step's loads are issued before the scan.
template <bool VEC>
__global__ void __launch_bounds__(kCThreads) k_compact(const __nv_bfloat16* __restrict__ g, float* __restrict__ res,
                                                       unsigned long long n, const SelState* st,
                                                       const unsigned long long* __restrict__ blk_off,
                                                       const unsigned int* __restrict__ blk_take,
                                                       unsigned int* __restrict__ out_idx,
                                                       __nv_fp8_e4m3* __restrict__ out_val, float* scale_out) {
  const unsigned int P = (st->bin1 << 12) | st->bin2;
  const float maxv = __uint_as_float(st->maxkey);
  const float scale = maxv > 0.f ? maxv / 448.f : 1.f;
  const float inv = 1.f / scale;
  if (blockIdx.x == 0 && threadIdx.x == 0) *scale_out = scale;
  const unsigned long long lo = blockIdx.x * kPerBlock, hi = min(n, lo + kPerBlock);
  __shared__ unsigned int wtot[2][kCThreads / 32];
  unsigned long long base = blk_off[blockIdx.x];
  unsigned int ties_left = blk_take[blockIdx.x];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float cur[kGroup] = {}, nxt[kGroup] = {};
  {
    const unsigned long long i = lo + threadIdx.x * kGroup;
    if (i < hi) load_group<VEC>(g, res, i, hi, cur);
  }
  int par = 0;
  for (unsigned long long t0 = lo; t0 < hi; t0 += kTile, par ^= 1) {
    const unsigned long long i = t0 + threadIdx.x * kGroup;
    {
      const unsigned long long inext = i + kTile;
      if (inext < hi) load_group<VEC>(g, res, inext, hi, nxt);
    }
    unsigned int na = 0, nt = 0, cls = 0;  // cls: 2 bits per element, 1 above, 2 tie
#pragma unroll
    for (int j = 0; j < kGroup; ++j) {
      if (i + j < hi) {
        const unsigned int p = prefix_of(cur[j]);
        if (p > P) {
          ++na;
          cls |= 1u << (2 * j);
        } else if (p == P) {
          ++nt;
          cls |= 2u << (2 * j);
        }
      }
    }
    const unsigned int mine = (nt << 16) | na;
    unsigned int incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned int x = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += x;
    }
    if (lane == 31) wtot[par][warp] = incl;
    __syncthreads();
    unsigned int before = incl - mine, total = 0;
#pragma unroll
    for (int w = 0; w < kCThreads / 32; ++w) {
      const unsigned int v = wtot[par][w];
      if (w < warp) before += v;
      total += v;
    }
    const unsigned int a_before = before & 0xFFFFu, t_before = before >> 16;
    if (cls != 0u) {
      unsigned long long pos = base + a_before + min(ties_left, t_before);
      unsigned int tie_rank = t_before;
#pragma unroll
      for (int j = 0; j < kGroup; ++j) {
        const unsigned int c = (cls >> (2 * j)) & 3u;
        bool take = c == 1u;
        if (c == 2u) take = tie_rank++ < ties_left;
        if (take) {
          const __nv_fp8_e4m3 q(cur[j] * inv);
          out_idx[pos] = (unsigned int)(i + j);
          out_val[pos] = q;
          ++pos;
          cur[j] -= static_cast<float>(q) * scale;
        }
      }
    }
    if (i < hi) store_group<VEC>(res, i, hi, cur);
    const unsigned int tot_a = total & 0xFFFFu, tot_t = total >> 16;
    base += tot_a + min(ties_left, tot_t);
    ties_left -= min(ties_left, tot_t);
#pragma unroll
    for (int j = 0; j < kGroup; ++j) cur[j] = nxt[j];
  }
}
// out[idx] (+)= e4m3 * scale for one rank's blob.
__global__ void __launch_bounds__(kCThreads) k_decompress_acc(const unsigned char* __restrict__ blob,
                                                              unsigned long long k, __nv_bfloat16* __restrict__ out,
                                                              float out_scale) {
  const float scale = *reinterpret_cast<const float*>(blob);
  const unsigned int* idx = reinterpret_cast<const unsigned int*>(blob + 16);
  const __nv_fp8_e4m3* val = reinterpret_cast<const __nv_fp8_e4m3*>(blob + 16 + 4 * k);
  for (unsigned long long j = blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x; j < k;
       j += (unsigned long long)gridDim.x * blockDim.x) {
    const unsigned int i = idx[j];
    const float v = static_cast<float>(val[j]) * scale * out_scale;
    out[i] = __float2bfloat16_rn(__bfloat162float(out[i]) + v);
  }
}

int sm_count() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

// Blocks for n threads' worth of work, capped at one resident wave of `kern`
// (the histogram passes are grid-stride loops).
template <class Kern>
int grid_for(unsigned long long n, Kern kern) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kCThreads, 0) != cudaSuccess || per_sm <= 0)
    per_sm = 1;
  unsigned long long b = (n + kCThreads - 1) / kCThreads;
  const unsigned long long cap = (unsigned long long)sm_count() * per_sm;
  if (b > cap) b = cap;
  return (int)(b < 1 ? 1 : b);
}

template <bool VEC>
cudaError_t run_select(const __nv_bfloat16* grad, float* residual, unsigned long long n, unsigned long long k,
                       unsigned char* blob, SelState* st, unsigned int* h1, unsigned int* h2,
                       unsigned int* blk_above, unsigned int* blk_tie, unsigned long long* blk_off,
                       unsigned int* blk_take, int nblk, cudaStream_t s) {
  // two groups of 8 per thread per iteration of the histogram passes
  const unsigned long long work = (n + 2 * kGroup - 1) / (2 * kGroup);
  k_hist<VEC, 1><<<grid_for(work, k_hist<VEC, 1>), kCThreads, 0, s>>>(grad, residual, n, h1, st);
  k_pick<<<1, 1024, 0, s>>>(h1, st, k, 1);
  k_hist<VEC, 2><<<grid_for(work, k_hist<VEC, 2>), kCThreads, 0, s>>>(grad, residual, n, h2, st);
  k_pick<<<1, 1024, 0, s>>>(h2, st, k, 2);
  k_count<VEC><<<nblk, kCThreads, 0, s>>>(grad, residual, n, st, blk_above, blk_tie);
  k_scan_blocks<<<1, 1024, 0, s>>>(blk_above, blk_tie, nblk, st, blk_off, blk_take);
  k_compact<VEC><<<nblk, kCThreads, 0, s>>>(grad, residual, n, st, blk_off, blk_take,
                                            reinterpret_cast<unsigned int*>(blob + 16),
                                            reinterpret_cast<__nv_fp8_e4m3*>(blob + 16 + 4 * k),
                                            reinterpret_cast<float*>(blob));
  return cudaGetLastError();
}
}  // namespace

size_t compress_workspace_bytes(unsigned long long n, int* nblk_out) {
  const int nblk = (int)((n + kPerBlock - 1) / kPerBlock);
  if (nblk_out) *nblk_out = nblk;
  return 256 + 2 * kBins * sizeof(unsigned int) + (size_t)nblk * (4 + 4 + 8 + 4) + 8;
}

size_t compress_blob_bytes(unsigned long long k) { return 16 + 5 * k; }

cudaError_t topk_fp8_compress(const __nv_bfloat16* grad, float* residual, unsigned long long n, unsigned long long k,
                              unsigned char* blob, void* ws, cudaStream_t s) {
  if (k == 0 || k > n || k > 0xffffffffull) return cudaErrorInvalidValue;
  int nblk = 0;
  compress_workspace_bytes(n, &nblk);
  char* w = static_cast<char*>(ws);
  SelState* st = reinterpret_cast<SelState*>(w);
  unsigned int* h1 = reinterpret_cast<unsigned int*>(w + 256);
  unsigned int* h2 = h1 + kBins;
  unsigned int* blk_above = h2 + kBins;
  unsigned int* blk_tie = blk_above + nblk;
  unsigned long long* blk_off = reinterpret_cast<unsigned long long*>(
      (reinterpret_cast<uintptr_t>(blk_tie + nblk) + 7) & ~uintptr_t(7));
  unsigned int* blk_take = reinterpret_cast<unsigned int*>(blk_off + nblk);
  cudaError_t e = cudaMemsetAsync(w, 0, 256 + 2 * kBins * sizeof(unsigned int), s);
  if (e != cudaSuccess) return e;
  const bool vec = (reinterpret_cast<uintptr_t>(grad) % 16 == 0) && (reinterpret_cast<uintptr_t>(residual) % 16 == 0);
  return vec ? run_select<true>(grad, residual, n, k, blob, st, h1, h2, blk_above, blk_tie, blk_off, blk_take, nblk, s)
             : run_select<false>(grad, residual, n, k, blob, st, h1, h2, blk_above, blk_tie, blk_off, blk_take, nblk, s);
}

cudaError_t decompress_accumulate(const unsigned char* blob, unsigned long long k, __nv_bfloat16* out, float out_scale,
                                  cudaStream_t s) {
  k_decompress_acc<<<grid_for(k, k_decompress_acc), kCThreads, 0, s>>>(blob, k, out, out_scale);
  return cudaGetLastError();
}

int compress_kernel_launches() { return 8; }

}  // namespace nexar
