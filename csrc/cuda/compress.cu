// Gradient compression for the all-reduce (sm_100a): error feedback, top-k
// selection by magnitude, fp8 (e4m3) quantisation, and decompress-accumulate.
//
// Pipeline for one call (all kernels stream over the dense gradient; nothing
// is sorted):
//   1. hist1   r = residual + grad (fp32, never stored); 4096-bin histogram of
//              the top 12 bits of |r|'s fp32 bit pattern, and the max |r|.
//   2. pick    single block: the bin where the count from the top reaches k.
//   3. hist2   same for the next 12 bits inside that bin.
//   4. pick    the 24-bit key prefix P of the k-th largest magnitude.
//   5. count   per block: elements with prefix > P ("above") and == P ("tie").
//   6. scan    single block: output offsets per block; ties are taken in index
//              order until exactly k elements are selected.
//   7. compact per block, order-preserving: selected (index, e4m3(r/scale))
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

struct SelState {
  unsigned int maxkey;      // max fp32 bit pattern of |r|
  unsigned int bin1, bin2;  // chosen bins
  unsigned long long above1;  // elements in bins above bin1
  unsigned long long above;   // elements with 24-bit prefix above P
  unsigned long long need_tie;  // ties to take (in index order)
};

NEXAR_D float ef_value(const __nv_bfloat16* g, const float* res, unsigned long long i) {
  return res[i] + __bfloat162float(g[i]);
}
NEXAR_D unsigned int key_of(float r) { return __float_as_uint(fabsf(r)); }

__global__ void __launch_bounds__(kCThreads) k_hist1(const __nv_bfloat16* __restrict__ g, const float* __restrict__ res,
                                                     unsigned long long n, unsigned int* __restrict__ hist,
                                                     SelState* st) {
  __shared__ unsigned int h[kBins];
  __shared__ unsigned int smax;
  for (int i = threadIdx.x; i < kBins; i += blockDim.x) h[i] = 0;
  if (threadIdx.x == 0) smax = 0;
  __syncthreads();
  unsigned int lmax = 0;
  for (unsigned long long i = blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x; i < n;
       i += (unsigned long long)gridDim.x * blockDim.x) {
    const unsigned int k = key_of(ef_value(g, res, i));
    atomicAdd(&h[k >> 20], 1u);
    lmax = max(lmax, k);
  }
  atomicMax(&smax, lmax);
  __syncthreads();
  for (int i = threadIdx.x; i < kBins; i += blockDim.x)
    if (h[i]) atomicAdd(&hist[i], h[i]);
  if (threadIdx.x == 0) atomicMax(&st->maxkey, smax);
}

__global__ void __launch_bounds__(kCThreads) k_hist2(const __nv_bfloat16* __restrict__ g, const float* __restrict__ res,
                                                     unsigned long long n, unsigned int* __restrict__ hist,
                                                     const SelState* st) {
  __shared__ unsigned int h[kBins];
  for (int i = threadIdx.x; i < kBins; i += blockDim.x) h[i] = 0;
  __syncthreads();
  const unsigned int b1 = st->bin1;
  for (unsigned long long i = blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x; i < n;
       i += (unsigned long long)gridDim.x * blockDim.x) {
    const unsigned int k = key_of(ef_value(g, res, i));
    if ((k >> 20) == b1) atomicAdd(&h[(k >> 8) & 0xFFFu], 1u);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < kBins; i += blockDim.x)
    if (h[i]) atomicAdd(&hist[i], h[i]);
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

NEXAR_D unsigned int prefix_of(float r) { return key_of(r) >> 8; }

// Per-block counts of "above" and "tie" elements over a contiguous range.
__global__ void __launch_bounds__(kCThreads) k_count(const __nv_bfloat16* __restrict__ g, const float* __restrict__ res,
                                                     unsigned long long n, unsigned long long per_block,
                                                     const SelState* st, unsigned int* __restrict__ blk_above,
                                                     unsigned int* __restrict__ blk_tie) {
  const unsigned int P = (st->bin1 << 12) | st->bin2;
  const unsigned long long lo = blockIdx.x * per_block, hi = min(n, lo + per_block);
  unsigned int a = 0, t = 0;
  for (unsigned long long i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    const unsigned int p = prefix_of(ef_value(g, res, i));
    a += p > P;
    t += p == P;
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

// Single block exclusive scan: output offset per block and the ties it takes.
__global__ void __launch_bounds__(1024) k_scan_blocks(const unsigned int* __restrict__ blk_above,
                                                      const unsigned int* __restrict__ blk_tie, int nblk,
                                                      const SelState* st, unsigned long long* __restrict__ blk_off,
                                                      unsigned int* __restrict__ blk_take) {
  if (threadIdx.x != 0) return;
  unsigned long long off = 0, ties_before = 0;
  const unsigned long long need = st->need_tie;
  for (int b = 0; b < nblk; ++b) {
    const unsigned long long avail = need > ties_before ? need - ties_before : 0;
    const unsigned long long tie_b = blk_tie[b];
    const unsigned int take = (unsigned int)(avail < tie_b ? avail : tie_b);
    blk_off[b] = off;
    blk_take[b] = take;
    off += blk_above[b] + take;
    ties_before += blk_tie[b];
  }
}

// Order-preserving compaction; writes the residual for every element.
__global__ void __launch_bounds__(kCThreads) k_compact(const __nv_bfloat16* __restrict__ g, float* __restrict__ res,
                                                       unsigned long long n, unsigned long long per_block,
                                                       const SelState* st, const unsigned long long* __restrict__ blk_off,
                                                       const unsigned int* __restrict__ blk_take,
                                                       unsigned int* __restrict__ out_idx,
                                                       __nv_fp8_e4m3* __restrict__ out_val, float* scale_out) {
  const unsigned int P = (st->bin1 << 12) | st->bin2;
  const float maxv = __uint_as_float(st->maxkey);
  const float scale = maxv > 0.f ? maxv / 448.f : 1.f;
  const float inv = 1.f / scale;
  if (blockIdx.x == 0 && threadIdx.x == 0) *scale_out = scale;
  const unsigned long long lo = blockIdx.x * per_block, hi = min(n, lo + per_block);
  __shared__ unsigned int wsum[kCThreads / 32];
  __shared__ unsigned int wtie[kCThreads / 32];
  unsigned long long base = blk_off[blockIdx.x];
  unsigned int ties_left = blk_take[blockIdx.x];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (unsigned long long t0 = lo; t0 < hi; t0 += blockDim.x) {
    const unsigned long long i = t0 + threadIdx.x;
    float r = 0.f;
    unsigned int p = 0;
    const bool valid = i < hi;
    if (valid) {
      r = ef_value(g, res, i);
      p = prefix_of(r);
    }
    const bool above = valid && p > P;
    const bool tie = valid && p == P;
    // ties are taken in index order: rank of this tie among the tile's ties
    const unsigned int tb = __ballot_sync(0xffffffffu, tie);
    const unsigned int tie_rank_w = __popc(tb & ((1u << lane) - 1));
    if (lane == 0) wtie[warp] = __popc(tb);
    __syncthreads();
    unsigned int tie_before = 0, ties_tile = 0;
    for (int w = 0; w < kCThreads / 32; ++w) {
      if (w < warp) tie_before += wtie[w];
      ties_tile += wtie[w];
    }
    const bool take = above || (tie && tie_before + tie_rank_w < ties_left);
    const unsigned int sb = __ballot_sync(0xffffffffu, take);
    const unsigned int sel_rank_w = __popc(sb & ((1u << lane) - 1));
    if (lane == 0) wsum[warp] = __popc(sb);
    __syncthreads();
    unsigned int sel_before = 0, sel_tile = 0;
    for (int w = 0; w < kCThreads / 32; ++w) {
      if (w < warp) sel_before += wsum[w];
      sel_tile += wsum[w];
    }
    if (take) {
      const unsigned long long pos = base + sel_before + sel_rank_w;
      const __nv_fp8_e4m3 q(r * inv);
      out_idx[pos] = (unsigned int)i;
      out_val[pos] = q;
      res[i] = r - static_cast<float>(q) * scale;
    } else if (valid) {
      res[i] = r;
    }
    base += sel_tile;
    ties_left -= min(ties_left, ties_tile);
    __syncthreads();
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

inline int grid_for(unsigned long long n) {
  unsigned long long b = (n + kCThreads - 1) / kCThreads;
  if (b > 148 * 8) b = 148 * 8;
  return (int)(b < 1 ? 1 : b);
}
}  // namespace

size_t compress_workspace_bytes(unsigned long long n, int* nblk_out) {
  const unsigned long long per = 1ull << 18;  // elements per compaction block
  const int nblk = (int)((n + per - 1) / per);
  if (nblk_out) *nblk_out = nblk;
  return 256 + 2 * kBins * sizeof(unsigned int) + (size_t)nblk * (4 + 4 + 8 + 4);
}

size_t compress_blob_bytes(unsigned long long k) { return 16 + 5 * k; }

cudaError_t topk_fp8_compress(const __nv_bfloat16* grad, float* residual, unsigned long long n, unsigned long long k,
                              unsigned char* blob, void* ws, cudaStream_t s) {
  if (k == 0 || k > n || k > 0xffffffffull) return cudaErrorInvalidValue;
  int nblk = 0;
  compress_workspace_bytes(n, &nblk);
  const unsigned long long per = 1ull << 18;
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
  const int grid = grid_for(n);
  k_hist1<<<grid, kCThreads, 0, s>>>(grad, residual, n, h1, st);
  k_pick<<<1, 1024, 0, s>>>(h1, st, k, 1);
  k_hist2<<<grid, kCThreads, 0, s>>>(grad, residual, n, h2, st);
  k_pick<<<1, 1024, 0, s>>>(h2, st, k, 2);
  k_count<<<nblk, kCThreads, 0, s>>>(grad, residual, n, per, st, blk_above, blk_tie);
  k_scan_blocks<<<1, 1024, 0, s>>>(blk_above, blk_tie, nblk, st, blk_off, blk_take);
  k_compact<<<nblk, kCThreads, 0, s>>>(grad, residual, n, per, st, blk_off, blk_take,
                                       reinterpret_cast<unsigned int*>(blob + 16),
                                       reinterpret_cast<__nv_fp8_e4m3*>(blob + 16 + 4 * k),
                                       reinterpret_cast<float*>(blob));
  return cudaGetLastError();
}

cudaError_t decompress_accumulate(const unsigned char* blob, unsigned long long k, __nv_bfloat16* out, float out_scale,
                                  cudaStream_t s) {
  k_decompress_acc<<<grid_for(k), kCThreads, 0, s>>>(blob, k, out, out_scale);
  return cudaGetLastError();
}

int compress_kernel_launches() { return 8; }

}  // namespace nexar
