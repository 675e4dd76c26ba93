// NVLS collectives: reductions and broadcasts done inside the NVSwitch.
//
// The communicator's NVLS region is physical memory on every GPU bound to one
// multicast object (nvls.cpp). `nvls_mc + off` names offset `off` on ALL ranks
// at once:
//   multimem.ld_reduce.add  returns the sum over every rank's copy (the switch
//                           reads and adds; bf16/f16 accumulate in fp32),
//   multimem.st             writes one value into every rank's copy,
//   multimem.red.add        atomically adds into every rank's copy (signals).
// Compared with the peer-to-peer two-shot all-reduce (each rank pulls W-1
// slices, then pushes W-1 slices) each byte crosses this GPU's NVLink ports
// about half as often.
//
// Work is cut into rounds. In round j, block b owns one chunk and the chunk
// is split into W sub-slices; rank r reduces sub-slice r. Each round is
//   [copy in] -> signal/wait A -> multimem work -> signal/wait B -> [copy out]
// Signals are per-block u32 counters in the region's signal pad, bumped on
// every rank by one multimem.red.release from each rank, so after round k a
// block's counter equals W * k on every GPU. The expected value comes from a
// per-block round counter in local device memory (nvls_seq), advanced
// identically on every rank, so CUDA graph replays keep working. Block b
// always uses staging chunk b, which makes reuse across rounds and calls safe:
// nobody writes chunk b of round j+1 before every rank passed wait B of round
// j for block b. Every wait is bounded by timeout_ns and records the failure
// in the status word.
#include "coll.cuh"
#include "coll_api.h"
#include "nvls_api.h"

namespace nexar {

namespace {

constexpr int kNvlsThreads = 512;

NEXAR_D unsigned int* nvls_flag(char* base, int block, int phase) {
  return reinterpret_cast<unsigned int*>(base + (size_t)block * 64 + phase * 4);
}

NEXAR_D unsigned int ld_acquire_sys_u32(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Signal this round's phase to every rank and wait until all W ranks did.
NEXAR_D bool nvls_sync(const CommDev& c, int phase, unsigned int target, int op) {
  __syncthreads();
  int ok = 1;
  if (threadIdx.x == 0) {
    asm volatile("fence.proxy.alias;" ::: "memory");
    fence_sys();
    asm volatile("multimem.red.release.sys.global.add.u32 [%0], %1;"
                 :: "l"(nvls_flag(c.nvls_mc, blockIdx.x, phase)), "r"(1u) : "memory");
    const unsigned int* mine = nvls_flag(c.nvls_uc, blockIdx.x, phase);
    if ((int)(ld_acquire_sys_u32(mine) - target) < 0) {
      const unsigned long long t0 = globaltimer_ns();
      unsigned int spins = 0;
      while ((int)(ld_acquire_sys_u32(mine) - target) < 0) {
        if ((++spins & 63u) == 0 && globaltimer_ns() - t0 > c.timeout_ns) {
          record_timeout(c, -1, op, target);
          ok = 0;
          break;
        }
      }
    }
    asm volatile("fence.proxy.alias;" ::: "memory");
  }
  return __syncthreads_and(ok) != 0;
}

template <typename T> struct MM;
template <> struct MM<float> {
  static NEXAR_D uint4 ld_reduce(const void* p) {
    uint4 v;
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p) : "memory");
    return v;
  }
  static NEXAR_D void st(void* p, uint4 v) {
    asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};"
                 :: "l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
  }
  static NEXAR_D uint4 scale(uint4 v, float s) {
    v.x = __float_as_uint(__uint_as_float(v.x) * s);
    v.y = __float_as_uint(__uint_as_float(v.y) * s);
    v.z = __float_as_uint(__uint_as_float(v.z) * s);
    v.w = __float_as_uint(__uint_as_float(v.w) * s);
    return v;
  }
};
template <> struct MM<__nv_bfloat16> {
  static NEXAR_D uint4 ld_reduce(const void* p) {
    uint4 v;
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p) : "memory");
    return v;
  }
  static NEXAR_D void st(void* p, uint4 v) {
    asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1,%2,%3,%4};"
                 :: "l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
  }
  static NEXAR_D uint4 scale(uint4 v, float s) {
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = __bfloat1622float2(h[i]);
      h[i] = __floats2bfloat162_rn(f.x * s, f.y * s);
    }
    return v;
  }
};
template <> struct MM<__half> {
  static NEXAR_D uint4 ld_reduce(const void* p) {
    uint4 v;
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.f16x2 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p) : "memory");
    return v;
  }
  static NEXAR_D void st(void* p, uint4 v) {
    asm volatile("multimem.st.relaxed.sys.global.v4.f16x2 [%0], {%1,%2,%3,%4};"
                 :: "l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
  }
  static NEXAR_D uint4 scale(uint4 v, float s) {
    __half2* h = reinterpret_cast<__half2*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = __half22float2(h[i]);
      h[i] = __floats2half2_rn(f.x * s, f.y * s);
    }
    return v;
  }
};

// Plain 16-byte copy of `nv` vectors (block-cooperative, 4 in flight).
NEXAR_D void copy_vec(uint4* __restrict__ dst, const uint4* __restrict__ src, unsigned long long nv) {
  unsigned long long i = threadIdx.x;
  for (; i + 3 * kNvlsThreads < nv; i += 4 * kNvlsThreads) {
    const uint4 a = src[i], b = src[i + kNvlsThreads], d = src[i + 2 * kNvlsThreads], e = src[i + 3 * kNvlsThreads];
    dst[i] = a;
    dst[i + kNvlsThreads] = b;
    dst[i + 2 * kNvlsThreads] = d;
    dst[i + 3 * kNvlsThreads] = e;
  }
  for (; i < nv; i += kNvlsThreads) dst[i] = src[i];
}

// Switch round trips are long: every loop keeps kUnroll multimem
// operations per thread in flight.
constexpr int kUnroll = 8;

// mc[v] = scale * sum over ranks of mc[v] for v in [lo, hi) (vectors).
template <typename T>
NEXAR_D void reduce_bcast_vec(char* mc, unsigned long long lo, unsigned long long hi, float scale) {
  uint4* p = reinterpret_cast<uint4*>(mc);
  unsigned long long i = lo + threadIdx.x;
  for (; i + (kUnroll - 1) * kNvlsThreads < hi; i += kUnroll * kNvlsThreads) {
    uint4 v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) v[u] = MM<T>::ld_reduce(p + i + u * kNvlsThreads);
    if (scale != 1.f) {
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) v[u] = MM<T>::scale(v[u], scale);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) MM<T>::st(p + i + u * kNvlsThreads, v[u]);
  }
  for (; i < hi; i += kNvlsThreads) {
    uint4 a = MM<T>::ld_reduce(p + i);
    if (scale != 1.f) a = MM<T>::scale(a, scale);
    MM<T>::st(p + i, a);
  }
}

// out[v] = scale * sum over ranks of mc[v] (result only local).
template <typename T>
NEXAR_D void reduce_to_local(uint4* __restrict__ out, const char* mc, unsigned long long nv, float scale) {
  const uint4* p = reinterpret_cast<const uint4*>(mc);
  unsigned long long i = threadIdx.x;
  for (; i + (kUnroll - 1) * kNvlsThreads < nv; i += kUnroll * kNvlsThreads) {
    uint4 v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) v[u] = MM<T>::ld_reduce(p + i + u * kNvlsThreads);
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) out[i + u * kNvlsThreads] = scale != 1.f ? MM<T>::scale(v[u], scale) : v[u];
  }
  for (; i < nv; i += kNvlsThreads) {
    uint4 a = MM<T>::ld_reduce(p + i);
    if (scale != 1.f) a = MM<T>::scale(a, scale);
    out[i] = a;
  }
}

// multimem.st of local data to every rank (any 16-byte type).
NEXAR_D void bcast_from_local(char* mc, const uint4* __restrict__ src, unsigned long long nv) {
  uint4* p = reinterpret_cast<uint4*>(mc);
  unsigned long long i = threadIdx.x;
  for (; i + (kUnroll - 1) * kNvlsThreads < nv; i += kUnroll * kNvlsThreads) {
    uint4 v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) v[u] = src[i + u * kNvlsThreads];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) MM<float>::st(p + i + u * kNvlsThreads, v[u]);
  }
  for (; i < nv; i += kNvlsThreads) MM<float>::st(p + i, src[i]);
}

// ---------------------------------------------------------------- all-reduce
// sym_off >= 0: the buffer lives in the NVLS user region at that offset (in
// place, no staging): one round per block over a contiguous block range.
template <typename T>
__global__ void __launch_bounds__(kNvlsThreads) k_allreduce_nvls(CommDev c, const T* in, T* out,
                                                                 unsigned long long nbytes, float scale,
                                                                 long long sym_off) {
  if (!entry_ok(c, kOpAllReduce, 0, sym_off >= 0 ? (unsigned long long)sym_off + nbytes : 0,
                sym_off >= 0 ? c.nvls_bytes : ~0ull))
    return;
  __shared__ unsigned int s_seq;
  if (threadIdx.x == 0) s_seq = c.nvls_seq[blockIdx.x];
  __syncthreads();
  unsigned int seq = s_seq;
  const unsigned int W = (unsigned)c.world;
  const unsigned long long nvec = nbytes / 16;
  if (sym_off >= 0) {
    unsigned long long lo, hi;
    block_range(nvec, gridDim.x, blockIdx.x, 1, &lo, &hi);
    if (nvls_sync(c, 0, W * (seq + 1), kOpAllReduce)) {
      const unsigned long long len = hi - lo;
      const unsigned long long a = lo + len * c.rank / W, b = lo + len * (c.rank + 1) / W;
      reduce_bcast_vec<T>(c.nvls_mc + sym_off, a, b, scale);
      nvls_sync(c, 1, W * (seq + 1), kOpAllReduce);
    }
    seq += 1;
  } else {
    constexpr unsigned long long kChunkVec = kNvlsChunkBytes / 16;
    const unsigned long long chunks = (nvec + kChunkVec - 1) / kChunkVec;
    char* slot_uc = c.nvls_uc + kNvlsSignalBytes + (size_t)blockIdx.x * kNvlsChunkBytes;
    char* slot_mc = c.nvls_mc + kNvlsSignalBytes + (size_t)blockIdx.x * kNvlsChunkBytes;
    for (unsigned long long ch = blockIdx.x; ch < chunks; ch += gridDim.x) {
      const unsigned long long v0 = ch * kChunkVec;
      const unsigned long long len = min(kChunkVec, nvec - v0);
      copy_vec(reinterpret_cast<uint4*>(slot_uc), reinterpret_cast<const uint4*>(in) + v0, len);
      if (!nvls_sync(c, 0, W * (seq + 1), kOpAllReduce)) break;
      const unsigned long long a = len * c.rank / W, b = len * (c.rank + 1) / W;
      reduce_bcast_vec<T>(slot_mc, a, b, scale);
      if (!nvls_sync(c, 1, W * (seq + 1), kOpAllReduce)) break;
      copy_vec(reinterpret_cast<uint4*>(out) + v0, reinterpret_cast<const uint4*>(slot_uc), len);
      seq += 1;
    }
  }
  if (threadIdx.x == 0) c.nvls_seq[blockIdx.x] = seq;
}

// ---------------------------------------------------------------- reduce-scatter
// in: [W][count] local, out: [count] = scale * sum over ranks of in[rank].
// in_sym >= 0: the input lives in the NVLS user region at that offset: no
// staging, one round per block over a contiguous range of the segment.
template <typename T>
__global__ void __launch_bounds__(kNvlsThreads) k_reduce_scatter_nvls(CommDev c, const T* in, T* out,
                                                                      unsigned long long count_bytes,
                                                                      float scale, long long in_sym) {
  if (!entry_ok(c, kOpReduceScatter)) return;
  __shared__ unsigned int s_seq;
  if (threadIdx.x == 0) s_seq = c.nvls_seq[blockIdx.x];
  __syncthreads();
  unsigned int seq = s_seq;
  const unsigned int W = (unsigned)c.world;
  const unsigned long long nvec = count_bytes / 16;
  if (in_sym >= 0) {
    unsigned long long lo, hi;
    block_range(nvec, gridDim.x, blockIdx.x, 1, &lo, &hi);
    if (nvls_sync(c, 0, W * (seq + 1), kOpReduceScatter)) {
      reduce_to_local<T>(reinterpret_cast<uint4*>(out) + lo, c.nvls_mc + in_sym + ((size_t)c.rank * nvec + lo) * 16,
                         hi - lo, scale);
      nvls_sync(c, 1, W * (seq + 1), kOpReduceScatter);
    }
    if (threadIdx.x == 0) c.nvls_seq[blockIdx.x] = seq + 1;
    return;
  }
  const unsigned long long per = (kNvlsChunkBytes / 16) / W;  // vectors of each rank's segment per round
  const unsigned long long chunks = (nvec + per - 1) / per;
  char* slot_uc = c.nvls_uc + kNvlsSignalBytes + (size_t)blockIdx.x * kNvlsChunkBytes;
  char* slot_mc = c.nvls_mc + kNvlsSignalBytes + (size_t)blockIdx.x * kNvlsChunkBytes;
  const uint4* in4 = reinterpret_cast<const uint4*>(in);
  for (unsigned long long ch = blockIdx.x; ch < chunks; ch += gridDim.x) {
    const unsigned long long v0 = ch * per;
    const unsigned long long len = min(per, nvec - v0);
    for (unsigned int q = 0; q < W; ++q)
      copy_vec(reinterpret_cast<uint4*>(slot_uc) + q * len, in4 + q * nvec + v0, len);
    if (!nvls_sync(c, 0, W * (seq + 1), kOpReduceScatter)) break;
    reduce_to_local<T>(reinterpret_cast<uint4*>(out) + v0, slot_mc + (size_t)c.rank * len * 16, len, scale);
    if (!nvls_sync(c, 1, W * (seq + 1), kOpReduceScatter)) break;
    seq += 1;
  }
  if (threadIdx.x == 0) c.nvls_seq[blockIdx.x] = seq;
}

// ---------------------------------------------------------------- all-gather / broadcast
// all-gather (root < 0): out[q][...] = in of rank q. broadcast (root >= 0):
// out = in of root (W segments of one = the whole message on every rank).
// out_sym >= 0: the output lives in the NVLS user region at that offset:
// the multimem stores land in every rank's output directly (entry sync:
// every rank is ready to receive; exit sync: every store has landed).
__global__ void __launch_bounds__(kNvlsThreads) k_gather_bcast_nvls(CommDev c, const void* in, void* out,
                                                                    unsigned long long count_bytes, int root,
                                                                    long long out_sym) {
  if (!entry_ok(c, root < 0 ? kOpAllGather : kOpBroadcast, root < 0 ? 0 : root)) return;
  __shared__ unsigned int s_seq;
  if (threadIdx.x == 0) s_seq = c.nvls_seq[blockIdx.x];
  __syncthreads();
  unsigned int seq = s_seq;
  const unsigned int W = (unsigned)c.world;
  const unsigned long long nvec = count_bytes / 16;
  const bool ag = root < 0;
  if (out_sym >= 0) {
    const int op = ag ? kOpAllGather : kOpBroadcast;
    unsigned long long lo, hi;
    block_range(nvec, gridDim.x, blockIdx.x, 1, &lo, &hi);
    if (nvls_sync(c, 0, W * (seq + 1), op)) {
      if (ag) {
        bcast_from_local(c.nvls_mc + out_sym + ((size_t)c.rank * nvec + lo) * 16,
                         reinterpret_cast<const uint4*>(in) + lo, hi - lo);
      } else if (c.rank == root) {
        bcast_from_local(c.nvls_mc + out_sym + lo * 16, reinterpret_cast<const uint4*>(in) + lo, hi - lo);
      }
      nvls_sync(c, 1, W * (seq + 1), op);
    }
    if (threadIdx.x == 0) c.nvls_seq[blockIdx.x] = seq + 1;
    return;
  }
  const unsigned long long per = ag ? (kNvlsChunkBytes / 16) / W : kNvlsChunkBytes / 16;
  const unsigned long long chunks = (nvec + per - 1) / per;
  char* slot_uc = c.nvls_uc + kNvlsSignalBytes + (size_t)blockIdx.x * kNvlsChunkBytes;
  char* slot_mc = c.nvls_mc + kNvlsSignalBytes + (size_t)blockIdx.x * kNvlsChunkBytes;
  const uint4* in4 = reinterpret_cast<const uint4*>(in);
  uint4* out4 = reinterpret_cast<uint4*>(out);
  const int op = ag ? kOpAllGather : kOpBroadcast;
  for (unsigned long long ch = blockIdx.x; ch < chunks; ch += gridDim.x) {
    const unsigned long long v0 = ch * per;
    const unsigned long long len = min(per, nvec - v0);
    if (ag) bcast_from_local(slot_mc + (size_t)c.rank * len * 16, in4 + v0, len);
    else if (c.rank == root) bcast_from_local(slot_mc, in4 + v0, len);
    if (!nvls_sync(c, 0, W * (seq + 1), op)) break;
    if (ag) {
      for (unsigned int q = 0; q < W; ++q)
        copy_vec(out4 + q * nvec + v0, reinterpret_cast<const uint4*>(slot_uc) + q * len, len);
    } else if (c.rank != root || in != out) {
      copy_vec(out4 + v0, reinterpret_cast<const uint4*>(slot_uc), len);
    }
    if (!nvls_sync(c, 1, W * (seq + 1), op)) break;
    seq += 1;
  }
  if (threadIdx.x == 0) c.nvls_seq[blockIdx.x] = seq;
}

// Up to kMaxBlocks CTAs (two per SM): while one CTA of an SM waits on a
// signal, the other copies, so HBM staging overlaps the NVLink phase.
// `max_blocks` (the communicator's limit, e.g. a small grid for collectives
// that overlap compute kernels) caps it further.
int nvls_grid(unsigned long long units, unsigned int max_blocks) {
  unsigned long long g = units < 1 ? 1 : units;
  if (g > (unsigned long long)kMaxBlocks) g = kMaxBlocks;
  if (max_blocks > 0 && g > max_blocks) g = max_blocks;
  return (int)g;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

bool nvls_can_reduce(const CommDev& c, int dt, int op, const void* in, const void* out, unsigned long long bytes) {
  if (!c.nvls_mc || c.world < 2) return false;
  if (op != kSum) return false;  // averaging is Sum with scale = 1/world
  if (dt != kF32 && dt != kBF16 && dt != kF16) return false;
  return bytes % 16 == 0 && aligned16(in) && aligned16(out);
}

bool nvls_can_move(const CommDev& c, const void* in, const void* out, unsigned long long bytes) {
  return c.nvls_mc && c.world >= 2 && bytes % 16 == 0 && aligned16(in) && aligned16(out);
}

cudaError_t launch_all_reduce_nvls(const CommDev& c, const void* in, void* out, int dt, unsigned long long bytes,
                                   float scale, long long sym_off, unsigned int max_blocks, cudaStream_t s) {
  const unsigned long long nvec = bytes / 16;
  int grid;
  if (sym_off >= 0) grid = nvls_grid((nvec + 4095) / 4096, max_blocks);  // >= 64 KB per CTA
  else grid = nvls_grid((bytes + kNvlsChunkBytes - 1) / kNvlsChunkBytes, max_blocks);
  switch (dt) {
    case kF32:
      k_allreduce_nvls<float><<<grid, kNvlsThreads, 0, s>>>(c, (const float*)in, (float*)out, bytes, scale, sym_off);
      break;
    case kBF16:
      k_allreduce_nvls<__nv_bfloat16><<<grid, kNvlsThreads, 0, s>>>(c, (const __nv_bfloat16*)in,
                                                                   (__nv_bfloat16*)out, bytes, scale, sym_off);
      break;
    case kF16:
      k_allreduce_nvls<__half><<<grid, kNvlsThreads, 0, s>>>(c, (const __half*)in, (__half*)out, bytes, scale,
                                                            sym_off);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_reduce_scatter_nvls(const CommDev& c, const void* in, void* out, int dt,
                                       unsigned long long count_bytes, float scale, long long in_sym,
                                       unsigned int max_blocks, cudaStream_t s) {
  const unsigned long long per = kNvlsChunkBytes / c.world;
  const int grid = in_sym >= 0 ? nvls_grid((count_bytes + 65535) / 65536, max_blocks)
                               : nvls_grid((count_bytes + per - 1) / per, max_blocks);
  switch (dt) {
    case kF32:
      k_reduce_scatter_nvls<float><<<grid, kNvlsThreads, 0, s>>>(c, (const float*)in, (float*)out, count_bytes, scale,
                                                                 in_sym);
      break;
    case kBF16:
      k_reduce_scatter_nvls<__nv_bfloat16><<<grid, kNvlsThreads, 0, s>>>(c, (const __nv_bfloat16*)in,
                                                                        (__nv_bfloat16*)out, count_bytes, scale, in_sym);
      break;
    case kF16:
      k_reduce_scatter_nvls<__half><<<grid, kNvlsThreads, 0, s>>>(c, (const __half*)in, (__half*)out, count_bytes,
                                                                 scale, in_sym);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_all_gather_nvls(const CommDev& c, const void* in, void* out, unsigned long long count_bytes,
                                   long long out_sym, unsigned int max_blocks, cudaStream_t s) {
  const unsigned long long per = kNvlsChunkBytes / c.world;
  const int grid = out_sym >= 0 ? nvls_grid((count_bytes + 65535) / 65536, max_blocks)
                                : nvls_grid((count_bytes + per - 1) / per, max_blocks);
  k_gather_bcast_nvls<<<grid, kNvlsThreads, 0, s>>>(c, in, out, count_bytes, -1, out_sym);
  return cudaGetLastError();
}

cudaError_t launch_broadcast_nvls(const CommDev& c, const void* in, void* out, unsigned long long bytes, int root,
                                  long long out_sym, unsigned int max_blocks, cudaStream_t s) {
  const int grid = out_sym >= 0 ? nvls_grid((bytes + 65535) / 65536, max_blocks)
                                : nvls_grid((bytes + kNvlsChunkBytes - 1) / kNvlsChunkBytes, max_blocks);
  k_gather_bcast_nvls<<<grid, kNvlsThreads, 0, s>>>(c, in, out, bytes, root, out_sym);
  return cudaGetLastError();
}

}  // namespace nexar
