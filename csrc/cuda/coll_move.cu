// Data-movement collectives: all-gather, all-to-all, broadcast, gather, scatter, barrier.
#include "coll_impl.cuh"

namespace nexar {

// ============================================================ all-gather
template <typename T>
__global__ void __launch_bounds__(kThreads) k_all_gather(CommDev c, const T* in, T* out,
                                                         unsigned long long count,
                                                         unsigned long long out_ld, bool vec) {
  const unsigned long long call = call_index(c);
  if (!entry_ok(c, kOpAllGather, 0, count * sizeof(T), c.slot_bytes)) {
    finish_call(c, call);
    return;
  }
  constexpr int V = PackOf<T>::V;
  const int N = c.world;
  unsigned long long lo, hi;
  block_range(count, gridDim.x, blockIdx.x, V, &lo, &hi);
  const int slot = (int)(call & 1ull);
  copy_range<T>(stage_ptr<T>(c, c.rank, slot), in, lo, hi, vec, false);
  if (block_barrier(c, epoch_of(call, 0), kOpAllGather)) {
    for (int q = 0; q < N; ++q) {
      const int p = (c.rank + q) % N;
      copy_range<T>(out + p * out_ld, stage_ptr<T>(c, p, slot), lo, hi, vec, p != c.rank);
    }
  }
  finish_call(c, call);
}

// ============================================================ all-to-all
// in: [N][count] (block p goes to rank p), out: [N][count] (block p came from p)
template <typename T>
__global__ void __launch_bounds__(kThreads) k_all_to_all(CommDev c, const T* in, T* out,
                                                         unsigned long long count,
                                                         unsigned long long in_ld,
                                                         unsigned long long out_ld, bool vec) {
  const unsigned long long call = call_index(c);
  if (!entry_ok(c, kOpAllToAll, 0, (unsigned long long)c.world * count * sizeof(T), c.slot_bytes)) {
    finish_call(c, call);
    return;
  }
  constexpr int V = PackOf<T>::V;
  const int N = c.world;
  unsigned long long lo, hi;
  block_range(count, gridDim.x, blockIdx.x, V, &lo, &hi);
  const int slot = (int)(call & 1ull);
  T* a = stage_ptr<T>(c, c.rank, slot);
  for (int p = 0; p < N; ++p) copy_range<T>(a + p * count, in + p * in_ld, lo, hi, vec, false);
  if (block_barrier(c, epoch_of(call, 0), kOpAllToAll)) {
    for (int q = 0; q < N; ++q) {
      const int p = (c.rank + q) % N;
      copy_range<T>(out + p * out_ld, stage_ptr<T>(c, p, slot) + (unsigned long long)c.rank * count,
                    lo, hi, vec, p != c.rank);
    }
  }
  finish_call(c, call);
}

// ============================================================ broadcast
template <typename T>
__global__ void __launch_bounds__(kThreads) k_broadcast(CommDev c, const T* in, T* out,
                                                        unsigned long long n, int root, bool vec) {
  const unsigned long long call = call_index(c);
  if (!entry_ok(c, kOpBroadcast, root, n * sizeof(T), c.slot_bytes)) {
    finish_call(c, call);
    return;
  }
  constexpr int V = PackOf<T>::V;
  unsigned long long lo, hi;
  block_range(n, gridDim.x, blockIdx.x, V, &lo, &hi);
  const int slot = (int)(call & 1ull);
  if (c.rank == root) {
    copy_range<T>(stage_ptr<T>(c, c.rank, slot), in, lo, hi, vec, false);
    if (out != in) copy_range<T>(out, in, lo, hi, vec, false);
  }
  if (block_barrier(c, epoch_of(call, 0), kOpBroadcast)) {
    if (c.rank != root) copy_range<T>(out, stage_ptr<T>(c, root, slot), lo, hi, vec, true);
  }
  finish_call(c, call);
}

// ============================================================ gather / scatter
template <typename T>
__global__ void __launch_bounds__(kThreads) k_gather(CommDev c, const T* in, T* out,
                                                     unsigned long long count,
                                                     unsigned long long out_ld, int root, bool vec) {
  const unsigned long long call = call_index(c);
  if (!entry_ok(c, kOpGather, root, count * sizeof(T), c.slot_bytes)) {
    finish_call(c, call);
    return;
  }
  constexpr int V = PackOf<T>::V;
  unsigned long long lo, hi;
  block_range(count, gridDim.x, blockIdx.x, V, &lo, &hi);
  const int slot = (int)(call & 1ull);
  copy_range<T>(stage_ptr<T>(c, c.rank, slot), in, lo, hi, vec, false);
  if (block_barrier(c, epoch_of(call, 0), kOpGather) && c.rank == root) {
    for (int q = 0; q < c.world; ++q) {
      const int p = (c.rank + q) % c.world;
      copy_range<T>(out + p * out_ld, stage_ptr<T>(c, p, slot), lo, hi, vec, p != c.rank);
    }
  }
  finish_call(c, call);
}

template <typename T>
__global__ void __launch_bounds__(kThreads) k_scatter(CommDev c, const T* in, T* out,
                                                      unsigned long long count,
                                                      unsigned long long in_ld, int root, bool vec) {
  const unsigned long long call = call_index(c);
  if (!entry_ok(c, kOpScatter, root, (unsigned long long)c.world * count * sizeof(T), c.slot_bytes)) {
    finish_call(c, call);
    return;
  }
  constexpr int V = PackOf<T>::V;
  unsigned long long lo, hi;
  block_range(count, gridDim.x, blockIdx.x, V, &lo, &hi);
  const int slot = (int)(call & 1ull);
  if (c.rank == root) {
    T* a = stage_ptr<T>(c, c.rank, slot);
    for (int p = 0; p < c.world; ++p) copy_range<T>(a + p * count, in + p * in_ld, lo, hi, vec, false);
  }
  if (block_barrier(c, epoch_of(call, 0), kOpScatter)) {
    copy_range<T>(out, stage_ptr<T>(c, root, slot) + (unsigned long long)c.rank * count, lo, hi, vec,
                  c.rank != root);
  }
  finish_call(c, call);
}

// ============================================================ barrier
__global__ void k_barrier(CommDev c) {
  const unsigned long long call = call_index(c);
  if (!entry_ok(c, kOpBarrier, 0, 0, c.slot_bytes)) {
    finish_call(c, call);
    return;
  }
  block_barrier(c, epoch_of(call, 0), kOpBarrier);
  finish_call(c, call);
}

cudaError_t launch_all_gather(const CommDev& c, const void* in, void* out, int dt,
                              unsigned long long count, unsigned long long out_ld,
                              unsigned int max_blocks, cudaStream_t s) {
  if (count == 0) return cudaSuccess;
  const int es = dtype_size(dt);
  const bool vec = aligned16(in) && aligned16(out) && (count * es) % 16 == 0 && (out_ld * es) % 16 == 0;
  const unsigned int g = pick_blocks(count * es, max_blocks);
  NEXAR_DISPATCH_ALL(dt, k_all_gather<T><<<g, kThreads, 0, s>>>(c, (const T*)in, (T*)out, count, out_ld, vec));
  return cudaGetLastError();
}

cudaError_t launch_all_to_all(const CommDev& c, const void* in, void* out, int dt,
                              unsigned long long count, unsigned long long in_ld,
                              unsigned long long out_ld, unsigned int max_blocks, cudaStream_t s) {
  if (count == 0) return cudaSuccess;
  const int es = dtype_size(dt);
  const bool vec = aligned16(in) && aligned16(out) && (count * es) % 16 == 0 &&
                   (in_ld * es) % 16 == 0 && (out_ld * es) % 16 == 0;
  const unsigned int g = pick_blocks(count * es, max_blocks);
  NEXAR_DISPATCH_ALL(dt, k_all_to_all<T><<<g, kThreads, 0, s>>>(c, (const T*)in, (T*)out, count, in_ld, out_ld, vec));
  return cudaGetLastError();
}

// Large broadcast as scatter + all-gather: every rank pulls its own 1/N chunk
// from the root (the root's helper, rank root+1, also pulls the root's chunk)
// and then pulls the other chunks from the ranks that hold them. The root
// sends each byte once instead of N-1 times (flat pull).
template <typename T>
__global__ void __launch_bounds__(kThreads) k_broadcast_sag(CommDev c, const T* in, T* out,
                                                            unsigned long long n, int root, bool vec) {
  const unsigned long long call = call_index(c);
  if (!entry_ok(c, kOpBroadcast, root, n * sizeof(T), c.slot_bytes)) {
    finish_call(c, call);
    return;
  }
  constexpr int V = PackOf<T>::V;
  const int N = c.world;
  unsigned long long chunk = (n + N - 1) / N;
  chunk = (chunk + V - 1) / V * V;
  unsigned long long slo, shi;
  block_range(chunk, gridDim.x, blockIdx.x, V, &slo, &shi);
  const int slot = (int)(call & 1ull);
  T* mine = stage_ptr<T>(c, c.rank, slot);
  const int helper = (root + 1) % N;
  auto rng = [&](int q, unsigned long long* lo, unsigned long long* hi) {
    *lo = q * chunk + slo;
    *hi = q * chunk + shi;
    if (*hi > n) *hi = n;
    return *lo < *hi;
  };
  unsigned long long lo, hi;
  if (c.rank == root) {
    for (int q = 0; q < N; ++q)
      if (rng(q, &lo, &hi)) {
        copy_range<T>(mine, in, lo, hi, vec, false);
        if (out != in) copy_range<T>(out, in, lo, hi, vec, false);
      }
  }
  bool ok = block_barrier(c, epoch_of(call, 0), kOpBroadcast);
  if (ok && c.rank != root) {
    const T* rs = stage_ptr<T>(c, root, slot);
    for (int q = 0; q < N; ++q) {
      if (!(q == c.rank || (c.rank == helper && q == root))) continue;
      if (rng(q, &lo, &hi)) {
        copy_range<T>(mine, rs, lo, hi, vec, true);
        __syncthreads();
        copy_range<T>(out, mine, lo, hi, vec, false);
      }
    }
  }
  ok = ok && block_barrier(c, epoch_of(call, 1), kOpBroadcast);
  if (ok && c.rank != root) {
    for (int d = 1; d < N; ++d) {
      const int q = (c.rank + d) % N;
      if (q == c.rank || (c.rank == helper && q == root)) continue;
      const int owner = q == root ? helper : q;
      if (rng(q, &lo, &hi)) copy_range<T>(out, stage_ptr<T>(c, owner, slot), lo, hi, vec, true);
    }
  }
  finish_call(c, call);
}

cudaError_t launch_broadcast(const CommDev& c, const void* in, void* out, int dt,
                             unsigned long long n, int root, unsigned int max_blocks,
                             cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  const int es = dtype_size(dt);
  const bool vec = aligned16(in) && aligned16(out) && (n * es) % 16 == 0;
  if (c.world >= 3 && n * es >= (256ull << 10)) {
    const unsigned int g = pick_blocks(n * es / c.world, max_blocks);
    NEXAR_DISPATCH_ALL(dt, k_broadcast_sag<T><<<g, kThreads, 0, s>>>(c, (const T*)in, (T*)out, n, root, vec));
    return cudaGetLastError();
  }
  const unsigned int g = pick_blocks(n * es, max_blocks);
  NEXAR_DISPATCH_ALL(dt, k_broadcast<T><<<g, kThreads, 0, s>>>(c, (const T*)in, (T*)out, n, root, vec));
  return cudaGetLastError();
}

cudaError_t launch_gather(const CommDev& c, const void* in, void* out, int dt,
                          unsigned long long count, unsigned long long out_ld, int root,
                          unsigned int max_blocks, cudaStream_t s) {
  if (count == 0) return cudaSuccess;
  const int es = dtype_size(dt);
  const bool vec = aligned16(in) && aligned16(out) && (count * es) % 16 == 0 && (out_ld * es) % 16 == 0;
  const unsigned int g = pick_blocks(count * es, max_blocks);
  NEXAR_DISPATCH_ALL(dt, k_gather<T><<<g, kThreads, 0, s>>>(c, (const T*)in, (T*)out, count, out_ld, root, vec));
  return cudaGetLastError();
}

cudaError_t launch_scatter(const CommDev& c, const void* in, void* out, int dt,
                           unsigned long long count, unsigned long long in_ld, int root,
                           unsigned int max_blocks, cudaStream_t s) {
  if (count == 0) return cudaSuccess;
  const int es = dtype_size(dt);
  const bool vec = aligned16(in) && aligned16(out) && (count * es) % 16 == 0 && (in_ld * es) % 16 == 0;
  const unsigned int g = pick_blocks(count * es, max_blocks);
  NEXAR_DISPATCH_ALL(dt, k_scatter<T><<<g, kThreads, 0, s>>>(c, (const T*)in, (T*)out, count, in_ld, root, vec));
  return cudaGetLastError();
}

cudaError_t launch_barrier(const CommDev& c, cudaStream_t s) {
  k_barrier<<<1, 32, 0, s>>>(c);
  return cudaGetLastError();
}

}  // namespace nexar
