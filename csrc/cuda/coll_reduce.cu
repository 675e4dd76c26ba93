// Reduce-scatter and reduce-to-root kernels over NVLink peer memory.
#include "coll_impl.cuh"

namespace nexar {

// ============================================================ reduce-scatter
// in: N*count elements, out: count. Rank r receives the reduction of chunk r
// (NCCL/MPI semantics; the reference's host ring leaves chunk (r+1) mod N on
// rank r, nexar/src/collective/reduce_scatter.rs:73-77).
template <typename T, typename TO, int OP>
__global__ void __launch_bounds__(kThreads) k_reduce_scatter(CommDev c, const T* in, TO* out,
                                                             unsigned long long count,
                                                             unsigned long long in_ld, float scale,
                                                             bool vec) {
  const unsigned long long call = call_index(c);
  if (!entry_ok(c, kOpReduceScatter, 0, (unsigned long long)c.world * count * sizeof(T), c.slot_bytes)) {
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
  if (block_barrier(c, epoch_of(call, 0), kOpReduceScatter)) {
    const T* srcs[kMaxRanks];
#pragma unroll
    for (int p = 0; p < kMaxRanks; ++p)
      srcs[p] = p < N ? stage_ptr<T>(c, p, slot) + (unsigned long long)c.rank * count : nullptr;
    reduce_range<T, TO, OP>(out, srcs, N, lo, hi, scale, vec);
  }
  finish_call(c, call);
}

// ============================================================ reduce (to root)
// Each rank reduces chunk `rank` from all peers and pushes it to the root's
// stage B; the root then copies B to its output. Root NVLink ingress is S.
template <typename T, typename TO, int OP>
__global__ void __launch_bounds__(kThreads) k_reduce(CommDev c, const T* in, TO* out,
                                                     unsigned long long n, int root, float scale,
                                                     bool vec) {
  const unsigned long long call = call_index(c);
  if (!entry_ok(c, kOpReduce, root, n * (sizeof(T) > sizeof(TO) ? sizeof(T) : sizeof(TO)), c.slot_bytes)) {
    finish_call(c, call);
    return;
  }
  constexpr int V = PackOf<T>::V;
  const int N = c.world;
  unsigned long long chunk = (n + N - 1) / N;
  chunk = (chunk + V - 1) / V * V;
  unsigned long long slo, shi;
  block_range(chunk, gridDim.x, blockIdx.x, V, &slo, &shi);
  T* a = stage_ptr<T>(c, c.rank, 0);
  for (int p = 0; p < N; ++p) {
    unsigned long long lo = p * chunk + slo, hi = p * chunk + shi;
    if (hi > n) hi = n;
    if (lo < hi) copy_range<T>(a, in, lo, hi, vec, false);
  }
  bool ok = block_barrier(c, epoch_of(call, 0), kOpReduce);
  if (ok) {
    const T* srcs[kMaxRanks];
#pragma unroll
    for (int p = 0; p < kMaxRanks; ++p) srcs[p] = p < N ? stage_ptr<T>(c, p, 0) : nullptr;
    unsigned long long lo = c.rank * chunk + slo, hi = c.rank * chunk + shi;
    if (hi > n) hi = n;
    TO* b = reinterpret_cast<TO*>(c.peer_base[root] + c.stage_off + c.slot_bytes);
    if (lo < hi) reduce_range<T, TO, OP>(c.rank == root ? out : b, srcs, N, lo, hi, scale, vec);
    ok = block_barrier(c, epoch_of(call, 1), kOpReduce);
    if (ok && c.rank == root) {
      const TO* bl = reinterpret_cast<const TO*>(c.peer_base[c.rank] + c.stage_off + c.slot_bytes);
      for (int p = 0; p < N; ++p) {
        if (p == root) continue;
        unsigned long long lo2 = p * chunk + slo, hi2 = p * chunk + shi;
        if (hi2 > n) hi2 = n;
        if (lo2 < hi2) copy_range<TO>(out, bl, lo2, hi2, vec, true);
      }
    }
  }
  finish_call(c, call);
}

cudaError_t launch_reduce_scatter(const CommDev& c, const void* in, void* out, int dt_in,
                                  int dt_out, int op, unsigned long long count,
                                  unsigned long long in_ld, float scale, unsigned int max_blocks,
                                  cudaStream_t s) {
  if (count == 0) return cudaSuccess;
  const int es = dtype_size(dt_in);
  const bool vec = aligned16(in) && aligned16(out) && (count * es) % 16 == 0 && (in_ld * es) % 16 == 0;
  const unsigned int g = pick_blocks(count * es, max_blocks);
  NEXAR_DISPATCH_OUT_OP(dt_in, dt_out, op, {
    k_reduce_scatter<T, TO, OP><<<g, kThreads, 0, s>>>(c, (const T*)in, (TO*)out, count, in_ld, scale, vec);
  });
  return cudaGetLastError();
}

cudaError_t launch_reduce(const CommDev& c, const void* in, void* out, int dt_in, int dt_out,
                          int op, unsigned long long n, int root, float scale,
                          unsigned int max_blocks, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  const int es = dtype_size(dt_in);
  const bool vec = aligned16(in) && aligned16(out) && (n * es) % 16 == 0;
  const unsigned int g = pick_blocks(n * es / c.world, max_blocks);
  NEXAR_DISPATCH_OUT_OP(dt_in, dt_out, op, {
    k_reduce<T, TO, OP><<<g, kThreads, 0, s>>>(c, (const T*)in, (TO*)out, n, root, scale, vec);
  });
  return cudaGetLastError();
}

}  // namespace nexar
