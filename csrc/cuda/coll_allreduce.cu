// All-reduce kernels: one-shot and two-shot over NVLink peer memory.
#include <type_traits>

#include "coll_impl.cuh"

namespace nexar {

// ============================================================ all-reduce
// One-shot: stage, barrier, every rank reduces the whole message reading all
// peers. Lowest latency; NVLink traffic (N-1)*S in per rank. When `sym_off`
// >= 0 the input already lives in the symmetric heap at that offset and no
// staging copy is made; a trailing barrier then protects it from reuse.
template <typename T, typename TO, int OP>
__global__ void __launch_bounds__(kThreads) k_ar_oneshot(CommDev c, const T* in, TO* out,
                                                         unsigned long long n, float scale,
                                                         bool vec, long long sym_off) {
  const unsigned long long call = call_index(c);
  if (!entry_ok(c, kOpAllReduce, 0, n * sizeof(T), (sym_off >= 0 ? c.heap_bytes - (unsigned long long)sym_off : c.slot_bytes))) {
    finish_call(c, call);
    return;
  }
  constexpr int V = PackOf<T>::V;
  unsigned long long lo, hi;
  block_range(n, gridDim.x, blockIdx.x, V, &lo, &hi);
  const bool sym = sym_off >= 0;
  const int slot = (int)(call & 1ull);
  const T* srcs[kMaxRanks];
#pragma unroll
  for (int p = 0; p < kMaxRanks; ++p)
    srcs[p] = p < c.world ? (sym ? heap_ptr<T>(c, p, (unsigned long long)sym_off) : stage_ptr<T>(c, p, slot)) : nullptr;
  if (!sym) copy_range<T>(stage_ptr<T>(c, c.rank, slot), in, lo, hi, vec, false);
  if (block_barrier(c, epoch_of(call, 0), kOpAllReduce)) {
    reduce_range<T, TO, OP>(out, srcs, c.world, lo, hi, scale, vec);
    if (sym) block_barrier(c, epoch_of(call, 1), kOpAllReduce);
  }
  finish_call(c, call);
}

// Two-shot: reduce-scatter by pulling chunk `rank` from all peers, then
// all-gather by pushing the reduced chunk into every peer. NVLink traffic
// (N-1)/N*S in and (N-1)/N*S out per rank. With `sym_off` >= 0 (input is a
// symmetric tensor and the operation is in place) the pushes go straight into
// the peers' tensors and no staging copies are made at all.
template <typename T, typename TO, int OP>
__global__ void __launch_bounds__(kThreads) k_ar_twoshot(CommDev c, const T* in, TO* out,
                                                         unsigned long long n, float scale,
                                                         bool vec, long long sym_off) {
  const unsigned long long call = call_index(c);
  if (!entry_ok(c, kOpAllReduce, 0, n * (sizeof(T) > sizeof(TO) ? sizeof(T) : sizeof(TO)), (sym_off >= 0 ? c.heap_bytes - (unsigned long long)sym_off : c.slot_bytes))) {
    finish_call(c, call);
    return;
  }
  constexpr int V = PackOf<T>::V;
  const int N = c.world;
  unsigned long long chunk = (n + N - 1) / N;
  chunk = (chunk + V - 1) / V * V;
  unsigned long long slo, shi;
  block_range(chunk, gridDim.x, blockIdx.x, V, &slo, &shi);
  const bool sym = sym_off >= 0;
  // stage A: staged input (T); stage B: gathered result (TO).
  if (!sym) {
    T* a = stage_ptr<T>(c, c.rank, 0);
    for (int p = 0; p < N; ++p) {
      unsigned long long lo = p * chunk + slo, hi = p * chunk + shi;
      if (hi > n) hi = n;
      if (lo < hi) copy_range<T>(a, in, lo, hi, vec, false);
    }
  }
  bool ok = block_barrier(c, epoch_of(call, 0), kOpAllReduce);
  if (ok) {
    const T* srcs[kMaxRanks];
    T* dsts[kMaxRanks];
#pragma unroll
    for (int p = 0; p < kMaxRanks; ++p) {
      srcs[p] = p < N ? (sym ? heap_ptr<T>(c, p, (unsigned long long)sym_off) : stage_ptr<T>(c, p, 0)) : nullptr;
      dsts[p] = (p < N && sym) ? heap_ptr<T>(c, p, (unsigned long long)sym_off) : nullptr;
    }
    unsigned long long lo = c.rank * chunk + slo, hi = c.rank * chunk + shi;
    if (hi > n) hi = n;
    if (lo < hi) {
      if (sym) {
        reduce_push_range<T, OP>(dsts, N, srcs, N, lo, hi, scale, vec);
      } else if constexpr (std::is_same<T, TO>::value) {
        // One pass: pull the chunk from every peer, reduce, and store the
        // result into our output and every peer's stage B in the same loop,
        // so NVLink inbound (loads) and outbound (stores) overlap.
        T* outs[kMaxRanks];
#pragma unroll
        for (int p = 0; p < kMaxRanks; ++p)
          outs[p] = p >= N ? nullptr
                           : (p == c.rank ? reinterpret_cast<T*>(out)
                                          : reinterpret_cast<T*>(c.peer_base[p] + c.stage_off + c.slot_bytes));
        reduce_push_range<T, OP>(outs, N, srcs, N, lo, hi, scale, vec);
      } else {
        // Fused cast: reduce once into our output, then push the TO result
        // into every peer's stage B.
        reduce_range<T, TO, OP>(out, srcs, N, lo, hi, scale, vec);
        __syncthreads();
        for (int q = 1; q < N; ++q) {
          const int p = (c.rank + q) % N;
          TO* b = reinterpret_cast<TO*>(c.peer_base[p] + c.stage_off + c.slot_bytes);
          copy_range<TO>(b, out, lo, hi, vec, false);
        }
      }
    }
    ok = block_barrier(c, epoch_of(call, 1), kOpAllReduce);
    if (ok && !sym) {
      const TO* b = reinterpret_cast<const TO*>(c.peer_base[c.rank] + c.stage_off + c.slot_bytes);
      for (int p = 0; p < N; ++p) {
        if (p == c.rank) continue;
        unsigned long long lo2 = p * chunk + slo, hi2 = p * chunk + shi;
        if (hi2 > n) hi2 = n;
        if (lo2 < hi2) copy_range<TO>(out, b, lo2, hi2, vec, true);
      }
    }
  }
  finish_call(c, call);
}

cudaError_t launch_all_reduce(const CommDev& c, const void* in, void* out, int dt_in, int dt_out,
                              int op, unsigned long long n, float scale, int algo,
                              long long sym_off, unsigned int max_blocks, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  const int es = dtype_size(dt_in);
  const bool vec = aligned16(in) && aligned16(out) && (n * es) % 16 == 0;
  const unsigned int g = pick_blocks(n * es / (algo == kAlgoTwoShot ? c.world : 1), max_blocks);
  NEXAR_DISPATCH_OUT_OP(dt_in, dt_out, op, {
    if (algo == kAlgoTwoShot) {
      k_ar_twoshot<T, TO, OP><<<g, kThreads, 0, s>>>(c, (const T*)in, (TO*)out, n, scale, vec, sym_off);
    } else {
      k_ar_oneshot<T, TO, OP><<<g, kThreads, 0, s>>>(c, (const T*)in, (TO*)out, n, scale, vec, sym_off);
    }
  });
  return cudaGetLastError();
}

}  // namespace nexar
