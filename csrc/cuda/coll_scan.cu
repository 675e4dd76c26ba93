// Scan (inclusive/exclusive) across ranks and the local elementwise reduce.
#include "coll_impl.cuh"

namespace nexar {

// ============================================================ scan
// Inclusive: out_r = in_0 op ... op in_r. Exclusive: out_r = in_0 op ... op
// in_{r-1}, rank 0 receives the op's identity (nexar/src/collective/scan.rs).
template <typename T, int OP>
__global__ void __launch_bounds__(kThreads) k_scan(CommDev c, const T* in, T* out,
                                                   unsigned long long n, bool exclusive, bool vec) {
  const unsigned long long call = call_index(c);
  if (!entry_ok(c, kOpScan, 0, n * sizeof(T), c.slot_bytes)) {
    finish_call(c, call);
    return;
  }
  constexpr int V = PackOf<T>::V;
  unsigned long long lo, hi;
  block_range(n, gridDim.x, blockIdx.x, V, &lo, &hi);
  const int slot = (int)(call & 1ull);
  copy_range<T>(stage_ptr<T>(c, c.rank, slot), in, lo, hi, vec, false);
  if (block_barrier(c, epoch_of(call, 0), kOpScan)) {
    const int nsrc = exclusive ? c.rank : c.rank + 1;
    if (nsrc == 0) {
      using A = typename AccOf<T>::type;
      const T id = from_acc<T, A>(identity_of<A, OP>());
      for (unsigned long long j = lo + threadIdx.x; j < hi; j += blockDim.x) out[j] = id;
    } else {
      const T* srcs[kMaxRanks];
#pragma unroll
      for (int p = 0; p < kMaxRanks; ++p) srcs[p] = p < nsrc ? stage_ptr<T>(c, p, slot) : nullptr;
      reduce_range<T, T, OP>(out, srcs, nsrc, lo, hi, 1.0f, vec);
    }
  }
  finish_call(c, call);
}

// ============================================================ local reduce
// dst = op(dst, src) elementwise: the device `reduce_inplace` of the
// DeviceAdapter (nexar/src/device/adapter.rs reduce_inplace; the reference's
// CUDA adapter stages through the host, nexar-rdma/src/cuda_adapter.rs:101-138).
template <typename T, int OP>
__global__ void __launch_bounds__(kThreads) k_reduce_inplace(T* dst, const T* src,
                                                             unsigned long long n, bool vec) {
  unsigned long long lo, hi;
  block_range(n, gridDim.x, blockIdx.x, PackOf<T>::V, &lo, &hi);
  const T* srcs[2] = {dst, src};
  reduce_range<T, T, OP>(dst, srcs, 2, lo, hi, 1.0f, vec);
}

cudaError_t launch_scan(const CommDev& c, const void* in, void* out, int dt, int op,
                        unsigned long long n, bool exclusive, unsigned int max_blocks,
                        cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  if (dt == kF8E4M3 || dt == kF8E5M2) return cudaErrorInvalidValue;
  const int es = dtype_size(dt);
  const bool vec = aligned16(in) && aligned16(out) && (n * es) % 16 == 0;
  const unsigned int g = pick_blocks(n * es, max_blocks);
  NEXAR_DISPATCH_ALL(dt, NEXAR_DISPATCH_OP(op, {
    k_scan<T, OP><<<g, kThreads, 0, s>>>(c, (const T*)in, (T*)out, n, exclusive, vec);
  }));
  return cudaGetLastError();
}

cudaError_t launch_reduce_inplace(void* dst, const void* src, int dt, int op,
                                  unsigned long long n, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  const int es = dtype_size(dt);
  const bool vec = aligned16(dst) && aligned16(src) && (n * es) % 16 == 0;
  const unsigned int g = pick_blocks(n * es, 148 * 2);
  NEXAR_DISPATCH_ALL(dt, NEXAR_DISPATCH_OP(op, {
    k_reduce_inplace<T, OP><<<g, kThreads, 0, s>>>((T*)dst, (const T*)src, n, vec);
  }));
  return cudaGetLastError();
}

}  // namespace nexar
