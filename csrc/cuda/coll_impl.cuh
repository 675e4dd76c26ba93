// Peer-memory collectives for one NVSwitch box (sm_100a): shared device code.
//
// Replaces the library calls of the reference's device path
// (nexar-nccl/src/group.rs:72-225: ncclAllReduce / ncclReduceScatter /
// ncclAllGather / ncclBroadcast / ncclReduce) and adds the collectives the
// reference only has on host memory (all_to_all, gather, scatter, scan:
// nexar/src/collective/{alltoall,gather,scatter,scan}.rs) as kernels that load
// and store peer HBM directly over NVLink 5.
//
// Structure shared by all kernels: each block owns a contiguous element range
// (identical on every rank), stages its part of the input into this rank's
// symmetric staging slot, meets the same-index block of every peer at a
// bounded barrier, and then reads the peers' slots. Floating reductions
// accumulate in fp32 (f64 for f64) in rank order 0..N-1, so every rank gets
// bit-identical results. The optional `scale` and output-dtype cast are fused
// into the final store.
#pragma once
#include "coll.cuh"
#include "coll_api.h"

namespace nexar {

// ---------------------------------------------------------------- identities
template <typename A, int OP> NEXAR_D A identity_of();
#define NEXAR_IDENT(A, S, P, MN, MX)                                \
  template <> NEXAR_D A identity_of<A, kSum>() { return S; }        \
  template <> NEXAR_D A identity_of<A, kProd>() { return P; }       \
  template <> NEXAR_D A identity_of<A, kMin>() { return MN; }       \
  template <> NEXAR_D A identity_of<A, kMax>() { return MX; }
// Floats use +-FLT_MAX as Min/Max identities like the reference
// (nexar/src/reduce_types.rs impl_identity!(float)). For 16-bit outputs the
// rounding of FLT_MAX gives +-inf, which also matches the reference.
NEXAR_IDENT(float, 0.f, 1.f, 3.402823466e38f, -3.402823466e38f)
NEXAR_IDENT(double, 0.0, 1.0, 1.7976931348623157e308, -1.7976931348623157e308)
NEXAR_IDENT(int8_t, 0, 1, 127, -128)
NEXAR_IDENT(uint8_t, 0, 1, 255, 0)
NEXAR_IDENT(int32_t, 0, 1, 2147483647, (-2147483647 - 1))
NEXAR_IDENT(uint32_t, 0u, 1u, 0xffffffffu, 0u)
NEXAR_IDENT(int64_t, 0, 1, 9223372036854775807ll, (-9223372036854775807ll - 1))
NEXAR_IDENT(uint64_t, 0ull, 1ull, 0xffffffffffffffffull, 0ull)
#undef NEXAR_IDENT

// ---------------------------------------------------------------- pack I/O
template <typename T> struct PackOf { static constexpr int V = 16 / sizeof(T); };

// Store V accumulators as TO elements at dst (dst aligned to V*sizeof(TO)).
template <typename TO, int V, typename A>
NEXAR_D void store_pack(TO* dst, const A* acc) {
  constexpr int B = V * (int)sizeof(TO);
  alignas(16) TO tmp[V];
#pragma unroll
  for (int v = 0; v < V; ++v) tmp[v] = from_acc<TO, A>(acc[v]);
  if constexpr (B % 16 == 0) {
#pragma unroll
    for (int k = 0; k < B / 16; ++k)
      reinterpret_cast<uint4*>(dst)[k] = reinterpret_cast<const uint4*>(tmp)[k];
  } else if constexpr (B == 8) {
    *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(tmp);
  } else if constexpr (B == 4) {
    *reinterpret_cast<uint32_t*>(dst) = *reinterpret_cast<const uint32_t*>(tmp);
  } else {
#pragma unroll
    for (int v = 0; v < V; ++v) dst[v] = tmp[v];
  }
}

template <typename T, typename A, int V>
NEXAR_D void unpack(const uint4& raw, A* out) {
  const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
  for (int v = 0; v < V; ++v) out[v] = to_acc<A, T>(e[v]);
}

// Copy elements [lo,hi) src->dst (same type). The vector path needs 16-byte
// alignment of both at lo; otherwise the copy is element-wise.
template <typename T>
NEXAR_D void copy_range(T* dst, const T* src, unsigned long long lo, unsigned long long hi,
                        bool vec, bool src_remote) {
  constexpr int V = PackOf<T>::V;
  constexpr int U = 4;  // packs in flight per thread (NVLink latency hiding)
  unsigned long long i = lo;
  vec = vec && ((reinterpret_cast<uintptr_t>(dst + lo) | reinterpret_cast<uintptr_t>(src + lo)) & 15u) == 0;
  if (vec) {
    const unsigned long long vhi = lo + (hi - lo) / V * V;
    const unsigned long long stride = (unsigned long long)blockDim.x * V;
    i = lo + (unsigned long long)threadIdx.x * V;
    for (; i + (U - 1) * stride < vhi; i += U * stride) {
      uint4 r[U];
#pragma unroll
      for (int u = 0; u < U; ++u) r[u] = src_remote ? ld16_volatile(src + i + u * stride) : ld16(src + i + u * stride);
#pragma unroll
      for (int u = 0; u < U; ++u) st16(dst + i + u * stride, r[u]);
    }
    for (; i < vhi; i += stride) {
      uint4 r = src_remote ? ld16_volatile(src + i) : ld16(src + i);
      st16(dst + i, r);
    }
    i = vhi;
  }
  for (unsigned long long j = i + threadIdx.x; j < hi; j += blockDim.x) {
    dst[j] = src_remote ? ldv<T>(src + j) : src[j];
  }
}

// Reduce nsrc arrays (in order) over [lo,hi) into dst (type TO), applying
// scale. Source p's element i lives at srcs[p] + i.
template <typename T, typename TO, int OP>
NEXAR_D void reduce_range(TO* dst, const T* const* srcs, int nsrc, unsigned long long lo,
                          unsigned long long hi, float scale, bool vec) {
  using A = typename AccOf<T>::type;
  constexpr int V = PackOf<T>::V;
  constexpr int U = 2;  // packs in flight per source per thread
  unsigned long long i = lo;
  if (vec) {
    const unsigned long long vhi = lo + (hi - lo) / V * V;
    const unsigned long long stride = (unsigned long long)blockDim.x * V;
    i = lo + (unsigned long long)threadIdx.x * V;
    for (; i < vhi; i += U * stride) {
      uint4 raw[kMaxRanks][U];
#pragma unroll
      for (int p = 0; p < kMaxRanks; ++p)
#pragma unroll
        for (int u = 0; u < U; ++u)
          if (p < nsrc && i + u * stride < vhi) raw[p][u] = ld16_volatile(srcs[p] + i + u * stride);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (i + u * stride >= vhi) break;
        A acc[V];
        unpack<T, A, V>(raw[0][u], acc);
#pragma unroll
        for (int p = 1; p < kMaxRanks; ++p) {
          if (p < nsrc) {
            A x[V];
            unpack<T, A, V>(raw[p][u], x);
#pragma unroll
            for (int v = 0; v < V; ++v) acc[v] = Red<OP, A>::apply(acc[v], x[v]);
          }
        }
#pragma unroll
        for (int v = 0; v < V; ++v) acc[v] = scale_acc<A>(acc[v], scale);
        store_pack<TO, V, A>(dst + i + u * stride, acc);
      }
    }
    i = vhi;
  }
  for (unsigned long long j = i + threadIdx.x; j < hi; j += blockDim.x) {
    A acc = to_acc<A, T>(ldv<T>(srcs[0] + j));
    for (int p = 1; p < nsrc; ++p) acc = Red<OP, A>::apply(acc, to_acc<A, T>(ldv<T>(srcs[p] + j)));
    dst[j] = from_acc<TO, A>(scale_acc<A>(acc, scale));
  }
}

// Like reduce_range but writes the result (type T) to ndst destinations,
// e.g. the same offset in every peer's symmetric tensor.
template <typename T, int OP>
NEXAR_D void reduce_push_range(T* const* dsts, int ndst, const T* const* srcs, int nsrc,
                               unsigned long long lo, unsigned long long hi, float scale, bool vec) {
  using A = typename AccOf<T>::type;
  constexpr int V = PackOf<T>::V;
  unsigned long long i = lo;
  if (vec) {
    const unsigned long long vhi = lo + (hi - lo) / V * V;
    for (i = lo + (unsigned long long)threadIdx.x * V; i < vhi; i += (unsigned long long)blockDim.x * V) {
      uint4 raw[kMaxRanks];
#pragma unroll
      for (int p = 0; p < kMaxRanks; ++p)
        if (p < nsrc) raw[p] = ld16_volatile(srcs[p] + i);
      A acc[V];
      unpack<T, A, V>(raw[0], acc);
#pragma unroll
      for (int p = 1; p < kMaxRanks; ++p) {
        if (p < nsrc) {
          A x[V];
          unpack<T, A, V>(raw[p], x);
#pragma unroll
          for (int v = 0; v < V; ++v) acc[v] = Red<OP, A>::apply(acc[v], x[v]);
        }
      }
      alignas(16) T res[V];
#pragma unroll
      for (int v = 0; v < V; ++v) res[v] = from_acc<T, A>(scale_acc<A>(acc[v], scale));
      const uint4 r = *reinterpret_cast<const uint4*>(res);
#pragma unroll
      for (int p = 0; p < kMaxRanks; ++p)
        if (p < ndst) st16(dsts[p] + i, r);
    }
    i = vhi;
  }
  for (unsigned long long j = i + threadIdx.x; j < hi; j += blockDim.x) {
    A acc = to_acc<A, T>(ldv<T>(srcs[0] + j));
    for (int p = 1; p < nsrc; ++p) acc = Red<OP, A>::apply(acc, to_acc<A, T>(ldv<T>(srcs[p] + j)));
    const T r = from_acc<T, A>(scale_acc<A>(acc, scale));
    for (int p = 0; p < ndst; ++p) dsts[p][j] = r;
  }
}

template <typename T>
NEXAR_D T* stage_ptr(const CommDev& c, int owner, int slot) {
  return reinterpret_cast<T*>(c.peer_base[owner] + c.stage_off + (unsigned long long)slot * c.slot_bytes);
}
template <typename T>
NEXAR_D T* heap_ptr(const CommDev& c, int owner, unsigned long long off) {
  return reinterpret_cast<T*>(c.peer_base[owner] + off);
}

// ---------------------------------------------------------------- launch helpers
inline unsigned int pick_blocks(unsigned long long bytes, unsigned int max_blocks) {
  // ~32 KiB per block keeps enough loads in flight; small messages use few
  // blocks so the barrier is cheap.
  unsigned long long b = (bytes + 32767) / 32768;
  if (b < 1) b = 1;
  if (b > max_blocks) b = max_blocks;
  if (b > (unsigned long long)kMaxBlocks) b = kMaxBlocks;
  return (unsigned int)b;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Expand BODY with T (input), TO (output) and OP bound. Mixed input/output
// types (the fused cast) are supported for Sum only.
#define NEXAR_DISPATCH_OUT_OP(dt_in, dt_out, op, ...)                                      \
  if (dt_in == dt_out) {                                                                   \
    NEXAR_DISPATCH_ALL(dt_in, using TO = T; NEXAR_DISPATCH_OP(op, __VA_ARGS__));           \
  } else if (op != kSum) {                                                                 \
    return cudaErrorInvalidValue;                                                          \
  } else {                                                                                 \
    constexpr int OP = kSum;                                                               \
    if (dt_out == kF32 && dt_in == kBF16) {                                                \
      using T = __nv_bfloat16; using TO = float; __VA_ARGS__;                              \
    } else if (dt_out == kF32 && dt_in == kF16) {                                          \
      using T = __half; using TO = float; __VA_ARGS__;                                     \
    } else if (dt_in == kF32 && dt_out == kBF16) {                                         \
      using T = float; using TO = __nv_bfloat16; __VA_ARGS__;                              \
    } else if (dt_in == kF32 && dt_out == kF16) {                                          \
      using T = float; using TO = __half; __VA_ARGS__;                                     \
    } else if (dt_in == kF32 && dt_out == kF8E4M3) {                                       \
      using T = float; using TO = __nv_fp8_e4m3; __VA_ARGS__;                              \
    } else if (dt_in == kBF16 && dt_out == kF8E4M3) {                                      \
      using T = __nv_bfloat16; using TO = __nv_fp8_e4m3; __VA_ARGS__;                      \
    } else {                                                                               \
      return cudaErrorInvalidValue;                                                        \
    }                                                                                      \
  }

}  // namespace nexar
