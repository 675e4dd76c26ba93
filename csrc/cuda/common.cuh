// Shared device helpers for the sm_100a kernels of nexar_b200.
//
// Element codes follow the reference wire format (nexar/src/types.rs:13-24,
// `DataType` repr(u8) 0..9); FP8 E4M3 = 10 and E5M2 = 11 are additions for the
// block-scaled fp8 paths and do not renumber the reference codes.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include "comm_types.h"

namespace nexar {

#define NEXAR_HD __host__ __device__ __forceinline__
#define NEXAR_D __device__ __forceinline__

// ---------------------------------------------------------------- memory ops
NEXAR_D unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

NEXAR_D unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
NEXAR_D void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" :: "l"(p), "l"(v) : "memory");
}
NEXAR_D void st_relaxed_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" :: "l"(p), "l"(v) : "memory");
}
NEXAR_D unsigned int ld_acquire_gpu_u32(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
NEXAR_D void fence_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// 16-byte vector loads/stores. `volatile` loads bypass L1 for peer memory that
// another GPU writes while this kernel runs.
NEXAR_D uint4 ld16(const void* p) { return *reinterpret_cast<const uint4*>(p); }
NEXAR_D uint4 ld16_volatile(const void* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p) : "memory");
  return v;
}
// L2-coherent 16-byte load (bypasses L1): for data another GPU or CTA
// published through a release/acquire flag that this CTA already observed.
NEXAR_D uint4 ld16_cg(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
NEXAR_D uint4 ld16_nc(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
NEXAR_D void st16(void* p, uint4 v) { *reinterpret_cast<uint4*>(p) = v; }

// Scalar volatile load of any 1/2/4/8-byte element type (peer memory).
template <typename T> NEXAR_D T ldv(const T* p) {
  T r;
  if constexpr (sizeof(T) == 1) {
    uint8_t v = *reinterpret_cast<const volatile uint8_t*>(p);
    memcpy(&r, &v, 1);
  } else if constexpr (sizeof(T) == 2) {
    uint16_t v = *reinterpret_cast<const volatile uint16_t*>(p);
    memcpy(&r, &v, 2);
  } else if constexpr (sizeof(T) == 4) {
    uint32_t v = *reinterpret_cast<const volatile uint32_t*>(p);
    memcpy(&r, &v, 4);
  } else {
    uint64_t v = *reinterpret_cast<const volatile uint64_t*>(p);
    memcpy(&r, &v, 8);
  }
  return r;
}

// ---------------------------------------------------------------- type traits
template <typename T> struct AccOf { using type = T; };
template <> struct AccOf<__half> { using type = float; };
template <> struct AccOf<__nv_bfloat16> { using type = float; };
template <> struct AccOf<__nv_fp8_e4m3> { using type = float; };
template <> struct AccOf<__nv_fp8_e5m2> { using type = float; };

template <typename A, typename T> NEXAR_D A to_acc(T v) { return static_cast<A>(v); }
template <> NEXAR_D float to_acc<float, __half>(__half v) { return __half2float(v); }
template <> NEXAR_D float to_acc<float, __nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <> NEXAR_D float to_acc<float, __nv_fp8_e4m3>(__nv_fp8_e4m3 v) { return static_cast<float>(v); }
template <> NEXAR_D float to_acc<float, __nv_fp8_e5m2>(__nv_fp8_e5m2 v) { return static_cast<float>(v); }

template <typename T, typename A> NEXAR_D T from_acc(A v) { return static_cast<T>(v); }
template <> NEXAR_D __half from_acc<__half, float>(float v) { return __float2half_rn(v); }
template <> NEXAR_D __nv_bfloat16 from_acc<__nv_bfloat16, float>(float v) { return __float2bfloat16_rn(v); }
template <> NEXAR_D __nv_fp8_e4m3 from_acc<__nv_fp8_e4m3, float>(float v) { return __nv_fp8_e4m3(v); }
template <> NEXAR_D __nv_fp8_e5m2 from_acc<__nv_fp8_e5m2, float>(float v) { return __nv_fp8_e5m2(v); }
template <> NEXAR_D float from_acc<float, float>(float v) { return v; }

// Reduction operators. Integer Sum/Prod wrap (two's complement), matching the
// reference's wrapping_add / wrapping_mul (nexar/src/reduce_types.rs).
template <int OP, typename A> struct Red;
template <typename A> struct Red<kSum, A> { static NEXAR_D A apply(A a, A b) { return a + b; } };
template <typename A> struct Red<kProd, A> { static NEXAR_D A apply(A a, A b) { return a * b; } };
template <typename A> struct Red<kMin, A> { static NEXAR_D A apply(A a, A b) { return b < a ? b : a; } };
template <typename A> struct Red<kMax, A> { static NEXAR_D A apply(A a, A b) { return b > a ? b : a; } };
template <> struct Red<kMin, float> { static NEXAR_D float apply(float a, float b) { return fminf(a, b); } };
template <> struct Red<kMax, float> { static NEXAR_D float apply(float a, float b) { return fmaxf(a, b); } };
template <> struct Red<kMin, double> { static NEXAR_D double apply(double a, double b) { return fmin(a, b); } };
template <> struct Red<kMax, double> { static NEXAR_D double apply(double a, double b) { return fmax(a, b); } };
// Wrapping signed arithmetic through the unsigned type avoids UB.
template <> struct Red<kSum, int32_t> { static NEXAR_D int32_t apply(int32_t a, int32_t b) { return (int32_t)((uint32_t)a + (uint32_t)b); } };
template <> struct Red<kProd, int32_t> { static NEXAR_D int32_t apply(int32_t a, int32_t b) { return (int32_t)((uint32_t)a * (uint32_t)b); } };
template <> struct Red<kSum, int64_t> { static NEXAR_D int64_t apply(int64_t a, int64_t b) { return (int64_t)((uint64_t)a + (uint64_t)b); } };
template <> struct Red<kProd, int64_t> { static NEXAR_D int64_t apply(int64_t a, int64_t b) { return (int64_t)((uint64_t)a * (uint64_t)b); } };
template <> struct Red<kSum, int8_t> { static NEXAR_D int8_t apply(int8_t a, int8_t b) { return (int8_t)((uint8_t)a + (uint8_t)b); } };
template <> struct Red<kProd, int8_t> { static NEXAR_D int8_t apply(int8_t a, int8_t b) { return (int8_t)((uint8_t)a * (uint8_t)b); } };
template <> struct Red<kSum, uint8_t> { static NEXAR_D uint8_t apply(uint8_t a, uint8_t b) { return (uint8_t)(a + b); } };
template <> struct Red<kProd, uint8_t> { static NEXAR_D uint8_t apply(uint8_t a, uint8_t b) { return (uint8_t)(a * b); } };

// Scaling only applies to floating accumulators; integer results are unscaled.
template <typename A> NEXAR_D A scale_acc(A v, float s) { return v; }
template <> NEXAR_D float scale_acc<float>(float v, float s) { return v * s; }
template <> NEXAR_D double scale_acc<double>(double v, float s) { return v * (double)s; }

NEXAR_HD int dtype_size(int dt) {
  switch (dt) {
    case kF32: case kI32: case kU32: return 4;
    case kF64: case kI64: case kU64: return 8;
    case kF16: case kBF16: return 2;
    case kI8: case kU8: case kF8E4M3: case kF8E5M2: return 1;
    default: return 0;
  }
}

NEXAR_HD unsigned int ceil_div_u(unsigned long long a, unsigned long long b) {
  return (unsigned int)((a + b - 1) / b);
}

}  // namespace nexar

// Dispatch helpers: expand BODY with `T` bound to the element type of `dt`.
#define NEXAR_DISPATCH_ALL(dt, ...)                                         \
  switch (dt) {                                                             \
    case nexar::kF32: { using T = float; __VA_ARGS__; break; }              \
    case nexar::kF64: { using T = double; __VA_ARGS__; break; }             \
    case nexar::kF16: { using T = __half; __VA_ARGS__; break; }             \
    case nexar::kBF16: { using T = __nv_bfloat16; __VA_ARGS__; break; }     \
    case nexar::kI8: { using T = int8_t; __VA_ARGS__; break; }              \
    case nexar::kI32: { using T = int32_t; __VA_ARGS__; break; }            \
    case nexar::kI64: { using T = int64_t; __VA_ARGS__; break; }            \
    case nexar::kU8: { using T = uint8_t; __VA_ARGS__; break; }             \
    case nexar::kU32: { using T = uint32_t; __VA_ARGS__; break; }           \
    case nexar::kU64: { using T = uint64_t; __VA_ARGS__; break; }           \
    case nexar::kF8E4M3: { using T = __nv_fp8_e4m3; __VA_ARGS__; break; }   \
    case nexar::kF8E5M2: { using T = __nv_fp8_e5m2; __VA_ARGS__; break; }   \
    default: return cudaErrorInvalidValue;                                  \
  }

#define NEXAR_DISPATCH_OP(op, ...)                                          \
  switch (op) {                                                             \
    case nexar::kSum: { constexpr int OP = nexar::kSum; __VA_ARGS__; break; }   \
    case nexar::kProd: { constexpr int OP = nexar::kProd; __VA_ARGS__; break; } \
    case nexar::kMin: { constexpr int OP = nexar::kMin; __VA_ARGS__; break; }   \
    case nexar::kMax: { constexpr int OP = nexar::kMax; __VA_ARGS__; break; }   \
    default: return cudaErrorInvalidValue;                                  \
  }
