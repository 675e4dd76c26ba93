#include "reduce.h"

#include <algorithm>
#include <cmath>
#include <limits>

namespace nexar {

// ------------------------------------------------------------ conversions
// bf16: keep the top 16 bits of the f32 pattern, rounding to nearest-even.
uint16_t f32_to_bf16(float f) {
  uint32_t b;
  std::memcpy(&b, &f, 4);
  if ((b & 0x7f800000u) == 0x7f800000u && (b & 0x007fffffu)) return (uint16_t)((b >> 16) | 0x0040u);  // quiet NaN
  const uint32_t lsb = (b >> 16) & 1u;
  b += 0x7fffu + lsb;
  return (uint16_t)(b >> 16);
}
float bf16_to_f32(uint16_t h) {
  uint32_t b = (uint32_t)h << 16;
  float f;
  std::memcpy(&f, &b, 4);
  return f;
}

// IEEE binary16 with round-to-nearest-even, written from the format definition.
uint16_t f32_to_f16(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t exp = (x >> 23) & 0xffu;
  uint32_t man = x & 0x7fffffu;
  if (exp == 0xff) return (uint16_t)(sign | 0x7c00u | (man ? 0x200u : 0u));
  int e = (int)exp - 127 + 15;
  if (e >= 31) return (uint16_t)(sign | 0x7c00u);  // overflow -> inf
  if (e <= 0) {
    // subnormal (or underflow to zero): shift in the implicit bit
    if (e < -10) return (uint16_t)sign;
    man |= 0x800000u;
    const int shift = 14 - e;  // 24-bit mantissa -> (10 + e) bits
    uint32_t q = man >> shift;
    const uint32_t rem = man & ((1u << shift) - 1u);
    const uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (q & 1u))) ++q;
    return (uint16_t)(sign | q);
  }
  uint32_t q = man >> 13;
  const uint32_t rem = man & 0x1fffu;
  uint32_t h = sign | ((uint32_t)e << 10) | q;
  if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) ++h;  // carries into the exponent correctly
  return (uint16_t)h;
}
float f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t man = h & 0x3ffu;
  uint32_t x;
  if (exp == 0) {
    if (man == 0) {
      x = sign;
    } else {
      int e = -1;
      do {
        ++e;
        man <<= 1;
      } while (!(man & 0x400u));
      x = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3ffu) << 13);
    }
  } else if (exp == 31) {
    x = sign | 0x7f800000u | (man << 13);
  } else {
    x = sign | ((exp - 15 + 127) << 23) | (man << 13);
  }
  float f;
  std::memcpy(&f, &x, 4);
  return f;
}

// ------------------------------------------------------------ typed kernels
namespace {

template <typename T> inline T wrap_add(T a, T b) {
  using U = typename std::make_unsigned<T>::type;
  return (T)((U)a + (U)b);
}
template <typename T> inline T wrap_mul(T a, T b) {
  using U = typename std::make_unsigned<T>::type;
  return (T)((U)a * (U)b);
}

template <typename T>
void reduce_int(T* __restrict d, const T* __restrict s, size_t n, ReduceOp op) {
  switch (op) {
    case ReduceOp::Sum: for (size_t i = 0; i < n; ++i) d[i] = wrap_add(d[i], s[i]); break;
    case ReduceOp::Prod: for (size_t i = 0; i < n; ++i) d[i] = wrap_mul(d[i], s[i]); break;
    case ReduceOp::Min: for (size_t i = 0; i < n; ++i) d[i] = std::min(d[i], s[i]); break;
    case ReduceOp::Max: for (size_t i = 0; i < n; ++i) d[i] = std::max(d[i], s[i]); break;
  }
}

// Float loops: the compiler vectorises these; target_clones picks the widest
// ISA the CPU supports at load time (AVX-512F, AVX2, or baseline SSE2).
#if defined(__x86_64__) && defined(__GNUC__) && !defined(__clang__)
#if defined(__SANITIZE_THREAD__) || defined(__SANITIZE_ADDRESS__)
// target_clones resolves through IFUNC during relocation, before a sanitizer
// runtime is initialised: sanitizer builds use the default clone only.
#define NEXAR_CLONES
#else
#define NEXAR_CLONES __attribute__((target_clones("avx512f", "avx2", "default")))
#endif
#else
#define NEXAR_CLONES
#endif

template <typename T>
inline void reduce_float_body(T* __restrict d, const T* __restrict s, size_t n, ReduceOp op) {
  switch (op) {
    case ReduceOp::Sum: for (size_t i = 0; i < n; ++i) d[i] = d[i] + s[i]; break;
    case ReduceOp::Prod: for (size_t i = 0; i < n; ++i) d[i] = d[i] * s[i]; break;
    // IEEE min/max with the reference's NaN-free semantics: b < a ? b : a
    case ReduceOp::Min: for (size_t i = 0; i < n; ++i) d[i] = s[i] < d[i] ? s[i] : d[i]; break;
    case ReduceOp::Max: for (size_t i = 0; i < n; ++i) d[i] = s[i] > d[i] ? s[i] : d[i]; break;
  }
}
NEXAR_CLONES void reduce_f32(float* __restrict d, const float* __restrict s, size_t n, ReduceOp op) {
  reduce_float_body(d, s, n, op);
}
NEXAR_CLONES void reduce_f64(double* __restrict d, const double* __restrict s, size_t n, ReduceOp op) {
  reduce_float_body(d, s, n, op);
}

inline float apply_f(float a, float b, ReduceOp op) {
  switch (op) {
    case ReduceOp::Sum: return a + b;
    case ReduceOp::Prod: return a * b;
    case ReduceOp::Min: return b < a ? b : a;
    case ReduceOp::Max: return b > a ? b : a;
  }
  return a;
}

NEXAR_CLONES void reduce_bf16(uint16_t* __restrict d, const uint16_t* __restrict s, size_t n, ReduceOp op) {
  constexpr size_t kBlk = 256;
  float a[kBlk], b[kBlk];
  for (size_t base = 0; base < n; base += kBlk) {
    const size_t m = std::min(kBlk, n - base);
    for (size_t i = 0; i < m; ++i) {
      a[i] = bf16_to_f32(d[base + i]);
      b[i] = bf16_to_f32(s[base + i]);
    }
    reduce_float_body(a, b, m, op);
    for (size_t i = 0; i < m; ++i) d[base + i] = f32_to_bf16(a[i]);
  }
}

void reduce_f16(uint16_t* d, const uint16_t* s, size_t n, ReduceOp op) {
  for (size_t i = 0; i < n; ++i) d[i] = f32_to_f16(apply_f(f16_to_f32(d[i]), f16_to_f32(s[i]), op));
}

template <typename T> void fill(void* dst, size_t n, T v) {
  T* d = static_cast<T*>(dst);
  for (size_t i = 0; i < n; ++i) d[i] = v;
}

template <typename T> T int_identity(ReduceOp op) {
  switch (op) {
    case ReduceOp::Sum: return 0;
    case ReduceOp::Prod: return 1;
    case ReduceOp::Min: return std::numeric_limits<T>::max();
    case ReduceOp::Max: return std::numeric_limits<T>::min();
  }
  return 0;
}
template <typename T> T float_identity(ReduceOp op) {
  switch (op) {
    case ReduceOp::Sum: return 0;
    case ReduceOp::Prod: return 1;
    case ReduceOp::Min: return std::numeric_limits<T>::max();
    case ReduceOp::Max: return std::numeric_limits<T>::lowest();
  }
  return 0;
}

}  // namespace

void reduce_slice(void* dst, const void* src, size_t n, DataType dt, ReduceOp op) {
  switch (dt) {
    case DataType::F32: reduce_f32((float*)dst, (const float*)src, n, op); break;
    case DataType::F64: reduce_f64((double*)dst, (const double*)src, n, op); break;
    case DataType::BF16: reduce_bf16((uint16_t*)dst, (const uint16_t*)src, n, op); break;
    case DataType::F16: reduce_f16((uint16_t*)dst, (const uint16_t*)src, n, op); break;
    case DataType::I8: reduce_int((int8_t*)dst, (const int8_t*)src, n, op); break;
    case DataType::I32: reduce_int((int32_t*)dst, (const int32_t*)src, n, op); break;
    case DataType::I64: reduce_int((int64_t*)dst, (const int64_t*)src, n, op); break;
    case DataType::U8: reduce_int((uint8_t*)dst, (const uint8_t*)src, n, op); break;
    case DataType::U32: reduce_int((uint32_t*)dst, (const uint32_t*)src, n, op); break;
    case DataType::U64: reduce_int((uint64_t*)dst, (const uint64_t*)src, n, op); break;
    default: fail(Err::UnsupportedDType, std::string("unsupported data type ") + dtype_name(dt) + " for reduce");
  }
}

void fill_identity(void* dst, size_t n, DataType dt, ReduceOp op) {
  switch (dt) {
    case DataType::F32: fill<float>(dst, n, float_identity<float>(op)); break;
    case DataType::F64: fill<double>(dst, n, float_identity<double>(op)); break;
    case DataType::BF16: fill<uint16_t>(dst, n, f32_to_bf16(float_identity<float>(op))); break;
    case DataType::F16: fill<uint16_t>(dst, n, f32_to_f16(float_identity<float>(op))); break;
    case DataType::I8: fill<int8_t>(dst, n, int_identity<int8_t>(op)); break;
    case DataType::I32: fill<int32_t>(dst, n, int_identity<int32_t>(op)); break;
    case DataType::I64: fill<int64_t>(dst, n, int_identity<int64_t>(op)); break;
    case DataType::U8: fill<uint8_t>(dst, n, int_identity<uint8_t>(op)); break;
    case DataType::U32: fill<uint32_t>(dst, n, int_identity<uint32_t>(op)); break;
    case DataType::U64: fill<uint64_t>(dst, n, int_identity<uint64_t>(op)); break;
    default: fail(Err::UnsupportedDType, std::string("unsupported data type ") + dtype_name(dt) + " for identity");
  }
}

const char* simd_path() {
#if defined(__x86_64__) && defined(__GNUC__)
  __builtin_cpu_init();
  if (__builtin_cpu_supports("avx512f")) return "avx512f";
  if (__builtin_cpu_supports("avx2")) return "avx2";
#endif
  return "scalar";
}

}  // namespace nexar
