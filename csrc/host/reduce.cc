#include "reduce.h"

#include <algorithm>
#include <cmath>
#include <limits>

#if defined(__x86_64__) && defined(__GNUC__)
#include <immintrin.h>
#endif

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

// bf16 <-> f32: widen = shift left by 16; narrow = round to nearest even on
// the top 16 bits, NaN kept quiet (f32_to_bf16). The scalar loop is the
// fallback; the x86 paths below do the same integer steps 16 or 8 lanes wide.
void reduce_bf16_scalar(uint16_t* d, const uint16_t* s, size_t n, ReduceOp op) {
  for (size_t i = 0; i < n; ++i) d[i] = f32_to_bf16(apply_f(bf16_to_f32(d[i]), bf16_to_f32(s[i]), op));
}

#if defined(__x86_64__) && defined(__GNUC__)
__attribute__((target("avx512f"))) inline __m512 bf16x16_to_f32(const uint16_t* p) {
  const __m512i w = _mm512_cvtepu16_epi32(_mm256_loadu_si256(reinterpret_cast<const __m256i*>(p)));
  return _mm512_castsi512_ps(_mm512_slli_epi32(w, 16));
}
__attribute__((target("avx512f"))) void reduce_bf16_avx512(uint16_t* d, const uint16_t* s, size_t n, ReduceOp op) {
  const __m512i bias = _mm512_set1_epi32(0x7fff), one = _mm512_set1_epi32(1);
  const __m512i absmask = _mm512_set1_epi32(0x7fffffff), inf = _mm512_set1_epi32(0x7f800000);
  const __m512i quiet = _mm512_set1_epi32(0x40);
  size_t i = 0;
  for (; i + 16 <= n; i += 16) {
    const __m512 a = bf16x16_to_f32(d + i), b = bf16x16_to_f32(s + i);
    __m512 r;
    switch (op) {
      case ReduceOp::Sum: r = _mm512_add_ps(a, b); break;
      case ReduceOp::Prod: r = _mm512_mul_ps(a, b); break;
      case ReduceOp::Min: r = _mm512_min_ps(b, a); break;
      default: r = _mm512_max_ps(b, a); break;
    }
    const __m512i x = _mm512_castps_si512(r);
    const __m512i lsb = _mm512_and_si512(_mm512_srli_epi32(x, 16), one);
    const __m512i rne = _mm512_srli_epi32(_mm512_add_epi32(x, _mm512_add_epi32(bias, lsb)), 16);
    const __m512i qnan = _mm512_or_si512(_mm512_srli_epi32(x, 16), quiet);
    const __mmask16 isnan = _mm512_cmpgt_epi32_mask(_mm512_and_si512(x, absmask), inf);
    const __m512i h = _mm512_mask_blend_epi32(isnan, rne, qnan);
    _mm256_storeu_si256(reinterpret_cast<__m256i*>(d + i), _mm512_cvtepi32_epi16(h));
  }
  reduce_bf16_scalar(d + i, s + i, n - i, op);
}
__attribute__((target("avx2"))) inline __m256 bf16x8_to_f32(const uint16_t* p) {
  const __m256i w = _mm256_cvtepu16_epi32(_mm_loadu_si128(reinterpret_cast<const __m128i*>(p)));
  return _mm256_castsi256_ps(_mm256_slli_epi32(w, 16));
}
__attribute__((target("avx2"))) void reduce_bf16_avx2(uint16_t* d, const uint16_t* s, size_t n, ReduceOp op) {
  const __m256i bias = _mm256_set1_epi32(0x7fff), one = _mm256_set1_epi32(1);
  const __m256i absmask = _mm256_set1_epi32(0x7fffffff), inf = _mm256_set1_epi32(0x7f800000);
  const __m256i quiet = _mm256_set1_epi32(0x40);
  size_t i = 0;
  for (; i + 8 <= n; i += 8) {
    const __m256 a = bf16x8_to_f32(d + i), b = bf16x8_to_f32(s + i);
    __m256 r;
    switch (op) {
      case ReduceOp::Sum: r = _mm256_add_ps(a, b); break;
      case ReduceOp::Prod: r = _mm256_mul_ps(a, b); break;
      case ReduceOp::Min: r = _mm256_min_ps(b, a); break;
      default: r = _mm256_max_ps(b, a); break;
    }
    const __m256i x = _mm256_castps_si256(r);
    const __m256i lsb = _mm256_and_si256(_mm256_srli_epi32(x, 16), one);
    const __m256i rne = _mm256_srli_epi32(_mm256_add_epi32(x, _mm256_add_epi32(bias, lsb)), 16);
    const __m256i qnan = _mm256_or_si256(_mm256_srli_epi32(x, 16), quiet);
    const __m256i isnan = _mm256_cmpgt_epi32(_mm256_and_si256(x, absmask), inf);
    const __m256i h = _mm256_blendv_epi8(rne, qnan, isnan);
    // 8 x u32 (each <= 0xffff) -> 8 x u16: pack within 128-bit lanes, then
    // bring the two lanes' low halves together.
    const __m256i packed = _mm256_permute4x64_epi64(_mm256_packus_epi32(h, h), 0x08);
    _mm_storeu_si128(reinterpret_cast<__m128i*>(d + i), _mm256_castsi256_si128(packed));
  }
  reduce_bf16_scalar(d + i, s + i, n - i, op);
}
#endif

using Half16Fn = void (*)(uint16_t*, const uint16_t*, size_t, ReduceOp);
Half16Fn pick_bf16() {
#if defined(__x86_64__) && defined(__GNUC__)
  __builtin_cpu_init();
  if (__builtin_cpu_supports("avx512f")) return reduce_bf16_avx512;
  if (__builtin_cpu_supports("avx2")) return reduce_bf16_avx2;
#endif
  return reduce_bf16_scalar;
}

void reduce_bf16(uint16_t* d, const uint16_t* s, size_t n, ReduceOp op) {
  static const Half16Fn fn = pick_bf16();
  fn(d, s, n, op);
}

void reduce_f16_scalar(uint16_t* d, const uint16_t* s, size_t n, ReduceOp op) {
  for (size_t i = 0; i < n; ++i) d[i] = f32_to_f16(apply_f(f16_to_f32(d[i]), f16_to_f32(s[i]), op));
}

#if defined(__x86_64__) && defined(__GNUC__)
// Hardware binary16 conversions (vcvtph2ps / vcvtps2ph, round to nearest
// even; the result equals f32_to_f16 except for NaN payload bits). Min / max
// keep the scalar rule `b < a ? b : a`: the x86 min / max return their second
// operand on equality or NaN.
__attribute__((target("avx512f"))) void reduce_f16_avx512(uint16_t* d, const uint16_t* s, size_t n, ReduceOp op) {
  size_t i = 0;
  for (; i + 16 <= n; i += 16) {
    const __m512 a = _mm512_cvtph_ps(_mm256_loadu_si256(reinterpret_cast<const __m256i*>(d + i)));
    const __m512 b = _mm512_cvtph_ps(_mm256_loadu_si256(reinterpret_cast<const __m256i*>(s + i)));
    __m512 r;
    switch (op) {
      case ReduceOp::Sum: r = _mm512_add_ps(a, b); break;
      case ReduceOp::Prod: r = _mm512_mul_ps(a, b); break;
      case ReduceOp::Min: r = _mm512_min_ps(b, a); break;
      default: r = _mm512_max_ps(b, a); break;
    }
    _mm256_storeu_si256(reinterpret_cast<__m256i*>(d + i),
                        _mm512_cvtps_ph(r, _MM_FROUND_TO_NEAREST_INT | _MM_FROUND_NO_EXC));
  }
  reduce_f16_scalar(d + i, s + i, n - i, op);
}
__attribute__((target("avx2,f16c"))) void reduce_f16_avx2(uint16_t* d, const uint16_t* s, size_t n, ReduceOp op) {
  size_t i = 0;
  for (; i + 8 <= n; i += 8) {
    const __m256 a = _mm256_cvtph_ps(_mm_loadu_si128(reinterpret_cast<const __m128i*>(d + i)));
    const __m256 b = _mm256_cvtph_ps(_mm_loadu_si128(reinterpret_cast<const __m128i*>(s + i)));
    __m256 r;
    switch (op) {
      case ReduceOp::Sum: r = _mm256_add_ps(a, b); break;
      case ReduceOp::Prod: r = _mm256_mul_ps(a, b); break;
      case ReduceOp::Min: r = _mm256_min_ps(b, a); break;
      default: r = _mm256_max_ps(b, a); break;
    }
    _mm_storeu_si128(reinterpret_cast<__m128i*>(d + i),
                     _mm256_cvtps_ph(r, _MM_FROUND_TO_NEAREST_INT | _MM_FROUND_NO_EXC));
  }
  reduce_f16_scalar(d + i, s + i, n - i, op);
}
#endif

Half16Fn pick_f16() {
#if defined(__x86_64__) && defined(__GNUC__)
  __builtin_cpu_init();
  if (__builtin_cpu_supports("avx512f")) return reduce_f16_avx512;
  if (__builtin_cpu_supports("avx2") && __builtin_cpu_supports("f16c")) return reduce_f16_avx2;
#endif
  return reduce_f16_scalar;
}

void reduce_f16(uint16_t* d, const uint16_t* s, size_t n, ReduceOp op) {
  static const Half16Fn fn = pick_f16();
  fn(d, s, n, op);
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
