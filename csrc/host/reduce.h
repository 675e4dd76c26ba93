// CPU elementwise reduction engine (the host oracle and the CPU data path).
//
// Semantics follow nexar/src/reduce.rs:11-137 and reduce_types.rs:
//   * integer Sum/Prod wrap, Min/Max are exact;
//   * identities: Sum 0, Prod 1, Min = type MAX, Max = type MIN (f32::MIN for
//     floats, which rounds to -inf in bf16/f16);
//   * bf16 and f16 are reduced in f32 and rounded back to nearest-even. The
//     reference's AVX2 bf16 path truncates instead (x86_64.rs:163); this
//     engine always rounds to nearest-even so the result does not depend on
//     the CPU's features.
#pragma once
#include "common.h"

namespace nexar {

void reduce_slice(void* dst, const void* src, size_t count, DataType dt, ReduceOp op);
void fill_identity(void* dst, size_t count, DataType dt, ReduceOp op);

uint16_t f32_to_bf16(float f);
float bf16_to_f32(uint16_t h);
uint16_t f32_to_f16(float f);
float f16_to_f32(uint16_t h);

// Which SIMD path the f32/f64 reductions use on this CPU ("avx512f", "avx2", "scalar").
const char* simd_path();

}  // namespace nexar
