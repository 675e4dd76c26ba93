// Host launch API of the NVLS (NVSwitch multicast) collectives.
#pragma once
#include <cuda_runtime.h>

namespace nexar {

struct CommDev;

// True if the NVLS path can take this message: region active, Sum (scaled) of
// f32 / bf16 / f16, 16-byte aligned pointers and a multiple of 16 bytes.
bool nvls_can_reduce(const CommDev& c, int dt, int op, const void* in, const void* out, unsigned long long bytes);
bool nvls_can_move(const CommDev& c, const void* in, const void* out, unsigned long long bytes);

// sym_off >= 0: in == out lives in the NVLS user region at that offset and
// is reduced in place with no staging copies.
cudaError_t launch_all_reduce_nvls(const CommDev& c, const void* in, void* out, int dt, unsigned long long bytes,
                                   float scale, long long sym_off, unsigned int max_blocks, cudaStream_t s);
// in: [world][count] (count_bytes per rank), out: this rank's reduced segment.
// in_sym >= 0: the input lives in the NVLS user region (no staging).
cudaError_t launch_reduce_scatter_nvls(const CommDev& c, const void* in, void* out, int dt,
                                       unsigned long long count_bytes, float scale, long long in_sym,
                                       unsigned int max_blocks, cudaStream_t s);
// out_sym >= 0: the output lives in the NVLS user region (stores land there directly).
cudaError_t launch_all_gather_nvls(const CommDev& c, const void* in, void* out, unsigned long long count_bytes,
                                   long long out_sym, unsigned int max_blocks, cudaStream_t s);
cudaError_t launch_broadcast_nvls(const CommDev& c, const void* in, void* out, unsigned long long bytes, int root,
                                  long long out_sym, unsigned int max_blocks, cudaStream_t s);

}  // namespace nexar
