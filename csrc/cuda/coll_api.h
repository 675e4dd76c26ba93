// Host-visible launch API for the peer-memory collective kernels.
#pragma once
#include <cuda_runtime.h>

namespace nexar {

struct CommDev;

// Collective ids recorded in the device status word on a wait timeout.
enum CollOpId : int {
  kOpAllReduce = 1, kOpReduceScatter = 2, kOpAllGather = 3, kOpAllToAll = 4,
  kOpBroadcast = 5, kOpReduce = 6, kOpGather = 7, kOpScatter = 8, kOpScan = 9,
  kOpBarrier = 10, kOpMoeDispatch = 11, kOpMoeCombine = 12, kOpGemmRs = 13,
  kOpAgGemm = 14, kOpCompressed = 15,
};

enum AllReduceAlgo : int { kAlgoAuto = 0, kAlgoOneShot = 1, kAlgoTwoShot = 2, kAlgoNvls = 3 };

cudaError_t launch_all_reduce(const CommDev& c, const void* in, void* out, int dt_in, int dt_out,
                              int op, unsigned long long n, float scale, int algo,
                              long long sym_off, unsigned int max_blocks, cudaStream_t s);
// Strided variants: rank p's block of the strided side starts at p * ld.
cudaError_t launch_reduce_scatter(const CommDev& c, const void* in, void* out, int dt_in,
                                  int dt_out, int op, unsigned long long count,
                                  unsigned long long in_ld, float scale, unsigned int max_blocks,
                                  cudaStream_t s);
cudaError_t launch_all_gather(const CommDev& c, const void* in, void* out, int dt,
                              unsigned long long count, unsigned long long out_ld,
                              unsigned int max_blocks, cudaStream_t s);
cudaError_t launch_all_to_all(const CommDev& c, const void* in, void* out, int dt,
                              unsigned long long count, unsigned long long in_ld,
                              unsigned long long out_ld, unsigned int max_blocks, cudaStream_t s);
cudaError_t launch_broadcast(const CommDev& c, const void* in, void* out, int dt,
                             unsigned long long n, int root, unsigned int max_blocks,
                             cudaStream_t s);
cudaError_t launch_reduce(const CommDev& c, const void* in, void* out, int dt_in, int dt_out,
                          int op, unsigned long long n, int root, float scale,
                          unsigned int max_blocks, cudaStream_t s);
cudaError_t launch_gather(const CommDev& c, const void* in, void* out, int dt,
                          unsigned long long count, unsigned long long out_ld, int root,
                          unsigned int max_blocks, cudaStream_t s);
cudaError_t launch_scatter(const CommDev& c, const void* in, void* out, int dt,
                           unsigned long long count, unsigned long long in_ld, int root,
                           unsigned int max_blocks, cudaStream_t s);
cudaError_t launch_scan(const CommDev& c, const void* in, void* out, int dt, int op,
                        unsigned long long n, bool exclusive, unsigned int max_blocks,
                        cudaStream_t s);
cudaError_t launch_barrier(const CommDev& c, cudaStream_t s);
cudaError_t launch_reduce_inplace(void* dst, const void* src, int dt, int op,
                                  unsigned long long n, cudaStream_t s);

}  // namespace nexar
