// Device communicator: the symmetric heap shared by the ranks of one box and
// the host state that the peer-memory kernels need.
//
// This is the on-box replacement for `NcclGroup` (nexar-nccl/src/group.rs:16-326)
// and for the host staging `CudaAdapter` (nexar-rdma/src/cuda_adapter.rs:14-139):
// device pointers never leave the device; kernels move them over NVLink.
#pragma once
#include <cstdint>
#include <string>
#include <vector>
#include <mutex>
#include <stdexcept>

#include <cuda.h>
#include <cuda_runtime.h>
#include "comm_types.h"

namespace nexar {

struct HeapHandle {
  uint32_t magic;
  int32_t device;
  uint64_t pid;
  uint64_t base;          // raw device VA in the exporting process
  uint64_t bytes;
  cudaIpcMemHandle_t ipc;  // 64 bytes
};

class DeviceComm {
 public:
  DeviceComm(int rank, int world, int device, uint64_t heap_bytes, uint64_t slot_bytes,
             uint64_t timeout_us);
  ~DeviceComm();
  DeviceComm(const DeviceComm&) = delete;
  DeviceComm& operator=(const DeviceComm&) = delete;

  // Serialized handle of this rank's heap, to be exchanged out of band.
  std::string export_handle() const;
  // Map every peer's heap. `handles[p]` is rank p's export_handle().
  void connect(const std::vector<std::string>& handles);
  bool connected() const { return connected_; }

  const CommDev& dev() const { return dev_; }
  int rank() const { return rank_; }
  int world() const { return world_; }
  int device() const { return device_; }
  uint64_t heap_bytes() const { return heap_bytes_; }
  uint64_t slot_bytes() const { return slot_bytes_; }
  uint64_t user_bytes_free() const { return heap_bytes_ - user_next_; }
  char* local_base() const { return base_; }
  char* peer_base(int p) const { return dev_.peer_base[p]; }

  // Bump-allocate `bytes` of symmetric memory; every rank must call this in
  // the same order with the same sizes. Returns the heap offset.
  uint64_t alloc_symmetric(uint64_t bytes, uint64_t align);
  void reset_symmetric();
  // Heap offset of `ptr` if it lies in the user region of the local heap, else -1.
  long long symmetric_offset(const void* ptr, uint64_t bytes) const;

  // Device status word (host-mapped).
  DeviceStatus status() const;
  void clear_status();
  void set_timeout_us(uint64_t us) { dev_.timeout_ns = us * 1000ull; }
  // Device argument checks in every collective kernel (see CommDev::checks).
  bool checks() const { return dev_.checks != 0; }
  void set_checks(bool on) { dev_.checks = on ? 1 : 0; }
  // Test hooks for the checks: overwrite the device call counter (a stale
  // counter makes the next barrier epoch not increase); launch a broadcast
  // kernel with an unvalidated root (refused unless checks are on, so the
  // kernel's entry check always stands between the root and any access).
  void debug_set_call_counter(unsigned long long v);
  // Tensor maps over every rank's staging slots as an [M, N] bf16 matrix
  // (boxes of 32 x 64; [2 slots][kMaxRanks owners], in device memory) for
  // the GEMM -> reduce-scatter epilogue's TMA stores. Rebuilt when (M, N)
  // changes; the rebuild synchronises the device, so it must not happen
  // while a stream is captured (call once per shape before capturing).
  const CUtensorMap* rs_maps(int M, int N);
  void debug_broadcast_raw_root(const void* in, void* out, int dt, unsigned long long n, int root,
                                cudaStream_t s);
  uint64_t timeout_us() const { return dev_.timeout_ns / 1000ull; }

  unsigned int max_blocks = 148;
  // Messages of at least this many bytes take the staged NVLS path when it
  // applies (all-reduce, reduce-scatter input, all-gather output, broadcast).
  // Buffers that live in the NVLS region take the zero-copy NVLS path at any
  // size. Staged all-gather loses to the peer-to-peer kernel: off by default.
  uint64_t nvls_min_bytes = 16ull << 20;
  uint64_t nvls_min_rs_bytes = 16ull << 20;
  uint64_t nvls_min_ag_bytes = ~0ull;
  uint64_t nvls_min_bcast_bytes = 1ull << 20;
  // Algorithm of the last all_reduce call (observability): 1 one-shot,
  // 2 two-shot, 3 NVLS staged, 4 NVLS in place, 5 two-shot in place, 0 local.
  int last_allreduce_algo = 0;

  // ---- NVLS (NVSwitch multicast), multi-process only; see nvls.cpp.
  // Setup order on every rank: rank 0 nvls_create() and hands the returned
  // POSIX fd to the others, which nvls_import() it; then every rank
  // nvls_add_device(); after ALL ranks added their device, every rank
  // nvls_bind_map(). Ranks must run these steps in lock step.
  bool nvls_supported() const;
  int nvls_create(uint64_t bytes);
  void nvls_import(int fd, uint64_t bytes);
  void nvls_add_device();
  void nvls_bind_map();
  bool nvls_active() const { return dev_.nvls_mc != nullptr; }
  uint64_t nvls_bytes() const { return dev_.nvls_bytes; }
  char* nvls_local() const { return dev_.nvls_uc; }
  uint64_t nvls_alloc(uint64_t bytes, uint64_t align);
  void nvls_reset();
  // Offset of [ptr, ptr+bytes) inside the NVLS user region, else -1.
  long long nvls_offset(const void* ptr, uint64_t bytes) const;
  // Unmap and release everything NVLS (also used when setup failed on a peer).
  void nvls_release();

 private:
  uint64_t nvls_size_ = 0, nvls_user_off_ = 0, nvls_user_next_ = 0;
  unsigned long long nvls_mc_handle_ = 0, nvls_phys_handle_ = 0;
  bool nvls_bound_ = false;
  int nvls_fd_ = -1;

  int rank_, world_, device_;
  uint64_t heap_bytes_, slot_bytes_;
  uint64_t user_off_ = 0, user_next_ = 0;
  char* base_ = nullptr;
  unsigned long long* ctrl_ = nullptr;
  DeviceStatus* status_host_ = nullptr;
  std::vector<char*> opened_;  // IPC-opened peer bases (to close)
  bool connected_ = false;
  CommDev dev_{};
  CUtensorMap* rs_maps_dev_ = nullptr;
  int rs_maps_m_ = -1, rs_maps_n_ = -1;
};

void check_cuda(cudaError_t e, const char* what);

}  // namespace nexar
