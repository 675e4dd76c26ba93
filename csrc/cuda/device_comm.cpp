#include "device_comm.h"
#include "coll_api.h"
#include "gemm_api.h"

#include <cstring>
#include <unistd.h>

namespace nexar {

static constexpr uint32_t kHandleMagic = 0x4e584231;  // "NXB1"

void check_cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    throw std::runtime_error(std::string("nexar_b200: ") + what + ": " + cudaGetErrorString(e));
  }
}

namespace {
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int d) {
    cudaGetDevice(&prev);
    if (prev != d) check_cuda(cudaSetDevice(d), "cudaSetDevice");
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};
}  // namespace

DeviceComm::DeviceComm(int rank, int world, int device, uint64_t heap_bytes, uint64_t slot_bytes,
                       uint64_t timeout_us)
    : rank_(rank), world_(world), device_(device), heap_bytes_(heap_bytes), slot_bytes_(slot_bytes) {
  if (world < 1 || world > kMaxRanks) throw std::invalid_argument("world size must be in [1, 8]");
  if (rank < 0 || rank >= world) throw std::invalid_argument("rank out of range");
  slot_bytes_ = (slot_bytes_ + 255) / 256 * 256;
  const uint64_t stage_off = kFlagBytes;
  user_off_ = stage_off + 2 * slot_bytes_;
  if (heap_bytes_ < user_off_) heap_bytes_ = user_off_;
  heap_bytes_ = (heap_bytes_ + (2ull << 20) - 1) / (2ull << 20) * (2ull << 20);
  user_next_ = user_off_;
  DeviceGuard g(device_);
  check_cuda(cudaMalloc(&base_, heap_bytes_), "cudaMalloc(symmetric heap)");
  check_cuda(cudaMemset(base_, 0, kFlagBytes), "cudaMemset(flags)");
  check_cuda(cudaMalloc(&ctrl_, 64), "cudaMalloc(ctrl)");
  check_cuda(cudaMemset(ctrl_, 0, 64), "cudaMemset(ctrl)");
  check_cuda(cudaHostAlloc(&status_host_, sizeof(DeviceStatus), cudaHostAllocMapped | cudaHostAllocPortable),
             "cudaHostAlloc(status)");
  std::memset(status_host_, 0, sizeof(DeviceStatus));
  DeviceStatus* status_dev = nullptr;
  check_cuda(cudaHostGetDevicePointer(reinterpret_cast<void**>(&status_dev), status_host_, 0),
             "cudaHostGetDevicePointer");
  check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  for (int p = 0; p < kMaxRanks; ++p) dev_.peer_base[p] = nullptr;
  dev_.peer_base[rank_] = base_;
  dev_.ctrl = ctrl_;
  dev_.status = status_dev;
  dev_.timeout_ns = timeout_us * 1000ull;
  dev_.stage_off = stage_off;
  dev_.slot_bytes = slot_bytes_;
  dev_.rank = rank_;
  dev_.world = world_;
  dev_.nvls_uc = dev_.nvls_mc = nullptr;
  dev_.nvls_bytes = 0;
  dev_.nvls_seq = nullptr;
  dev_.checks = 0;
  dev_.heap_bytes = heap_bytes_;
  if (world_ == 1) connected_ = true;
}

const CUtensorMap* DeviceComm::rs_maps(int M, int N) {
  if (rs_maps_dev_ && rs_maps_m_ == M && rs_maps_n_ == N) return rs_maps_dev_;
  DeviceGuard g(device_);
  if (!rs_maps_dev_)
    check_cuda(cudaMalloc(&rs_maps_dev_, 2 * kMaxRanks * sizeof(CUtensorMap)), "cudaMalloc(rs tensor maps)");
  std::vector<CUtensorMap> maps(2 * kMaxRanks);
  std::memset(maps.data(), 0, maps.size() * sizeof(CUtensorMap));
  for (int s = 0; s < 2; ++s)
    for (int o = 0; o < world_; ++o) {
      char* base = dev_.peer_base[o];
      if (!base) throw std::runtime_error("rs_maps: peer heaps not connected");
      check_cuda(make_tmap_bf16(&maps[s * kMaxRanks + o], base + dev_.stage_off + (uint64_t)s * slot_bytes_, M, N,
                                N, 32, 64),
                 "tensor map (reduce-scatter staging)");
    }
  // In-flight kernels may still read the previous maps.
  check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  check_cuda(cudaMemcpy(rs_maps_dev_, maps.data(), maps.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice),
             "cudaMemcpy(rs tensor maps)");
  rs_maps_m_ = M;
  rs_maps_n_ = N;
  return rs_maps_dev_;
}

void DeviceComm::debug_set_call_counter(unsigned long long v) {
  DeviceGuard g(device_);
  check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  check_cuda(cudaMemcpy(ctrl_, &v, sizeof(v), cudaMemcpyHostToDevice), "cudaMemcpy(call counter)");
}

void DeviceComm::debug_broadcast_raw_root(const void* in, void* out, int dt, unsigned long long n, int root,
                                          cudaStream_t s) {
  if (!dev_.checks) throw std::runtime_error("debug_broadcast_raw_root needs device checks on (set_checks)");
  if ((unsigned long long)n * 16 > slot_bytes_) throw std::invalid_argument("debug_broadcast_raw_root: n too large");
  DeviceGuard g(device_);
  check_cuda(launch_broadcast(dev_, in, out, dt, n, root, 1, s), "debug broadcast");
}

DeviceComm::~DeviceComm() {
  int cur = -1;
  cudaGetDevice(&cur);
  cudaSetDevice(device_);
  cudaDeviceSynchronize();
  nvls_release();
  for (char* p : opened_) cudaIpcCloseMemHandle(p);
  if (base_) cudaFree(base_);
  if (ctrl_) cudaFree(ctrl_);
  if (rs_maps_dev_) cudaFree(rs_maps_dev_);
  if (status_host_) cudaFreeHost(status_host_);
  if (cur >= 0) cudaSetDevice(cur);
}

std::string DeviceComm::export_handle() const {
  HeapHandle h{};
  h.magic = kHandleMagic;
  h.device = device_;
  h.pid = static_cast<uint64_t>(getpid());
  h.base = reinterpret_cast<uint64_t>(base_);
  h.bytes = heap_bytes_;
  DeviceGuard g(device_);
  check_cuda(cudaIpcGetMemHandle(&h.ipc, base_), "cudaIpcGetMemHandle");
  return std::string(reinterpret_cast<const char*>(&h), sizeof(h));
}

void DeviceComm::connect(const std::vector<std::string>& handles) {
  if ((int)handles.size() != world_) throw std::invalid_argument("need one handle per rank");
  DeviceGuard g(device_);
  const uint64_t me = static_cast<uint64_t>(getpid());
  for (int p = 0; p < world_; ++p) {
    if (p == rank_) continue;
    if (handles[p].size() != sizeof(HeapHandle)) throw std::invalid_argument("bad heap handle size");
    HeapHandle h;
    std::memcpy(&h, handles[p].data(), sizeof(h));
    if (h.magic != kHandleMagic) throw std::invalid_argument("bad heap handle magic");
    if (h.bytes != heap_bytes_) throw std::invalid_argument("symmetric heaps differ in size across ranks");
    if (h.pid == me) {
      // Same process (one thread per GPU): plain peer access on the UVA pointer.
      if (h.device != device_) {
        int can = 0;
        check_cuda(cudaDeviceCanAccessPeer(&can, device_, h.device), "cudaDeviceCanAccessPeer");
        if (!can) throw std::runtime_error("GPUs cannot access each other's memory (no P2P)");
        cudaError_t e = cudaDeviceEnablePeerAccess(h.device, 0);
        if (e == cudaErrorPeerAccessAlreadyEnabled) cudaGetLastError();
        else check_cuda(e, "cudaDeviceEnablePeerAccess");
      }
      dev_.peer_base[p] = reinterpret_cast<char*>(h.base);
    } else {
      void* ptr = nullptr;
      check_cuda(cudaIpcOpenMemHandle(&ptr, h.ipc, cudaIpcMemLazyEnablePeerAccess),
                 "cudaIpcOpenMemHandle");
      opened_.push_back(static_cast<char*>(ptr));
      dev_.peer_base[p] = static_cast<char*>(ptr);
    }
  }
  connected_ = true;
}

uint64_t DeviceComm::alloc_symmetric(uint64_t bytes, uint64_t align) {
  if (align < 256) align = 256;
  uint64_t off = (user_next_ + align - 1) / align * align;
  if (off + bytes > heap_bytes_) {
    throw std::runtime_error("symmetric heap exhausted: requested " + std::to_string(bytes) +
                             " bytes, free " + std::to_string(heap_bytes_ - user_next_));
  }
  user_next_ = off + bytes;
  return off;
}

void DeviceComm::reset_symmetric() { user_next_ = user_off_; }

long long DeviceComm::symmetric_offset(const void* ptr, uint64_t bytes) const {
  const char* p = static_cast<const char*>(ptr);
  if (p >= base_ + user_off_ && p + bytes <= base_ + heap_bytes_) return (long long)(p - base_);
  return -1;
}

DeviceStatus DeviceComm::status() const {
  DeviceStatus s;
  std::memcpy(&s, const_cast<const DeviceStatus*>(status_host_), sizeof(s));
  return s;
}

void DeviceComm::clear_status() { std::memset(status_host_, 0, sizeof(DeviceStatus)); }

}  // namespace nexar
