// NVLS region of the device communicator: physical memory on every GPU bound
// to one NVSwitch multicast object (CUDA driver VMM + multicast API, resolved
// at run time through cudaGetDriverEntryPoint so nothing links libcuda).
//
// Each rank keeps its physical backing private; only the multicast object is
// shared (rank 0 creates it and exports a POSIX file descriptor that the
// other ranks import; the descriptor itself travels over a Unix socket, see
// nexar_b200/device/nvls.py). Kernels then use two views of the region:
//   nvls_uc  this rank's own copy (ordinary loads and stores),
//   nvls_mc  the multicast view: multimem.ld_reduce sums the addressed
//            element over every rank's copy inside the switch, multimem.st /
//            multimem.red write it to every rank's copy at once.
#include <cuda.h>

#include <cstring>
#include <mutex>
#include <unistd.h>

#include "device_comm.h"

namespace nexar {

namespace {
struct DriverApi {
  decltype(&cuDeviceGet) DeviceGet = nullptr;
  decltype(&cuDeviceGetAttribute) DeviceGetAttribute = nullptr;
  decltype(&cuMemCreate) MemCreate = nullptr;
  decltype(&cuMemRelease) MemRelease = nullptr;
  decltype(&cuMemAddressReserve) MemAddressReserve = nullptr;
  decltype(&cuMemAddressFree) MemAddressFree = nullptr;
  decltype(&cuMemMap) MemMap = nullptr;
  decltype(&cuMemUnmap) MemUnmap = nullptr;
  decltype(&cuMemSetAccess) MemSetAccess = nullptr;
  decltype(&cuMemGetAllocationGranularity) MemGetAllocationGranularity = nullptr;
  decltype(&cuMemExportToShareableHandle) MemExportToShareableHandle = nullptr;
  decltype(&cuMemImportFromShareableHandle) MemImportFromShareableHandle = nullptr;
  decltype(&cuMulticastCreate) MulticastCreate = nullptr;
  decltype(&cuMulticastAddDevice) MulticastAddDevice = nullptr;
  decltype(&cuMulticastBindMem) MulticastBindMem = nullptr;
  decltype(&cuMulticastUnbind) MulticastUnbind = nullptr;
  decltype(&cuMulticastGetGranularity) MulticastGetGranularity = nullptr;
  bool ok = false;
};

template <class F>
bool resolve(const char* name, F& fn) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess)
    return false;
  fn = reinterpret_cast<F>(p);
  return true;
}

const DriverApi& api() {
  static DriverApi a;
  static std::once_flag once;
  std::call_once(once, [] {
    bool ok = true;
    ok &= resolve("cuDeviceGet", a.DeviceGet);
    ok &= resolve("cuDeviceGetAttribute", a.DeviceGetAttribute);
    ok &= resolve("cuMemCreate", a.MemCreate);
    ok &= resolve("cuMemRelease", a.MemRelease);
    ok &= resolve("cuMemAddressReserve", a.MemAddressReserve);
    ok &= resolve("cuMemAddressFree", a.MemAddressFree);
    ok &= resolve("cuMemMap", a.MemMap);
    ok &= resolve("cuMemUnmap", a.MemUnmap);
    ok &= resolve("cuMemSetAccess", a.MemSetAccess);
    ok &= resolve("cuMemGetAllocationGranularity", a.MemGetAllocationGranularity);
    ok &= resolve("cuMemExportToShareableHandle", a.MemExportToShareableHandle);
    ok &= resolve("cuMemImportFromShareableHandle", a.MemImportFromShareableHandle);
    ok &= resolve("cuMulticastCreate", a.MulticastCreate);
    ok &= resolve("cuMulticastAddDevice", a.MulticastAddDevice);
    ok &= resolve("cuMulticastBindMem", a.MulticastBindMem);
    ok &= resolve("cuMulticastUnbind", a.MulticastUnbind);
    ok &= resolve("cuMulticastGetGranularity", a.MulticastGetGranularity);
    a.ok = ok;
  });
  return a;
}

void check_cu(CUresult r, const char* what) {
  if (r != CUDA_SUCCESS) throw std::runtime_error(std::string("nexar_b200: ") + what + " failed (CUresult " +
                                                  std::to_string((int)r) + ")");
}

uint64_t round_up(uint64_t v, uint64_t g) { return (v + g - 1) / g * g; }

CUmulticastObjectProp mc_prop(int world, uint64_t bytes) {
  CUmulticastObjectProp p;
  std::memset(&p, 0, sizeof(p));
  p.numDevices = (unsigned)world;
  p.size = bytes;
  p.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  return p;
}

CUmemAllocationProp phys_prop(int device) {
  CUmemAllocationProp prop;
  std::memset(&prop, 0, sizeof(prop));
  prop.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  prop.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  prop.location.id = device;
  // Backing bound to a multicast object must be shareable the same way.
  prop.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  return prop;
}

// Region size: a multiple of both the multicast and the allocation
// granularity (powers of two), fixed before the multicast object exists.
uint64_t nvls_granule(const DriverApi& a, int world, int device) {
  CUmulticastObjectProp p = mc_prop(world, 0);
  size_t g = 0, ag = 0;
  check_cu(a.MulticastGetGranularity(&g, &p, CU_MULTICAST_GRANULARITY_RECOMMENDED), "cuMulticastGetGranularity");
  CUmemAllocationProp prop = phys_prop(device);
  check_cu(a.MemGetAllocationGranularity(&ag, &prop, CU_MEM_ALLOC_GRANULARITY_MINIMUM),
           "cuMemGetAllocationGranularity");
  if (g == 0) g = 2ull << 20;
  return g > ag ? g : ag;
}
}  // namespace

bool DeviceComm::nvls_supported() const {
  const DriverApi& a = api();
  if (!a.ok) return false;
  CUdevice d;
  if (a.DeviceGet(&d, device_) != CUDA_SUCCESS) return false;
  int mc = 0, fd = 0;
  if (a.DeviceGetAttribute(&mc, CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, d) != CUDA_SUCCESS) return false;
  if (a.DeviceGetAttribute(&fd, CU_DEVICE_ATTRIBUTE_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR_SUPPORTED, d) != CUDA_SUCCESS)
    return false;
  return mc != 0 && fd != 0;
}

int DeviceComm::nvls_create(uint64_t bytes) {
  const DriverApi& a = api();
  check_cuda(cudaSetDevice(device_), "cudaSetDevice");  // driver calls need the context current
  if (!a.ok) throw std::runtime_error("nexar_b200: CUDA driver multicast API unavailable");
  if (nvls_mc_handle_) throw std::runtime_error("nexar_b200: NVLS region already created");
  nvls_size_ = round_up(bytes, nvls_granule(a, world_, device_));
  CUmulticastObjectProp p = mc_prop(world_, nvls_size_);
  CUmemGenericAllocationHandle h;
  check_cu(a.MulticastCreate(&h, &p), "cuMulticastCreate");
  nvls_mc_handle_ = h;
  int fd = -1;
  check_cu(a.MemExportToShareableHandle(&fd, h, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0),
           "cuMemExportToShareableHandle(multicast)");
  nvls_fd_ = fd;
  return fd;
}

void DeviceComm::nvls_import(int fd, uint64_t bytes) {
  const DriverApi& a = api();
  check_cuda(cudaSetDevice(device_), "cudaSetDevice");  // driver calls need the context current
  if (!a.ok) throw std::runtime_error("nexar_b200: CUDA driver multicast API unavailable");
  if (nvls_mc_handle_) throw std::runtime_error("nexar_b200: NVLS region already created");
  nvls_size_ = round_up(bytes, nvls_granule(a, world_, device_));
  CUmemGenericAllocationHandle h;
  check_cu(a.MemImportFromShareableHandle(&h, reinterpret_cast<void*>(static_cast<uintptr_t>(fd)),
                                          CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR),
           "cuMemImportFromShareableHandle(multicast)");
  nvls_mc_handle_ = h;
  nvls_fd_ = fd;
}

void DeviceComm::nvls_add_device() {
  const DriverApi& a = api();
  check_cuda(cudaSetDevice(device_), "cudaSetDevice");  // driver calls need the context current
  if (!nvls_mc_handle_) throw std::runtime_error("nexar_b200: NVLS region not created");
  CUdevice d;
  check_cu(a.DeviceGet(&d, device_), "cuDeviceGet");
  check_cu(a.MulticastAddDevice(nvls_mc_handle_, d), "cuMulticastAddDevice");
}

void DeviceComm::nvls_bind_map() {
  const DriverApi& a = api();
  if (!nvls_mc_handle_) throw std::runtime_error("nexar_b200: NVLS region not created");
  int cur = -1;
  cudaGetDevice(&cur);
  check_cuda(cudaSetDevice(device_), "cudaSetDevice");
  CUmemAllocationProp prop = phys_prop(device_);
  size_t ag = 0;
  check_cu(a.MemGetAllocationGranularity(&ag, &prop, CU_MEM_ALLOC_GRANULARITY_MINIMUM),
           "cuMemGetAllocationGranularity");
  CUmemGenericAllocationHandle phys;
  check_cu(a.MemCreate(&phys, nvls_size_, &prop, 0), "cuMemCreate(NVLS backing)");
  nvls_phys_handle_ = phys;
  check_cu(a.MulticastBindMem(nvls_mc_handle_, 0, phys, 0, nvls_size_, 0), "cuMulticastBindMem");
  nvls_bound_ = true;
  CUmemAccessDesc acc;
  std::memset(&acc, 0, sizeof(acc));
  acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  acc.location.id = device_;
  acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  CUdeviceptr uc = 0, mc = 0;
  check_cu(a.MemAddressReserve(&uc, nvls_size_, ag, 0, 0), "cuMemAddressReserve(unicast)");
  check_cu(a.MemMap(uc, nvls_size_, 0, phys, 0), "cuMemMap(unicast)");
  check_cu(a.MemSetAccess(uc, nvls_size_, &acc, 1), "cuMemSetAccess(unicast)");
  check_cu(a.MemAddressReserve(&mc, nvls_size_, ag, 0, 0), "cuMemAddressReserve(multicast)");
  check_cu(a.MemMap(mc, nvls_size_, 0, nvls_mc_handle_, 0), "cuMemMap(multicast)");
  check_cu(a.MemSetAccess(mc, nvls_size_, &acc, 1), "cuMemSetAccess(multicast)");
  check_cuda(cudaMemset(reinterpret_cast<void*>(uc), 0, kNvlsSignalBytes), "cudaMemset(NVLS signals)");
  unsigned int* seq = nullptr;
  check_cuda(cudaMalloc(&seq, kMaxBlocks * sizeof(unsigned int)), "cudaMalloc(NVLS seq)");
  check_cuda(cudaMemset(seq, 0, kMaxBlocks * sizeof(unsigned int)), "cudaMemset(NVLS seq)");
  check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  dev_.nvls_uc = reinterpret_cast<char*>(uc);
  dev_.nvls_mc = reinterpret_cast<char*>(mc);
  dev_.nvls_bytes = nvls_size_;
  dev_.nvls_seq = seq;
  nvls_user_off_ = kNvlsSignalBytes + kNvlsStageBytes;
  if (nvls_user_off_ > nvls_size_) throw std::runtime_error("nexar_b200: NVLS region smaller than its staging area");
  nvls_user_next_ = nvls_user_off_;
  if (cur >= 0) cudaSetDevice(cur);
}

uint64_t DeviceComm::nvls_alloc(uint64_t bytes, uint64_t align) {
  if (!nvls_active()) throw std::runtime_error("nexar_b200: NVLS region not active");
  if (align < 256) align = 256;
  const uint64_t off = (nvls_user_next_ + align - 1) / align * align;
  if (off + bytes > nvls_size_)
    throw std::runtime_error("NVLS region exhausted: requested " + std::to_string(bytes) + " bytes, free " +
                             std::to_string(nvls_size_ - nvls_user_next_));
  nvls_user_next_ = off + bytes;
  return off;
}

void DeviceComm::nvls_reset() { nvls_user_next_ = nvls_user_off_; }

long long DeviceComm::nvls_offset(const void* ptr, uint64_t bytes) const {
  if (!nvls_active()) return -1;
  const char* p = static_cast<const char*>(ptr);
  const char* b = dev_.nvls_uc;
  if (p >= b + nvls_user_off_ && p + bytes <= b + nvls_size_) return (long long)(p - b);
  return -1;
}

void DeviceComm::nvls_release() {
  const DriverApi& a = api();
  if (!a.ok) return;
  if (dev_.nvls_mc) {
    a.MemUnmap(reinterpret_cast<CUdeviceptr>(dev_.nvls_mc), nvls_size_);
    a.MemAddressFree(reinterpret_cast<CUdeviceptr>(dev_.nvls_mc), nvls_size_);
  }
  if (dev_.nvls_uc) {
    a.MemUnmap(reinterpret_cast<CUdeviceptr>(dev_.nvls_uc), nvls_size_);
    a.MemAddressFree(reinterpret_cast<CUdeviceptr>(dev_.nvls_uc), nvls_size_);
  }
  if (nvls_bound_) {
    CUdevice d;
    if (a.DeviceGet(&d, device_) == CUDA_SUCCESS) a.MulticastUnbind(nvls_mc_handle_, d, 0, nvls_size_);
  }
  if (nvls_phys_handle_) a.MemRelease(nvls_phys_handle_);
  if (nvls_mc_handle_) a.MemRelease(nvls_mc_handle_);
  if (dev_.nvls_seq) cudaFree(dev_.nvls_seq);
  if (nvls_fd_ >= 0) close(nvls_fd_);
  dev_.nvls_uc = dev_.nvls_mc = nullptr;
  dev_.nvls_seq = nullptr;
  dev_.nvls_bytes = 0;
  nvls_mc_handle_ = nvls_phys_handle_ = 0;
  nvls_bound_ = false;
  nvls_fd_ = -1;
}

}  // namespace nexar
