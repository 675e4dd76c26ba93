// CudaStagingAdapter: device buffers staged through host memory
// (nexar-rdma/src/cuda_adapter.rs:14-139).
//
// The CUDA runtime is resolved with dlopen at first use: the copy already
// loaded in the process (torch loads one) first, then the loader's search.
// Copies use cudaMemcpy with cudaMemcpyDefault, so unified addressing picks
// the direction and the device that owns each pointer. When neither side is
// GPU memory (a host buffer handed to the typed host calls, or a process
// without a GPU) the copy is a plain memcpy.
#include <dlfcn.h>

#include <cstring>
#include <mutex>

#include "client.h"

namespace nexar {
namespace {

// Runtime entry points (signatures of the CUDA runtime API; error codes are ints).
struct PointerAttributes {  // layout of cudaPointerAttributes
  int type;                 // 0 unregistered host, 1 host, 2 device, 3 managed
  int device;
  void* device_pointer;
  void* host_pointer;
};
using MemcpyFn = int (*)(void*, const void*, size_t, int);
using ErrorStringFn = const char* (*)(int);
using PointerAttributesFn = int (*)(PointerAttributes*, const void*);
using GetLastErrorFn = int (*)();
constexpr int kMemcpyDefault = 4;  // cudaMemcpyDefault

struct Cudart {
  MemcpyFn memcpy = nullptr;
  ErrorStringFn error_string = nullptr;
  PointerAttributesFn attributes = nullptr;
  GetLastErrorFn last_error = nullptr;
  std::string error;
};

const Cudart& cudart() {
  static Cudart rt;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = nullptr;
    for (const char* name : {"libcudart.so.12", "libcudart.so"}) {
      h = dlopen(name, RTLD_NOW | RTLD_NOLOAD);
      if (h) break;
    }
    if (!h) {
      for (const char* name : {"libcudart.so.12", "libcudart.so"}) {
        h = dlopen(name, RTLD_NOW | RTLD_GLOBAL);
        if (h) break;
      }
    }
    if (!h) {
      const char* e = dlerror();
      rt.error = std::string("cannot load the CUDA runtime: ") + (e ? e : "not found");
      return;
    }
    rt.memcpy = reinterpret_cast<MemcpyFn>(dlsym(h, "cudaMemcpy"));
    rt.error_string = reinterpret_cast<ErrorStringFn>(dlsym(h, "cudaGetErrorString"));
    rt.attributes = reinterpret_cast<PointerAttributesFn>(dlsym(h, "cudaPointerGetAttributes"));
    rt.last_error = reinterpret_cast<GetLastErrorFn>(dlsym(h, "cudaGetLastError"));
    if (!rt.memcpy || !rt.error_string || !rt.attributes || !rt.last_error) {
      rt.memcpy = nullptr;
      rt.error = "the CUDA runtime lacks cudaMemcpy / cudaGetErrorString / cudaPointerGetAttributes";
    }
  });
  return rt;
}

// Whether `p` is memory a GPU owns (device or managed). A failed query (no
// device in this process, say) means plain host memory; its error is cleared
// so that it does not surface in a later unrelated error check.
bool on_device(const Cudart& rt, const void* p) {
  if (!rt.memcpy) return false;
  PointerAttributes a{};
  if (rt.attributes(&a, p) != 0) {
    rt.last_error();
    return false;
  }
  return a.type == 2 || a.type == 3;
}

void copy(void* dst, const void* src, size_t n, const char* what) {
  if (n == 0) return;
  const Cudart& rt = cudart();
  if (!on_device(rt, dst) && !on_device(rt, src)) {
    std::memcpy(dst, src, n);  // both sides are host memory
    return;
  }
  int e = rt.memcpy(dst, src, n, kMemcpyDefault);
  if (e != 0) fail(Err::DeviceError, std::string("cuda adapter: ") + what + ": " + rt.error_string(e));
}

}  // namespace

bool CudaStagingAdapter::runtime_available() { return cudart().memcpy != nullptr; }

void CudaStagingAdapter::stage_for_send(const void* ptr, size_t n, uint8_t* out) {
  copy(out, ptr, n, "device to host copy");
}

void CudaStagingAdapter::receive_to_device(const uint8_t* src, size_t n, void* ptr) {
  copy(ptr, src, n, "host to device copy");
}

void CudaStagingAdapter::reduce_inplace(void* dst, const void* src, size_t count, DataType dt, ReduceOp op) {
  const size_t nb = count * dtype_size(dt);
  Bytes a(nb), b(nb);
  copy(a.data(), dst, nb, "device to host copy");
  copy(b.data(), src, nb, "device to host copy");
  reduce_slice(a.data(), b.data(), count, dt, op);
  copy(dst, a.data(), nb, "host to device copy");
}

}  // namespace nexar
