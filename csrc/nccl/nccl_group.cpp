// NcclGroup: one raw NCCL communicator bound to one device and one stream.
//
// This is the on-box counterpart of the reference's `NcclGroup`
// (nexar-nccl/src/group.rs:16-326) and of its type mapping
// (nexar-nccl/src/types.rs:5-28). nexar_b200 runs every intra-box collective on
// its own peer-memory kernels; this group carries what stays on NCCL:
//   * pipeline-style point-to-point send / recv (ncclSend / ncclRecv), and
//   * the reference's own NCCL call sequence, which the collective benchmarks
//     use as their comparator.
//
// libnccl is resolved at run time (dlopen of the copy that torch already
// loaded, else an explicit path), as the reference loads it dynamically through
// cudarc. Pointers are raw device addresses (u64) as in nexar's pointer model;
// counts are elements. The DataType / ReduceOp arguments are nexar's wire codes
// (F32=0 .. U64=9, F8E4M3=10, F8E5M2=11; Sum=0, Prod=1, Min=2, Max=3).
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>
#include <pybind11/pybind11.h>

#include <cstdint>
#include <cstring>
#include <mutex>
#include <stdexcept>
#include <string>

namespace py = pybind11;

namespace {

// ---------------------------------------------------------------- library
struct NcclApi {
  void* handle = nullptr;
  std::string path;
  decltype(&ncclGetVersion) GetVersion = nullptr;
  decltype(&ncclGetUniqueId) GetUniqueId = nullptr;
  decltype(&ncclCommInitRank) CommInitRank = nullptr;
  decltype(&ncclCommAbort) CommAbort = nullptr;
  decltype(&ncclCommDestroy) CommDestroy = nullptr;
  decltype(&ncclCommGetAsyncError) CommGetAsyncError = nullptr;
  decltype(&ncclGetErrorString) GetErrorString = nullptr;
  decltype(&ncclGetLastError) GetLastError = nullptr;
  decltype(&ncclAllReduce) AllReduce = nullptr;
  decltype(&ncclReduceScatter) ReduceScatter = nullptr;
  decltype(&ncclAllGather) AllGather = nullptr;
  decltype(&ncclBroadcast) Broadcast = nullptr;
  decltype(&ncclReduce) Reduce = nullptr;
  decltype(&ncclSend) Send = nullptr;
  decltype(&ncclRecv) Recv = nullptr;
  decltype(&ncclGroupStart) GroupStart = nullptr;
  decltype(&ncclGroupEnd) GroupEnd = nullptr;
};

NcclApi g_api;
std::mutex g_api_mu;

template <typename F>
void resolve(void* h, F& fn, const char* name) {
  fn = reinterpret_cast<F>(dlsym(h, name));
  if (!fn) throw std::runtime_error(std::string("libnccl has no symbol ") + name);
}

// Loads libnccl once per process. `path` is used only when no copy is loaded yet.
const NcclApi& api(const std::string& path = "") {
  std::lock_guard<std::mutex> lk(g_api_mu);
  if (g_api.handle) return g_api;
  void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
  std::string where = "libnccl.so.2 (already loaded)";
  if (!h && !path.empty()) {
    h = dlopen(path.c_str(), RTLD_NOW | RTLD_GLOBAL);
    where = path;
  }
  if (!h) {
    h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    where = "libnccl.so.2";
  }
  if (!h) {
    const char* e = dlerror();
    throw std::runtime_error(std::string("cannot load libnccl: ") + (e ? e : "unknown error"));
  }
  NcclApi a;
  a.handle = h;
  a.path = where;
  resolve(h, a.GetVersion, "ncclGetVersion");
  resolve(h, a.GetUniqueId, "ncclGetUniqueId");
  resolve(h, a.CommInitRank, "ncclCommInitRank");
  resolve(h, a.CommAbort, "ncclCommAbort");
  resolve(h, a.CommDestroy, "ncclCommDestroy");
  resolve(h, a.CommGetAsyncError, "ncclCommGetAsyncError");
  resolve(h, a.GetErrorString, "ncclGetErrorString");
  resolve(h, a.GetLastError, "ncclGetLastError");
  resolve(h, a.AllReduce, "ncclAllReduce");
  resolve(h, a.ReduceScatter, "ncclReduceScatter");
  resolve(h, a.AllGather, "ncclAllGather");
  resolve(h, a.Broadcast, "ncclBroadcast");
  resolve(h, a.Reduce, "ncclReduce");
  resolve(h, a.Send, "ncclSend");
  resolve(h, a.Recv, "ncclRecv");
  resolve(h, a.GroupStart, "ncclGroupStart");
  resolve(h, a.GroupEnd, "ncclGroupEnd");
  g_api = a;  // published only once every symbol resolved
  return g_api;
}

// ---------------------------------------------------------------- errors
// Raised as nexar_b200.device.nccl.NcclCommError subclasses by the Python layer,
// which maps the `kind` prefix ("nccl", "cuda", "usage").
[[noreturn]] void fail(const std::string& kind, const std::string& what) {
  throw std::runtime_error(kind + ": " + what);
}

void check_nccl(ncclResult_t r, const char* call, ncclComm_t comm = nullptr) {
  if (r == ncclSuccess || r == ncclInProgress) return;
  const NcclApi& a = api();
  std::string msg = std::string(call) + " failed: " + a.GetErrorString(r) + " (ncclResult " +
                    std::to_string(static_cast<int>(r)) + ")";
  const char* last = a.GetLastError(comm);
  if (last && *last) msg += ": " + std::string(last);
  fail("nccl", msg);
}

void check_cuda(cudaError_t e, const char* call) {
  if (e == cudaSuccess) return;
  fail("cuda", std::string(call) + " failed: " + cudaGetErrorString(e));
}

// ---------------------------------------------------------------- mapping
// nexar DataType code -> NCCL type (nexar-nccl/src/types.rs:5-19, plus fp8).
ncclDataType_t to_nccl_dtype(int code) {
  switch (code) {
    case 0: return ncclFloat32;
    case 1: return ncclFloat64;
    case 2: return ncclFloat16;
    case 3: return ncclBfloat16;
    case 4: return ncclInt8;
    case 5: return ncclInt32;
    case 6: return ncclInt64;
    case 7: return ncclUint8;
    case 8: return ncclUint32;
    case 9: return ncclUint64;
    case 10: return ncclFloat8e4m3;
    case 11: return ncclFloat8e5m2;
    default: fail("usage", "unknown DataType code " + std::to_string(code));
  }
}

// nexar ReduceOp code (Sum, Prod, Min, Max) -> NCCL op (nexar-nccl/src/types.rs:21-28).
// NCCL orders its ops Sum, Prod, Max, Min, so Min and Max swap places.
ncclRedOp_t to_nccl_op(int code) {
  switch (code) {
    case 0: return ncclSum;
    case 1: return ncclProd;
    case 2: return ncclMin;
    case 3: return ncclMax;
    default: fail("usage", "unknown ReduceOp code " + std::to_string(code));
  }
}

// Restores the calling thread's current device on scope exit.
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    check_cuda(cudaGetDevice(&prev), "cudaGetDevice");
    if (prev != dev) check_cuda(cudaSetDevice(dev), "cudaSetDevice");
  }
  ~DeviceGuard() {
    int cur = -1;
    if (cudaGetDevice(&cur) == cudaSuccess && cur != prev && prev >= 0) cudaSetDevice(prev);
  }
};

py::bytes unique_id() {
  ncclUniqueId id;
  {
    py::gil_scoped_release nogil;
    check_nccl(api().GetUniqueId(&id), "ncclGetUniqueId");
  }
  return py::bytes(id.internal, NCCL_UNIQUE_ID_BYTES);
}

// ---------------------------------------------------------------- group
class NcclGroup {
 public:
  // Collective over the `local_world` ranks that pass the same `id`; blocks
  // until all of them have joined. `stream` 0 makes a private non-blocking
  // stream on `device`, otherwise the given stream handle is used (not owned).
  NcclGroup(int local_rank, int local_world, const std::string& id, int device, std::uintptr_t stream)
      : local_rank_(local_rank), local_world_(local_world), device_(device) {
    if (local_world < 1 || local_rank < 0 || local_rank >= local_world)
      fail("usage", "invalid rank " + std::to_string(local_rank) + ": world size is " +
                        std::to_string(local_world));
    if (id.size() != NCCL_UNIQUE_ID_BYTES)
      fail("usage", "an NCCL id is " + std::to_string(NCCL_UNIQUE_ID_BYTES) + " bytes, got " +
                        std::to_string(id.size()));
    ncclUniqueId uid;
    std::memcpy(uid.internal, id.data(), NCCL_UNIQUE_ID_BYTES);
    const NcclApi& a = api();
    py::gil_scoped_release nogil;
    DeviceGuard g(device_);
    if (stream == 0) {
      check_cuda(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "cudaStreamCreateWithFlags");
      own_stream_ = true;
    } else {
      stream_ = reinterpret_cast<cudaStream_t>(stream);
    }
    ncclResult_t r = a.CommInitRank(&comm_, local_world, uid, local_rank);
    if (r != ncclSuccess) {
      if (own_stream_) cudaStreamDestroy(stream_);
      own_stream_ = false;
      comm_ = nullptr;
      check_nccl(r, "ncclCommInitRank");
    }
  }

  ~NcclGroup() {
    // As the reference's Drop: abort, which never waits on peers.
    if (comm_) api().CommAbort(comm_);
    comm_ = nullptr;
    if (own_stream_) {
      int prev = -1;
      cudaGetDevice(&prev);
      cudaSetDevice(device_);
      cudaStreamDestroy(stream_);
      if (prev >= 0) cudaSetDevice(prev);
    }
  }

  NcclGroup(const NcclGroup&) = delete;
  NcclGroup& operator=(const NcclGroup&) = delete;

  int local_rank() const { return local_rank_; }
  int local_world() const { return local_world_; }
  int device() const { return device_; }
  std::uintptr_t stream() const { return reinterpret_cast<std::uintptr_t>(stream_); }
  bool closed() const { return comm_ == nullptr; }

  void all_reduce_inplace(std::uintptr_t ptr, size_t count, int dt, int op) {
    all_reduce(ptr, ptr, count, dt, op);
  }

  void all_reduce(std::uintptr_t send, std::uintptr_t recv, size_t count, int dt, int op) {
    ncclComm_t c = live();
    auto t = to_nccl_dtype(dt);
    auto o = to_nccl_op(op);
    py::gil_scoped_release nogil;
    check_nccl(api().AllReduce(vp(send), vp(recv), count, t, o, c, stream_), "ncclAllReduce", c);
  }

  // `recv_count` elements per rank: send holds recv_count * local_world.
  // Rank r receives the reduction of chunk r.
  void reduce_scatter(std::uintptr_t send, std::uintptr_t recv, size_t recv_count, int dt, int op) {
    ncclComm_t c = live();
    auto t = to_nccl_dtype(dt);
    auto o = to_nccl_op(op);
    py::gil_scoped_release nogil;
    check_nccl(api().ReduceScatter(vp(send), vp(recv), recv_count, t, o, c, stream_), "ncclReduceScatter", c);
  }

  // `send_count` elements per rank: recv holds send_count * local_world in rank order.
  void all_gather(std::uintptr_t send, std::uintptr_t recv, size_t send_count, int dt) {
    ncclComm_t c = live();
    auto t = to_nccl_dtype(dt);
    py::gil_scoped_release nogil;
    check_nccl(api().AllGather(vp(send), vp(recv), send_count, t, c, stream_), "ncclAllGather", c);
  }

  void broadcast_inplace(std::uintptr_t ptr, size_t count, int dt, int root) {
    ncclComm_t c = live();
    check_root(root);
    auto t = to_nccl_dtype(dt);
    py::gil_scoped_release nogil;
    check_nccl(api().Broadcast(vp(ptr), vp(ptr), count, t, root, c, stream_), "ncclBroadcast", c);
  }

  // In place; only the root's buffer holds the result afterwards.
  void reduce_inplace(std::uintptr_t ptr, size_t count, int dt, int op, int root) {
    ncclComm_t c = live();
    check_root(root);
    auto t = to_nccl_dtype(dt);
    auto o = to_nccl_op(op);
    py::gil_scoped_release nogil;
    check_nccl(api().Reduce(vp(ptr), vp(ptr), count, t, o, root, c, stream_), "ncclReduce", c);
  }

  void send(std::uintptr_t ptr, size_t count, int dt, int peer) {
    ncclComm_t c = live();
    check_root(peer);
    auto t = to_nccl_dtype(dt);
    py::gil_scoped_release nogil;
    check_nccl(api().Send(vp(ptr), count, t, peer, c, stream_), "ncclSend", c);
  }

  void recv(std::uintptr_t ptr, size_t count, int dt, int peer) {
    ncclComm_t c = live();
    check_root(peer);
    auto t = to_nccl_dtype(dt);
    py::gil_scoped_release nogil;
    check_nccl(api().Recv(vp(ptr), count, t, peer, c, stream_), "ncclRecv", c);
  }

  // Send to `send_peer` and receive from `recv_peer` as one NCCL group, so a
  // ring shift or a pipeline exchange cannot deadlock on call order.
  void send_recv(std::uintptr_t send_ptr, size_t send_count, int send_peer, std::uintptr_t recv_ptr,
                 size_t recv_count, int recv_peer, int dt) {
    ncclComm_t c = live();
    check_root(send_peer);
    check_root(recv_peer);
    auto t = to_nccl_dtype(dt);
    const NcclApi& a = api();
    py::gil_scoped_release nogil;
    check_nccl(a.GroupStart(), "ncclGroupStart");
    ncclResult_t r1 = a.Send(vp(send_ptr), send_count, t, send_peer, c, stream_);
    ncclResult_t r2 = a.Recv(vp(recv_ptr), recv_count, t, recv_peer, c, stream_);
    ncclResult_t r3 = a.GroupEnd();
    check_nccl(r1, "ncclSend", c);
    check_nccl(r2, "ncclRecv", c);
    check_nccl(r3, "ncclGroupEnd", c);
  }

  void synchronize() {
    live();
    py::gil_scoped_release nogil;
    DeviceGuard g(device_);
    check_cuda(cudaStreamSynchronize(stream_), "cudaStreamSynchronize");
  }

  // Events for overlapping this group's stream with other work
  // (nexar-nccl/src/group.rs: create_event / record_event / stream_wait_event / destroy_event).
  std::uintptr_t create_event() {
    DeviceGuard g(device_);
    cudaEvent_t e = nullptr;
    check_cuda(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreateWithFlags");
    return reinterpret_cast<std::uintptr_t>(e);
  }

  void record_event(std::uintptr_t ev) {
    DeviceGuard g(device_);
    check_cuda(cudaEventRecord(reinterpret_cast<cudaEvent_t>(ev), stream_), "cudaEventRecord");
  }

  // Makes `stream` (0: this group's stream) wait for the event.
  void stream_wait_event(std::uintptr_t stream, std::uintptr_t ev) {
    DeviceGuard g(device_);
    cudaStream_t s = stream ? reinterpret_cast<cudaStream_t>(stream) : stream_;
    check_cuda(cudaStreamWaitEvent(s, reinterpret_cast<cudaEvent_t>(ev), 0), "cudaStreamWaitEvent");
  }

  bool event_query(std::uintptr_t ev) {
    DeviceGuard g(device_);
    cudaError_t e = cudaEventQuery(reinterpret_cast<cudaEvent_t>(ev));
    if (e == cudaErrorNotReady) return false;
    check_cuda(e, "cudaEventQuery");
    return true;
  }

  void destroy_event(std::uintptr_t ev) {
    DeviceGuard g(device_);
    check_cuda(cudaEventDestroy(reinterpret_cast<cudaEvent_t>(ev)), "cudaEventDestroy");
  }

  // The communicator's asynchronous error state (ncclSuccess = 0 while healthy).
  int async_error() {
    ncclComm_t c = live();
    ncclResult_t st = ncclSuccess;
    check_nccl(api().CommGetAsyncError(c, &st), "ncclCommGetAsyncError", c);
    return static_cast<int>(st);
  }

  // Tears the communicator down without waiting on peers (ncclCommAbort).
  void abort() {
    if (!comm_) return;
    ncclComm_t c = comm_;
    comm_ = nullptr;
    py::gil_scoped_release nogil;
    check_nccl(api().CommAbort(c), "ncclCommAbort");
  }

  // Orderly teardown; every rank calls it after its last operation.
  void destroy() {
    if (!comm_) return;
    ncclComm_t c = comm_;
    comm_ = nullptr;
    py::gil_scoped_release nogil;
    DeviceGuard g(device_);
    check_cuda(cudaStreamSynchronize(stream_), "cudaStreamSynchronize");
    check_nccl(api().CommDestroy(c), "ncclCommDestroy");
  }

 private:
  static void* vp(std::uintptr_t p) { return reinterpret_cast<void*>(p); }

  ncclComm_t live() const {
    if (!comm_) fail("usage", "the NCCL communicator was destroyed or aborted");
    return comm_;
  }

  void check_root(int r) const {
    if (r < 0 || r >= local_world_)
      fail("usage", "invalid rank " + std::to_string(r) + ": world size is " + std::to_string(local_world_));
  }

  int local_rank_;
  int local_world_;
  int device_;
  ncclComm_t comm_ = nullptr;
  cudaStream_t stream_ = nullptr;
  bool own_stream_ = false;
};

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "NCCL communicator (libnccl resolved at run time) for device p2p and the NCCL comparator";
  m.attr("UNIQUE_ID_BYTES") = NCCL_UNIQUE_ID_BYTES;
  m.def("load", [](const std::string& path) { return api(path).path; }, py::arg("path") = "",
        "Resolve libnccl (the copy already loaded in the process first); returns where it came from.");
  m.def("version", []() {
    int v = 0;
    check_nccl(api().GetVersion(&v), "ncclGetVersion");
    return v;
  });
  m.def("unique_id", &unique_id, "A fresh 128-byte NCCL unique id (the lead rank creates it).");
  m.def("nccl_dtype", [](int code) { return static_cast<int>(to_nccl_dtype(code)); },
        "NCCL's ncclDataType_t value for a nexar DataType code.");
  m.def("nccl_op", [](int code) { return static_cast<int>(to_nccl_op(code)); },
        "NCCL's ncclRedOp_t value for a nexar ReduceOp code.");
  m.def("error_string", [](int code) { return std::string(api().GetErrorString(static_cast<ncclResult_t>(code))); });

  py::class_<NcclGroup>(m, "NcclGroup")
      .def(py::init<int, int, const std::string&, int, std::uintptr_t>(), py::arg("local_rank"),
           py::arg("local_world"), py::arg("id"), py::arg("device"), py::arg("stream") = 0)
      .def_property_readonly("local_rank", &NcclGroup::local_rank)
      .def_property_readonly("local_world", &NcclGroup::local_world)
      .def_property_readonly("device", &NcclGroup::device)
      .def_property_readonly("stream", &NcclGroup::stream)
      .def_property_readonly("closed", &NcclGroup::closed)
      .def("all_reduce_inplace", &NcclGroup::all_reduce_inplace)
      .def("all_reduce", &NcclGroup::all_reduce)
      .def("reduce_scatter", &NcclGroup::reduce_scatter)
      .def("all_gather", &NcclGroup::all_gather)
      .def("broadcast_inplace", &NcclGroup::broadcast_inplace)
      .def("reduce_inplace", &NcclGroup::reduce_inplace)
      .def("send", &NcclGroup::send)
      .def("recv", &NcclGroup::recv)
      .def("send_recv", &NcclGroup::send_recv)
      .def("synchronize", &NcclGroup::synchronize)
      .def("create_event", &NcclGroup::create_event)
      .def("record_event", &NcclGroup::record_event)
      .def("stream_wait_event", &NcclGroup::stream_wait_event)
      .def("event_query", &NcclGroup::event_query)
      .def("destroy_event", &NcclGroup::destroy_event)
      .def("async_error", &NcclGroup::async_error)
      .def("abort", &NcclGroup::abort)
      .def("destroy", &NcclGroup::destroy);
}
