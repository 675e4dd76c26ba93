// NexarClient: the communicator of the host runtime.
//
// API and semantics follow the reference's NexarClient
// (nexar/src/client/async_client.rs:62-414 and the impl blocks in
// collectives.rs, collectives_nb.rs, byte_transport.rs, messaging.rs,
// split.rs, rebuild.rs, elastic.rs, bootstrap.rs). Calls are synchronous;
// the *_nb variants run on a worker thread and return a CollectiveHandle.
//
// A Mesh owns the TCP connections, the per-source mailboxes, the heartbeat
// monitor and the relay routing of one process's rank. Communicators derived
// by split / rebuild_excluding / rebuild_adding share their parent's Mesh and
// address peers through a rank map (communicator rank -> mesh rank); their
// traffic is kept apart by comm_id.
#pragma once

#include <condition_variable>
#include <functional>
#include <future>
#include <map>
#include <memory>
#include <set>

#include "cluster.h"
#include "compression.h"
#include "reduce.h"

namespace nexar {

// ------------------------------------------------------------------ device adapter
// Bridge between a device's memory and host-side collectives
// (nexar/src/device/adapter.rs:19-128).
class DeviceAdapter {
 public:
  virtual ~DeviceAdapter() = default;
  virtual std::string name() const = 0;
  virtual bool supports_host_offload() const { return true; }
  // Kernels on the device itself perform collectives (no host staging).
  virtual bool supports_device_collectives() const { return false; }
  // Buffers are ordinary host memory: collectives and p2p read and write them
  // in place, without staging copies.
  virtual bool host_addressable() const { return false; }
  virtual void stage_for_send(const void* ptr, size_t nbytes, uint8_t* out) = 0;
  virtual void receive_to_device(const uint8_t* src, size_t nbytes, void* ptr) = 0;
  virtual void reduce_inplace(void* dst, const void* src, size_t count, DataType dt, ReduceOp op) = 0;
  // Gather / scatter forms (nexar/src/device/adapter.rs: stage_for_send_iov,
  // receive_to_device_iov): regions are packed back to back in `out` / `src`.
  virtual void stage_for_send_iov(const std::vector<std::pair<const void*, size_t>>& iov, uint8_t* out) {
    size_t off = 0;
    for (auto& e : iov) {
      stage_for_send(e.first, e.second, out + off);
      off += e.second;
    }
  }
  virtual void receive_to_device_iov(const uint8_t* src, const std::vector<std::pair<void*, size_t>>& iov) {
    size_t off = 0;
    for (auto& e : iov) {
      receive_to_device(src + off, e.second, e.first);
      off += e.second;
    }
  }
};

// Host pointers used directly (nexar/src/device/cpu.rs:7-52).
class CpuAdapter : public DeviceAdapter {
 public:
  std::string name() const override { return "cpu"; }
  bool host_addressable() const override { return true; }
  void stage_for_send(const void* ptr, size_t n, uint8_t* out) override { std::memcpy(out, ptr, n); }
  void receive_to_device(const uint8_t* src, size_t n, void* ptr) override { std::memcpy(ptr, src, n); }
  void reduce_inplace(void* dst, const void* src, size_t count, DataType dt, ReduceOp op) override {
    reduce_slice(dst, src, count, dt, op);
  }
};

// CUDA device memory staged through host memory (nexar-rdma/src/cuda_adapter.rs:14-139):
// copies go through the CUDA runtime (libcudart, resolved at first use, so this
// module needs no CUDA at build or load time); reduce_inplace brings both
// operands to the host, reduces there and writes the result back. This is the
// path for device pointers that cross hosts; on one box, device pointers go to
// the peer-memory kernels of the device communicator instead.
class CudaStagingAdapter : public DeviceAdapter {
 public:
  std::string name() const override { return "cuda"; }
  void stage_for_send(const void* ptr, size_t n, uint8_t* out) override;
  void receive_to_device(const uint8_t* src, size_t n, void* ptr) override;
  void reduce_inplace(void* dst, const void* src, size_t count, DataType dt, ReduceOp op) override;
  // Whether libcudart could be resolved in this process (no device needed).
  static bool runtime_available();
};

// ------------------------------------------------------------------ mesh
class Mesh : public std::enable_shared_from_this<Mesh> {
 public:
  // `pool` serves the routers' receive buffers (nullptr: a Training-profile pool).
  Mesh(Rank rank, uint32_t world, Config cfg, Bytes token, std::shared_ptr<BufferPool> pool = nullptr);
  ~Mesh();
  const std::shared_ptr<BufferPool>& pool() const { return pool_; }
  Rank rank() const { return rank_; }
  uint32_t world() const { return world_; }
  const Config& config() const { return cfg_; }

  // Adopt an established connection to mesh rank r (handshake done).
  void add_connection(Rank r, std::shared_ptr<Stream> io);
  // TLS for mesh links: with an identity set, dial() / answer() run a mutually
  // authenticated TLS handshake on a freshly connected / accepted socket (and
  // take ownership of it); without one they wrap it as plain TCP.
  void set_tls(const TlsIdentity& id) { tls_id_ = id; }
  bool tls() const { return tls_id_.valid(); }
  std::shared_ptr<Stream> dial(int fd) const;
  std::shared_ptr<Stream> answer(int fd) const;
  void grow(uint32_t new_world);
  bool has_direct(Rank r) const;
  // True if this mesh has links and every one of them runs TLS.
  bool all_encrypted() const;
  std::shared_ptr<Mailbox> box(Rank r) const;
  std::shared_ptr<PeerConnection> conn(Rank r) const;
  void set_routing(const TopologyStrategy& t);
  bool sparse() const { return sparse_; }
  long long next_hop(Rank dest) const;

  // Relay-aware sends (mesh ranks).
  void send_tagged(Rank dest, uint64_t comm, uint64_t tag, const void* p, size_t n);
  void send_raw(Rank dest, uint64_t comm, const void* p, size_t n);
  void send_message(Rank dest, const Message& m, Priority prio);
  // One Data message (tag, this rank, payload) written from the caller's
  // buffer on a direct link; relayed as an encoded message otherwise.
  void send_data(Rank dest, uint32_t tag, const void* p, size_t n);

  // Failure detection (nexar/src/cluster/health.rs:11-103): a background
  // thread sends heartbeats every interval and declares a peer dead when a
  // send fails, when its connection drops, or when nothing has been received
  // from it for longer than the timeout (the reference checks sends only).
  void start_health_monitor();
  void stop_health_monitor();
  std::vector<Rank> dead_ranks() const;
  uint64_t failure_version() const;
  // Wait until the dead set changes after `seen_version` (or timeout).
  std::vector<Rank> wait_failure(uint64_t seen_version, double timeout_s, uint64_t* version_out);
  void mark_dead(Rank r, const std::string& why);

  // Fault injection: shut every connection (nexar/src/client/async_client.rs:399-403).
  void close();
  bool closed() const { return closed_; }
  int listen_fd = -1;
  std::string listen_addr;
  const Bytes& token() const { return token_; }

 private:
  void on_relay(const Message& m);
  void health_loop();
  Rank rank_;
  uint32_t world_;
  Config cfg_;
  Bytes token_;
  std::shared_ptr<BufferPool> pool_;
  TlsIdentity tls_id_;
  mutable std::mutex mu_;
  std::map<Rank, std::shared_ptr<PeerConnection>> conns_;
  std::map<Rank, std::unique_ptr<PeerRouter>> routers_;
  std::vector<std::shared_ptr<Mailbox>> boxes_;
  bool sparse_ = false;
  TopologyStrategy topo_;
  RoutingTable rt_;
  // failures
  mutable std::mutex fmu_;
  std::condition_variable fcv_;
  std::set<Rank> dead_;
  uint64_t fversion_ = 0;
  std::thread health_thr_;
  std::atomic<bool> health_stop_{false};
  std::atomic<bool> closed_{false};
};

// ------------------------------------------------------------------ handles
// Completion handle of a non-blocking operation (nexar/src/collective/handle.rs).
class CollectiveHandle {
 public:
  CollectiveHandle() = default;
  explicit CollectiveHandle(std::shared_future<void> f) : f_(std::move(f)) {}
  void wait() const { f_.get(); }
  bool is_finished() const {
    return f_.valid() && f_.wait_for(std::chrono::seconds(0)) == std::future_status::ready;
  }

 private:
  std::shared_future<void> f_;
};

class CollectiveGroup {
 public:
  void push(CollectiveHandle h) { hs_.push_back(std::move(h)); }
  // Waits for all; rethrows the first error.
  void wait_all();
  size_t size() const { return hs_.size(); }

 private:
  std::vector<CollectiveHandle> hs_;
};

using RpcHandler = std::function<Bytes(const Bytes&)>;

// ------------------------------------------------------------------ client
class NexarClient : public std::enable_shared_from_this<NexarClient> {
 public:
  NexarClient(std::shared_ptr<Mesh> mesh, Rank rank, uint32_t world, uint64_t comm_id,
              std::vector<Rank> rank_map, std::shared_ptr<DeviceAdapter> adapter);

  // ---- bootstrap
  // `pool`: receive buffer pool shared by the ranks' routers (nullptr: one
  // Training-profile pool per rank), the reference's new_with_pool.
  static std::vector<std::shared_ptr<NexarClient>> bootstrap_local(uint32_t world, const Config& cfg,
                                                                   std::shared_ptr<BufferPool> pool = nullptr);
  // Multi-process: every process calls this; the process with rank_hint 0
  // may host the seed (`seed` non-null). Builds the full or sparse mesh.
  static std::shared_ptr<NexarClient> bootstrap_worker(const std::string& seed_addr, const Bytes& token,
                                                       const Config& cfg, const std::string& bind_host,
                                                       std::shared_ptr<BufferPool> pool = nullptr);
  static std::shared_ptr<NexarClient> from_worker_info(WorkerInfo info, const Config& cfg,
                                                       std::shared_ptr<BufferPool> pool = nullptr);

  Rank rank() const { return rank_; }
  uint32_t world_size() const { return world_; }
  uint64_t comm_id() const { return comm_id_; }
  const Config& config() const { return mesh_->config(); }
  std::shared_ptr<Mesh> mesh() const { return mesh_; }
  const std::vector<Rank>& rank_map() const { return rank_map_; }
  std::shared_ptr<DeviceAdapter> adapter() const { return adapter_; }
  // Replace the adapter; call before the first operation that uses it.
  // Communicators derived later by split / rebuild inherit it.
  void set_adapter(std::shared_ptr<DeviceAdapter> a);
  Rank mesh_rank(Rank r) const;
  bool has_direct_peer(Rank r) const { return mesh_->has_direct(mesh_rank(r)); }
  bool is_sparse() const { return mesh_->sparse(); }

  // ---- point to point (nexar/src/client/async_client.rs:312-379)
  void send(const void* ptr, size_t size, Rank dest, uint32_t tag);
  void recv(void* ptr, size_t size, Rank src, uint32_t tag);
  void send_iov(const std::vector<std::pair<const void*, size_t>>& iov, Rank dest, uint32_t tag);
  void recv_iov(const std::vector<std::pair<void*, size_t>>& iov, Rank src, uint32_t tag);
  // The payload of the oldest p2p message from src with this tag.
  Bytes recv_p2p(Rank src, uint32_t tag);
  void send_bytes(Rank dest, const void* p, size_t n);
  Bytes recv_bytes(Rank src);
  void send_bytes_tagged(Rank dest, uint64_t tag, const void* p, size_t n);
  Bytes recv_bytes_tagged(Rank src, uint64_t tag, double timeout_s = -1);
  void send_message_to(Rank dest, const Message& m, Priority prio);
  Message recv_control_from(Rank src, double timeout_s);

  // ---- rpc (nexar/src/client/messaging.rs, nexar/src/rpc/*)
  void register_rpc(uint16_t fn_id, RpcHandler h);
  Bytes rpc(Rank target, uint16_t fn_id, const Bytes& args, double timeout_s = -1);
  Message recv_rpc_request(Rank src, double timeout_s = -1);
  // Handle one request (registry lookup, handler, response).
  void handle_rpc_request(Rank src, const Message& req);
  // Serve requests from every peer on a background thread until stopped.
  void start_rpc_server();
  void stop_rpc_server();

  // ---- collectives on host memory (count semantics as the reference:
  // elements per rank-chunk for all_gather / reduce_scatter / all_to_all /
  // gather / scatter, total elements otherwise)
  void all_reduce(void* ptr, size_t count, DataType dt, ReduceOp op);
  void all_reduce_rs_ag(void* ptr, size_t count, DataType dt, ReduceOp op);
  void all_reduce_bucketed(const std::vector<std::pair<void*, size_t>>& entries, DataType dt, ReduceOp op);
  void all_reduce_compressed(void* ptr, size_t count, DataType dt, ReduceOp op, Compressor& comp, void* residual);
  void broadcast(void* ptr, size_t count, DataType dt, Rank root);
  void all_gather(const void* send, void* recv, size_t count, DataType dt);
  void reduce_scatter(const void* send, void* recv, size_t count, DataType dt, ReduceOp op);
  void reduce(void* ptr, size_t count, DataType dt, ReduceOp op, Rank root);
  void all_to_all(const void* send, void* recv, size_t count, DataType dt);
  void gather(const void* send, void* recv, size_t count, DataType dt, Rank root);
  void scatter(const void* send, void* recv, size_t count, DataType dt, Rank root);
  void scan(void* ptr, size_t count, DataType dt, ReduceOp op);
  void exclusive_scan(void* ptr, size_t count, DataType dt, ReduceOp op);
  void barrier();
  void barrier_with_timeout(double timeout_s);

  // Variants with an explicit collective tag (used by *_nb: the tag is taken
  // at call time so concurrent collectives are isolated).
  uint64_t next_collective_tag() { return collective_tag_.fetch_add(1); }
  void all_reduce_tagged(void* ptr, size_t count, DataType dt, ReduceOp op, uint64_t tag);
  void all_reduce_bucketed_tagged(const std::vector<std::pair<void*, size_t>>& entries, DataType dt, ReduceOp op,
                                  uint64_t tag);
  void all_reduce_compressed_tagged(void* ptr, size_t count, DataType dt, ReduceOp op, Compressor& comp,
                                    void* residual, uint64_t tag);
  CollectiveHandle spawn(std::function<void()> fn);

  // ---- communicator management
  std::shared_ptr<NexarClient> split(uint32_t color, uint32_t key);
  std::shared_ptr<NexarClient> rebuild_excluding(const std::vector<Rank>& dead);
  // Append peers (mesh ranks already connected) to this communicator.
  // `comm_id` != 0 fixes the new communicator's id (joiners must agree on it).
  std::shared_ptr<NexarClient> rebuild_adding(const std::vector<Rank>& new_mesh_ranks, uint64_t comm_id = 0);

  // ---- failures
  std::vector<Rank> dead_ranks() const;  // communicator ranks
  void close() { mesh_->close(); }

  // ---- internals shared with the collectives
  double collective_timeout() const { return mesh_->config().collective_timeout_s; }
  void coll_send(Rank dest, uint64_t tag, const void* p, size_t n, const char* op);
  Bytes coll_recv(Rank src, uint64_t tag, const char* op);
  uint64_t next_barrier_epoch() { return ++barrier_epoch_; }
  std::atomic<uint64_t> barrier_epoch_{0};

 private:
  // Root communicator: a Data message; split / rebuilt ones: a tagged frame.
  void p2p_send(const void* ptr, size_t size, Rank dest, uint32_t tag);
  std::shared_ptr<Mesh> mesh_;
  Rank rank_;
  uint32_t world_;
  uint64_t comm_id_;
  std::vector<Rank> rank_map_;
  std::shared_ptr<DeviceAdapter> adapter_;
  std::atomic<uint64_t> collective_tag_{1};
  std::atomic<uint64_t> split_generation_{0};
  std::atomic<uint64_t> rebuild_generation_{0};
  std::atomic<uint64_t> rpc_req_id_{1};
  std::shared_ptr<std::mutex> rpc_mu_;
  std::shared_ptr<std::map<uint16_t, RpcHandler>> rpc_registry_;
  std::thread rpc_thr_;
  std::atomic<bool> rpc_stop_{false};
};

// Host collective algorithms (collectives.cc).
namespace coll {
size_t ceil_log2(uint32_t n);
uint64_t step_tag(uint64_t base, uint64_t step);
struct ChunkLayout {
  ChunkLayout(size_t count, uint32_t world);
  size_t offset(uint32_t i) const { return offsets[i]; }
  size_t chunk(uint32_t i) const { return i < remainder ? base + 1 : base; }
  std::vector<size_t> offsets;
  size_t base, remainder;
};
void ring_allreduce(NexarClient& c, uint8_t* buf, size_t count, DataType dt, ReduceOp op, uint64_t tag);
void halving_doubling_allreduce(NexarClient& c, uint8_t* buf, size_t count, DataType dt, ReduceOp op, uint64_t tag);
void recursive_doubling_allreduce(NexarClient& c, uint8_t* buf, size_t count, DataType dt, ReduceOp op, uint64_t tag);
void pipelined_ring_allreduce(NexarClient& c, uint8_t* buf, size_t count, DataType dt, ReduceOp op, uint64_t tag);
void rs_ag_allreduce(NexarClient& c, uint8_t* buf, size_t count, DataType dt, ReduceOp op, uint64_t tag);
void ring_allgather(NexarClient& c, const uint8_t* send, uint8_t* recv, size_t count, DataType dt, uint64_t tag);
void ring_reduce_scatter(NexarClient& c, const uint8_t* send, uint8_t* recv, size_t count, DataType dt,
                         ReduceOp op, uint64_t tag);
void broadcast(NexarClient& c, uint8_t* buf, size_t nbytes, Rank root, uint64_t tag);
void reduce(NexarClient& c, uint8_t* buf, size_t count, DataType dt, ReduceOp op, Rank root, uint64_t tag);
void alltoall(NexarClient& c, const uint8_t* send, uint8_t* recv, size_t count, DataType dt, uint64_t tag);
void gather(NexarClient& c, const uint8_t* send, uint8_t* recv, size_t count, DataType dt, Rank root, uint64_t tag);
void scatter(NexarClient& c, const uint8_t* send, uint8_t* recv, size_t count, DataType dt, Rank root, uint64_t tag);
void scan(NexarClient& c, uint8_t* buf, size_t count, DataType dt, ReduceOp op, bool exclusive, uint64_t tag);
void barrier(NexarClient& c, double timeout_s);
void compressed_allreduce(NexarClient& c, uint8_t* buf, size_t count, DataType dt, ReduceOp op, Compressor& comp,
                          uint8_t* residual, uint64_t tag);
}  // namespace coll

}  // namespace nexar
