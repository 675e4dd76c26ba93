// Python bindings of the host runtime (module nexar_b200._host).
//
// Buffers are passed as raw addresses (int) with element counts, as in the
// reference's pointer API (nexar/src/client/collectives.rs). Blocking calls
// release the GIL. NexarError is raised as the matching nexar_b200.core
// exception class.
#include <sys/socket.h>
#include <unistd.h>

#include <cstring>
#include <pybind11/functional.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include "buffer_pool.h"
#include "client.h"
#include "tls.h"
#include "recovery.h"

namespace py = pybind11;
using namespace nexar;

namespace {
void* P(uint64_t p) { return reinterpret_cast<void*>(p); }
Bytes to_bytes(const py::bytes& b) {
  std::string s = b;
  return Bytes(s.begin(), s.end());
}
py::bytes from_bytes(const Bytes& b) { return py::bytes(reinterpret_cast<const char*>(b.data()), b.size()); }
using GR = py::call_guard<py::gil_scoped_release>;

py::dict msg_to_dict(const Message& m) {
  py::dict d;
  d["kind"] = msg_kind_name(m.kind);
  d["epoch"] = m.epoch;
  d["comm_id"] = m.comm_id;
  d["rank"] = m.rank;
  d["world_size"] = m.world_size;
  d["req_id"] = m.req_id;
  d["fn_id"] = m.fn_id;
  d["tag"] = m.tag;
  d["src_rank"] = m.src_rank;
  d["payload"] = from_bytes(m.payload);
  d["dead_ranks"] = m.dead_ranks;
  d["timestamp_ns"] = m.timestamp_ns;
  return d;
}
}  // namespace

// TLS check over a local socket pair between two identities; both sides
// verify the peer. Returns true if the handshake and an echo succeed.
static bool tls_identities_check(const TlsIdentity& sid, const TlsIdentity& cid) {
  int sv[2];
  if (socketpair(AF_UNIX, SOCK_STREAM, 0, sv) != 0) fail(Err::ConnectionFailed, "socketpair failed");
  bool server_ok = false;
  std::thread srv([&] {
    try {
      auto s = tls_server(sv[0], sid, true, 5.0);
      char b[4];
      server_ok = s->read_exact(b, 4) && std::memcmp(b, "ping", 4) == 0;
      if (server_ok) s->write_all("pong", 4);
    } catch (const std::exception&) {
      server_ok = false;
    }
  });
  bool client_ok = false;
  try {
    auto c = tls_client(sv[1], cid, true, 5.0);
    c->write_all("ping", 4);
    char b[4];
    client_ok = c->read_exact(b, 4) && std::memcmp(b, "pong", 4) == 0;
  } catch (const std::exception&) {
    client_ok = false;
  }
  srv.join();
  return server_ok && client_ok;
}

// A server with an identity from CA `a` and a client with one from CA `a`
// (same_ca) or from an unrelated CA.
static bool tls_pair_check(bool same_ca) {
  auto ca_a = ClusterCA::generate("ca-a");
  auto ca_b = same_ca ? ca_a : ClusterCA::generate("ca-b");
  return tls_identities_check(ca_a->issue("server"), ca_b->issue("client"));
}

// Python subclasses of DeviceAdapter (the reference's DeviceAdapter trait is
// public so applications can bring their own memory). Buffers cross as
// integer addresses; the override runs with the GIL taken, from whichever
// thread runs the collective.
class PyDeviceAdapter : public DeviceAdapter {
 public:
  std::string name() const override { PYBIND11_OVERRIDE_PURE(std::string, DeviceAdapter, name); }
  bool supports_host_offload() const override {
    PYBIND11_OVERRIDE(bool, DeviceAdapter, supports_host_offload);
  }
  bool host_addressable() const override { PYBIND11_OVERRIDE(bool, DeviceAdapter, host_addressable); }
  void stage_for_send(const void* ptr, size_t n, uint8_t* out) override {
    py::gil_scoped_acquire gil;
    py::function f = py::get_override(static_cast<const DeviceAdapter*>(this), "stage_for_send");
    if (!f) fail(Err::DeviceError, "DeviceAdapter subclass lacks stage_for_send");
    f(reinterpret_cast<uint64_t>(ptr), n, reinterpret_cast<uint64_t>(out));
  }
  void receive_to_device(const uint8_t* src, size_t n, void* ptr) override {
    py::gil_scoped_acquire gil;
    py::function f = py::get_override(static_cast<const DeviceAdapter*>(this), "receive_to_device");
    if (!f) fail(Err::DeviceError, "DeviceAdapter subclass lacks receive_to_device");
    f(reinterpret_cast<uint64_t>(src), n, reinterpret_cast<uint64_t>(ptr));
  }
  void reduce_inplace(void* dst, const void* src, size_t count, DataType dt, ReduceOp op) override {
    py::gil_scoped_acquire gil;
    py::function f = py::get_override(static_cast<const DeviceAdapter*>(this), "reduce_inplace");
    if (!f) fail(Err::DeviceError, "DeviceAdapter subclass lacks reduce_inplace");
    f(reinterpret_cast<uint64_t>(dst), reinterpret_cast<uint64_t>(src), count, static_cast<int>(dt),
      static_cast<int>(op));
  }
};

PYBIND11_MODULE(_host, m) {
  m.def("tls_pair_check", &tls_pair_check, py::arg("same_ca"), py::call_guard<py::gil_scoped_release>());
  m.doc() = "nexar_b200 host runtime (C++): TCP control plane, CPU collectives, cluster management";

  py::register_exception_translator([](std::exception_ptr p) {
    try {
      if (p) std::rethrow_exception(p);
    } catch (const NexarError& e) {
      py::gil_scoped_acquire g;
      py::object core = py::module_::import("nexar_b200.core");
      py::object table = core.attr("ERRORS_BY_CODE");
      py::object cls = table.attr("get")((int)e.code(), core.attr("NexarError"));
      PyErr_SetString(cls.ptr(), e.what());
    }
  });

  // ------------------------------------------------------------ config
  py::class_<TopologyStrategy>(m, "TopologyStrategy")
      .def(py::init<>())
      .def_property_readonly("kind", [](const TopologyStrategy& t) { return (int)t.kind; })
      .def_readonly("degree", &TopologyStrategy::degree)
      .def("is_sparse", &TopologyStrategy::is_sparse)
      .def("__str__", &TopologyStrategy::to_string);
  m.def("parse_topology", &parse_topology);

  py::class_<Config>(m, "Config")
      .def(py::init<>())
      .def_static("from_env", &Config::from_env)
      .def_property("topology", [](const Config& c) { return c.topology.to_string(); },
                    [](Config& c, const std::string& s) { c.topology = parse_topology(s); })
      .def_readwrite("collective_timeout_s", &Config::collective_timeout_s)
      .def_readwrite("barrier_timeout_s", &Config::barrier_timeout_s)
      .def_readwrite("rpc_timeout_s", &Config::rpc_timeout_s)
      .def_readwrite("large_msg_bytes", &Config::large_msg_bytes)
      .def_readwrite("small_msg_bytes", &Config::small_msg_bytes)
      .def_readwrite("pipeline_segment_bytes", &Config::pipeline_segment_bytes)
      .def_readwrite("ring_max_world", &Config::ring_max_world)
      .def_readwrite("enable_tcp_bulk_sidecar", &Config::enable_tcp_bulk_sidecar)
      .def_readwrite("encrypt_bulk_transport", &Config::encrypt_bulk_transport)
      .def_readwrite("tls", &Config::tls)
      .def_readwrite("compressed_allreduce_max_bytes", &Config::compressed_allreduce_max_bytes)
      .def_readwrite("heartbeat_interval_s", &Config::heartbeat_interval_s)
      .def_readwrite("heartbeat_timeout_s", &Config::heartbeat_timeout_s)
      .def_readwrite("recovery_timeout_s", &Config::recovery_timeout_s)
      .def_readwrite("elastic_enabled", &Config::elastic_enabled)
      .def_readwrite("elastic_min_world_size", &Config::elastic_min_world_size)
      .def_readwrite("elastic_max_world_size", &Config::elastic_max_world_size)
      .def_readwrite("elastic_checkpoint_timeout_s", &Config::elastic_checkpoint_timeout_s)
      .def_property("recovery_policy", [](const Config& c) { return (int)c.recovery_policy; },
                    [](Config& c, int p) { c.recovery_policy = (RecoveryPolicy)p; })
      .def_readwrite("ar_oneshot_max", &Config::ar_oneshot_max)
      .def_readwrite("device_wait_timeout_us", &Config::device_wait_timeout_us);

  // ------------------------------------------------------------ reduce engine
  m.def("reduce_slice", [](uint64_t dst, uint64_t src, size_t count, int dt, int op) {
    reduce_slice(P(dst), P(src), count, (DataType)dt, (ReduceOp)op);
  }, GR());
  m.def("fill_identity", [](uint64_t dst, size_t count, int dt, int op) { fill_identity(P(dst), count, (DataType)dt, (ReduceOp)op); });
  m.def("f32_to_bf16", &f32_to_bf16);
  m.def("bf16_to_f32", &bf16_to_f32);
  m.def("f32_to_f16", &f32_to_f16);
  m.def("f16_to_f32", &f16_to_f32);
  m.def("simd_path", &simd_path);
  m.def("fnv1a_comm_id", [](const std::vector<py::bytes>& parts) {
    std::vector<Bytes> v;
    for (auto& p : parts) v.push_back(to_bytes(p));
    return fnv1a_comm_id(v);
  });

  // ------------------------------------------------------------ wire
  m.def("encode_header", [](uint32_t len, int prio, int type) {
    Header h;
    h.payload_length = len;
    h.priority = (uint8_t)prio;
    h.message_type = (uint8_t)type;
    uint8_t b[kHeaderSize];
    h.encode(b);
    return py::bytes(reinterpret_cast<char*>(b), kHeaderSize);
  });
  m.def("decode_header", [](const py::bytes& b) -> py::object {
    std::string s = b;
    if (s.size() < kHeaderSize) throw NexarError(Err::DecodeFailed, "header too short");
    Header h;
    if (!Header::decode(reinterpret_cast<const uint8_t*>(s.data()), &h)) return py::none();
    return py::make_tuple(h.payload_length, h.priority, h.message_type);
  });
  m.def("message_roundtrip_selftest", []() {
    // Encode and decode one of every variant; returns the number that round-trip exactly.
    std::vector<Message> ms = {
        Message::hello({1, 2, 3}, "127.0.0.1:9"), Message::welcome(3, 8, {{0, "a:1"}, {1, "b:2"}}),
        Message::barrier(7, 9), Message::barrier_ack(7, 9), Message::heartbeat(123), Message::node_joined(5, "x:1"),
        Message::node_left(5), Message::rpc(1, 2, {9, 9}), Message::rpc_response(1, {8}), Message::data(4, 2, {1, 2, 3}),
        Message::split_request(1, 2), Message::recovery_vote(3, {1, 2}), Message::recovery_agreement(3, {1}),
        Message::elastic_checkpoint(4), Message::elastic_checkpoint_ack(4, {{9, "j:1"}}, {2}, 9),
        Message::relay(1, 2, 77, {5, 5})};
    Message rd;
    rd.kind = MsgKind::RdmaEndpoint;
    rd.lid = 3;
    rd.qpn = 4;
    rd.psn = 5;
    rd.gid = Bytes(16, 7);
    ms.push_back(rd);
    int ok = 0;
    for (auto& x : ms) {
      Bytes e = encode_message(x, Priority::Realtime);
      if (decode_message(e.data(), e.size()) == x) ++ok;
    }
    return py::make_tuple(ok, (int)ms.size());
  });
  m.def("decode_message", [](const py::bytes& b) {
    std::string s = b;
    return msg_to_dict(decode_message(reinterpret_cast<const uint8_t*>(s.data()), s.size()));
  });
  m.def("encode_barrier", [](uint64_t epoch, uint64_t comm, int prio) {
    return from_bytes(encode_message(Message::barrier(epoch, comm), (Priority)prio));
  });
  m.def("encode_data", [](uint32_t tag, uint32_t src, const py::bytes& payload) {
    return from_bytes(encode_message(Message::data(tag, src, to_bytes(payload)), Priority::Bulk));
  });

  // ------------------------------------------------------------ topology
  m.def("build_neighbors", [](const std::string& t, Rank r, uint32_t w) {
    auto s = build_neighbors(parse_topology(t), r, w);
    return std::vector<Rank>(s.begin(), s.end());
  });
  m.def("build_routing_table", [](const std::string& t, Rank r, uint32_t w) {
    RoutingTable rt = build_routing_table(parse_topology(t), r, w);
    return py::make_tuple(std::vector<Rank>(rt.neighbors.begin(), rt.neighbors.end()), rt.next_hop);
  });
  m.def("build_spanning_tree", [](const std::string& t, Rank root, uint32_t w) {
    SpanningTree st = build_spanning_tree(parse_topology(t), root, w);
    return py::make_tuple(st.parent, st.children);
  });
  m.def("find_alternative_hop", [](const std::string& t, Rank r, Rank d, Rank failed, uint32_t w) {
    return find_alternative_hop(parse_topology(t), r, d, failed, w);
  });
  m.def("optimal_ring_order", &optimal_ring_order);

  py::class_<ClusterMap, std::shared_ptr<ClusterMap>>(m, "ClusterMap")
      .def(py::init<>())
      .def("add_peer", &ClusterMap::add_peer)
      .def("remove_peer", &ClusterMap::remove_peer)
      .def("heartbeat", &ClusterMap::heartbeat)
      .def("alive_peers", &ClusterMap::alive_peers)
      .def("check_timeouts", &ClusterMap::check_timeouts)
      .def("size", &ClusterMap::size)
      .def("contains", &ClusterMap::contains)
      .def("addr", &ClusterMap::addr)
      .def_property_readonly("epoch", &ClusterMap::epoch);

  // ------------------------------------------------------------ compression
  py::class_<CompressedTensor>(m, "CompressedTensor")
      .def_property_readonly("k", &CompressedTensor::k)
      .def_property_readonly("data", [](const CompressedTensor& c) { return from_bytes(c.data); })
      .def_property_readonly("indices", &CompressedTensor::indices)
      .def_readonly("original_count", &CompressedTensor::original_count);
  py::class_<Compressor, std::shared_ptr<Compressor>>(m, "Compressor")
      .def("name", &Compressor::name)
      .def("compress", [](Compressor& c, uint64_t input, size_t count, int dt, uint64_t residual) {
        return c.compress(static_cast<const uint8_t*>(P(input)), count, (DataType)dt, static_cast<uint8_t*>(P(residual)));
      }, GR())
      .def("decompress", [](const Compressor& c, const py::bytes& data, size_t count, int dt, uint64_t out) {
        CompressedTensor t;
        t.data = to_bytes(data);
        t.original_count = count;
        t.dtype = (DataType)dt;
        c.decompress(t, static_cast<uint8_t*>(P(out)));
      });
  py::class_<TopKCompressor, Compressor, std::shared_ptr<TopKCompressor>>(m, "TopKCompressor").def(py::init<double>());
  py::class_<RandomKCompressor, Compressor, std::shared_ptr<RandomKCompressor>>(m, "RandomKCompressor").def(py::init<double>());
  py::class_<NoCompression, Compressor, std::shared_ptr<NoCompression>>(m, "NoCompression").def(py::init<>());

  // ------------------------------------------------------------ buffer pool
  py::class_<PooledBuf>(m, "PooledBuf")
      .def_property_readonly("size", &PooledBuf::size)
      .def_property_readonly("tier", [](const PooledBuf& b) { return (int)b.tier(); })
      .def_property_readonly("address", [](PooledBuf& b) { return (uint64_t)b.data(); })
      .def("tobytes", [](PooledBuf& b) { return from_bytes(b.bytes()); });
  py::class_<BufferPool, std::shared_ptr<BufferPool>>(m, "BufferPool")
      .def_static("with_profile", [](int p) { return BufferPool::with_profile((PoolProfile)p); })
      .def_static("with_config", &BufferPool::with_config)
      .def_static("from_tiers", [](std::pair<size_t, size_t> s, std::pair<size_t, size_t> l, std::pair<size_t, size_t> h,
                                   std::pair<size_t, size_t> g) {
        return BufferPool::from_tiers({s.first, s.second}, {l.first, l.second}, {h.first, h.second}, {g.first, g.second});
      })
      .def("checkout", &BufferPool::checkout)
      .def("tier_for_size", [](const BufferPool& b, size_t n) { return (int)b.tier_for_size(n); })
      .def("free_count", [](const BufferPool& b, int t) { return b.free_count((PoolTier)t); })
      .def("blocks_reused", [](const BufferPool& b, int t) { return b.blocks_reused((PoolTier)t); })
      .def("blocks_fresh", [](const BufferPool& b, int t) { return b.blocks_fresh((PoolTier)t); });

  // ------------------------------------------------------------ handles
  py::class_<CollectiveHandle>(m, "CollectiveHandle")
      .def("wait", &CollectiveHandle::wait, GR())
      .def("is_finished", &CollectiveHandle::is_finished);
  py::class_<CollectiveGroup>(m, "CollectiveGroup")
      .def(py::init<>())
      .def("push", &CollectiveGroup::push)
      .def("wait_all", &CollectiveGroup::wait_all, GR())
      .def("__len__", &CollectiveGroup::size);

  // ------------------------------------------------------------ seed / worker
  py::class_<TlsIdentity>(m, "TlsIdentity")
      .def_readonly("ca_cert_pem", &TlsIdentity::ca_cert_pem)
      .def_readonly("cert_pem", &TlsIdentity::cert_pem)
      .def("valid", &TlsIdentity::valid);
  py::class_<ClusterCA, std::shared_ptr<ClusterCA>>(m, "ClusterCA")
      .def_static("generate", &ClusterCA::generate, py::arg("name") = "nexar-cluster-ca")
      .def_static("from_pem", [](const std::string& key, const std::string& cert) { return ClusterCA::from_pem(key, cert); })
      .def("issue", &ClusterCA::issue)
      .def("cert_pem", &ClusterCA::cert_pem)
      .def("key_pem", &ClusterCA::key_pem);
  m.def("tls_identities_check", &tls_identities_check, py::arg("server"), py::arg("client"),
        py::call_guard<py::gil_scoped_release>());
  py::class_<SeedNode, std::shared_ptr<SeedNode>>(m, "SeedNode")
      .def_static("bind", [](const std::string& addr, const py::object& token, bool tls) {
        Bytes t = token.is_none() ? token_from_env() : to_bytes(token.cast<py::bytes>());
        return SeedNode::bind(addr, t, tls);
      }, py::arg("addr"), py::arg("token") = py::none(), py::arg("tls") = false)
      .def_static("bind_local", &SeedNode::bind_local, py::arg("tls") = false)
      .def("tls", &SeedNode::tls)
      .def("local_addr", &SeedNode::local_addr)
      .def("token", [](const SeedNode& s) { return from_bytes(s.token()); })
      .def("with_formation_timeout", [](std::shared_ptr<SeedNode> s, double t) { s->set_formation_timeout(t); return s; })
      .def("use_ca", &SeedNode::use_ca)
      .def("ca", &SeedNode::ca)
      .def("form_cluster", &SeedNode::form_cluster, GR())
      .def("accept_elastic", &SeedNode::accept_elastic)
      .def("close", &SeedNode::close, GR());

  // ------------------------------------------------------------ worker (nexar/src/cluster/worker.rs)
  // WorkerNode.connect binds the mesh listener, joins through the seed and
  // returns what the Welcome carried; NexarClient.from_worker_info then builds
  // the mesh (bootstrap_worker does both in one call).
  py::class_<WorkerInfo, std::shared_ptr<WorkerInfo>>(m, "WorkerInfo")
      .def_property_readonly("rank", [](const WorkerInfo& w) { return w.rank; })
      .def_property_readonly("world_size", [](const WorkerInfo& w) { return w.world_size; })
      .def_property_readonly("peers", [](const WorkerInfo& w) { return w.peers; })
      .def_property_readonly("listen_addr", [](const WorkerInfo& w) { return w.listen_addr; })
      .def_property_readonly("has_certificate", [](const WorkerInfo& w) { return w.tls.valid(); })
      .def_property_readonly("consumed", [](const WorkerInfo& w) { return w.listen_fd < 0; })
      .def("close", [](WorkerInfo& w) {
        if (w.listen_fd >= 0) ::close(w.listen_fd);
        w.listen_fd = -1;
      });
  struct WorkerNodeApi {};
  py::class_<WorkerNodeApi>(m, "WorkerNode")
      .def_static("connect", [](const std::string& seed, const py::object& token, const std::string& host, bool tls) {
        Bytes t = token.is_none() ? token_from_env() : to_bytes(token.cast<py::bytes>());
        py::gil_scoped_release r;
        return std::make_shared<WorkerInfo>(WorkerNode::connect(seed, t, host, tls));
      }, py::arg("seed_addr"), py::arg("token") = py::none(), py::arg("bind_host") = "127.0.0.1",
         py::arg("tls") = false);

  // ------------------------------------------------------------ device adapters
  py::class_<DeviceAdapter, PyDeviceAdapter, std::shared_ptr<DeviceAdapter>>(m, "DeviceAdapter")
      .def(py::init<>())
      .def("name", &DeviceAdapter::name)
      .def("supports_host_offload", &DeviceAdapter::supports_host_offload)
      .def("supports_device_collectives", &DeviceAdapter::supports_device_collectives)
      .def("host_addressable", &DeviceAdapter::host_addressable)
      .def("stage_for_send", [](DeviceAdapter& a, uint64_t ptr, size_t n, uint64_t out) {
        a.stage_for_send(P(ptr), n, static_cast<uint8_t*>(P(out)));
      }, GR())
      .def("receive_to_device", [](DeviceAdapter& a, uint64_t src, size_t n, uint64_t ptr) {
        a.receive_to_device(static_cast<const uint8_t*>(P(src)), n, P(ptr));
      }, GR())
      .def("reduce_inplace", [](DeviceAdapter& a, uint64_t dst, uint64_t src, size_t count, int dt, int op) {
        a.reduce_inplace(P(dst), P(src), count, static_cast<DataType>(dt), static_cast<ReduceOp>(op));
      }, GR());
  py::class_<CpuAdapter, DeviceAdapter, std::shared_ptr<CpuAdapter>>(m, "CpuAdapter").def(py::init<>());
  py::class_<CudaStagingAdapter, DeviceAdapter, std::shared_ptr<CudaStagingAdapter>>(m, "CudaAdapter")
      .def(py::init<>())
      .def_static("runtime_available", &CudaStagingAdapter::runtime_available);

  // ------------------------------------------------------------ client
  py::class_<NexarClient, std::shared_ptr<NexarClient>>(m, "NexarClient")
      .def_static("bootstrap_local", &NexarClient::bootstrap_local, py::arg("world"), py::arg("config"),
                  py::arg("pool") = std::shared_ptr<BufferPool>(), GR())
      .def_static("bootstrap_worker", [](const std::string& seed, const py::object& token, const Config& cfg,
                                         const std::string& host, std::shared_ptr<BufferPool> pool) {
        Bytes t = token.is_none() ? token_from_env() : to_bytes(token.cast<py::bytes>());
        py::gil_scoped_release r;
        return NexarClient::bootstrap_worker(seed, t, cfg, host, std::move(pool));
      }, py::arg("seed_addr"), py::arg("token") = py::none(), py::arg("config") = Config(),
         py::arg("bind_host") = "127.0.0.1", py::arg("pool") = std::shared_ptr<BufferPool>())
      .def_static("from_worker_info", [](std::shared_ptr<WorkerInfo> info, const Config& cfg,
                                         std::shared_ptr<BufferPool> pool) {
        if (!info || info->listen_fd < 0) fail(Err::ConnectionFailed, "worker info already used or closed");
        WorkerInfo w = *info;
        info->listen_fd = -1;  // the mesh owns the listener now
        py::gil_scoped_release r;
        return NexarClient::from_worker_info(std::move(w), cfg, std::move(pool));
      }, py::arg("info"), py::arg("config") = Config(), py::arg("pool") = std::shared_ptr<BufferPool>())
      .def_property_readonly("pool", [](const NexarClient& c) { return c.mesh()->pool(); })
      .def_property_readonly("rank", &NexarClient::rank)
      .def_property_readonly("world_size", &NexarClient::world_size)
      .def_property_readonly("comm_id", &NexarClient::comm_id)
      .def_property_readonly("rank_map", &NexarClient::rank_map)
      .def_property_readonly("mesh_rank_of_self", [](const NexarClient& c) { return c.mesh()->rank(); })
      .def_property_readonly("adapter_name", [](const NexarClient& c) { return c.adapter()->name(); })
      .def("adapter", &NexarClient::adapter)
      .def("set_adapter", &NexarClient::set_adapter)
      .def("has_direct_peer", &NexarClient::has_direct_peer)
      .def("transport_encrypted", [](const NexarClient& c) { return c.mesh()->all_encrypted(); })
      .def("is_sparse", &NexarClient::is_sparse)
      .def("config", &NexarClient::config)
      // p2p
      .def("send", [](NexarClient& c, uint64_t p, size_t n, Rank d, uint32_t t) { c.send(P(p), n, d, t); }, GR())
      .def("recv", [](NexarClient& c, uint64_t p, size_t n, Rank s, uint32_t t) { c.recv(P(p), n, s, t); }, GR())
      .def("send_iov", [](NexarClient& c, const std::vector<std::pair<uint64_t, size_t>>& iov, Rank d, uint32_t t) {
        std::vector<std::pair<const void*, size_t>> v;
        for (auto& e : iov) v.emplace_back(P(e.first), e.second);
        c.send_iov(v, d, t);
      }, GR())
      .def("recv_iov", [](NexarClient& c, const std::vector<std::pair<uint64_t, size_t>>& iov, Rank s, uint32_t t) {
        std::vector<std::pair<void*, size_t>> v;
        for (auto& e : iov) v.emplace_back(P(e.first), e.second);
        c.recv_iov(v, s, t);
      }, GR())
      .def("send_bytes", [](NexarClient& c, Rank d, const py::bytes& b) {
        std::string s = b;
        py::gil_scoped_release r;
        c.send_bytes(d, s.data(), s.size());
      })
      .def("recv_bytes", [](NexarClient& c, Rank s) {
        Bytes b;
        {
          py::gil_scoped_release r;
          b = c.recv_bytes(s);
        }
        return from_bytes(b);
      })
      .def("send_bytes_tagged", [](NexarClient& c, Rank d, uint64_t tag, const py::bytes& b) {
        std::string s = b;
        py::gil_scoped_release r;
        c.send_bytes_tagged(d, tag, s.data(), s.size());
      })
      .def("recv_bytes_tagged", [](NexarClient& c, Rank s, uint64_t tag, double timeout) {
        Bytes b;
        {
          py::gil_scoped_release r;
          b = c.recv_bytes_tagged(s, tag, timeout);
        }
        return from_bytes(b);
      }, py::arg("src"), py::arg("tag"), py::arg("timeout_s") = -1.0)
      // rpc
      .def("register_rpc", [](NexarClient& c, uint16_t fn_id, py::function f) {
        auto fp = std::make_shared<py::function>(std::move(f));
        c.register_rpc(fn_id, [fp](const Bytes& args) -> Bytes {
          py::gil_scoped_acquire g;
          py::object r = (*fp)(from_bytes(args));
          return to_bytes(r.cast<py::bytes>());
        });
      })
      .def("rpc", [](NexarClient& c, Rank t, uint16_t fn, const py::bytes& args, double timeout) {
        Bytes a = to_bytes(args), r;
        {
          py::gil_scoped_release rel;
          r = c.rpc(t, fn, a, timeout);
        }
        return from_bytes(r);
      }, py::arg("target"), py::arg("fn_id"), py::arg("args"), py::arg("timeout_s") = -1.0)
      .def("recv_rpc_request", [](NexarClient& c, Rank s, double timeout) {
        Message m;
        {
          py::gil_scoped_release r;
          m = c.recv_rpc_request(s, timeout);
        }
        return msg_to_dict(m);
      }, py::arg("src"), py::arg("timeout_s") = -1.0)
      .def("serve_rpc_once", [](NexarClient& c, Rank s, double timeout) {
        py::gil_scoped_release r;
        Message m = c.recv_rpc_request(s, timeout);
        c.handle_rpc_request(s, m);
      }, py::arg("src"), py::arg("timeout_s") = -1.0)
      .def("start_rpc_server", &NexarClient::start_rpc_server)
      .def("stop_rpc_server", &NexarClient::stop_rpc_server, GR())
      // collectives
      .def("all_reduce", [](NexarClient& c, uint64_t p, size_t n, int dt, int op) { c.all_reduce(P(p), n, (DataType)dt, (ReduceOp)op); }, GR())
      .def("all_reduce_rs_ag", [](NexarClient& c, uint64_t p, size_t n, int dt, int op) { c.all_reduce_rs_ag(P(p), n, (DataType)dt, (ReduceOp)op); }, GR())
      .def("all_reduce_bucketed", [](NexarClient& c, const std::vector<std::pair<uint64_t, size_t>>& es, int dt, int op) {
        std::vector<std::pair<void*, size_t>> v;
        for (auto& e : es) v.emplace_back(P(e.first), e.second);
        c.all_reduce_bucketed(v, (DataType)dt, (ReduceOp)op);
      }, GR())
      .def("all_reduce_compressed", [](NexarClient& c, uint64_t p, size_t n, int dt, int op, std::shared_ptr<Compressor> comp,
                                       uint64_t residual) {
        c.all_reduce_compressed(P(p), n, (DataType)dt, (ReduceOp)op, *comp, P(residual));
      }, GR())
      .def("broadcast", [](NexarClient& c, uint64_t p, size_t n, int dt, Rank root) { c.broadcast(P(p), n, (DataType)dt, root); }, GR())
      .def("all_gather", [](NexarClient& c, uint64_t s, uint64_t r, size_t n, int dt) { c.all_gather(P(s), P(r), n, (DataType)dt); }, GR())
      .def("reduce_scatter", [](NexarClient& c, uint64_t s, uint64_t r, size_t n, int dt, int op) {
        c.reduce_scatter(P(s), P(r), n, (DataType)dt, (ReduceOp)op);
      }, GR())
      .def("reduce", [](NexarClient& c, uint64_t p, size_t n, int dt, int op, Rank root) { c.reduce(P(p), n, (DataType)dt, (ReduceOp)op, root); }, GR())
      .def("all_to_all", [](NexarClient& c, uint64_t s, uint64_t r, size_t n, int dt) { c.all_to_all(P(s), P(r), n, (DataType)dt); }, GR())
      .def("gather", [](NexarClient& c, uint64_t s, uint64_t r, size_t n, int dt, Rank root) { c.gather(P(s), P(r), n, (DataType)dt, root); }, GR())
      .def("scatter", [](NexarClient& c, uint64_t s, uint64_t r, size_t n, int dt, Rank root) { c.scatter(P(s), P(r), n, (DataType)dt, root); }, GR())
      .def("scan", [](NexarClient& c, uint64_t p, size_t n, int dt, int op) { c.scan(P(p), n, (DataType)dt, (ReduceOp)op); }, GR())
      .def("exclusive_scan", [](NexarClient& c, uint64_t p, size_t n, int dt, int op) { c.exclusive_scan(P(p), n, (DataType)dt, (ReduceOp)op); }, GR())
      .def("barrier", &NexarClient::barrier, GR())
      .def("barrier_with_timeout", &NexarClient::barrier_with_timeout, GR())
      // non-blocking: the tag is taken now, the work runs on a worker thread
      .def("all_reduce_nb", [](std::shared_ptr<NexarClient> c, uint64_t p, size_t n, int dt, int op) {
        const uint64_t tag = c->next_collective_tag();
        return c->spawn([c, p, n, dt, op, tag] { c->all_reduce_tagged(P(p), n, (DataType)dt, (ReduceOp)op, tag); });
      })
      .def("all_reduce_bucketed_nb", [](std::shared_ptr<NexarClient> c, const std::vector<std::pair<uint64_t, size_t>>& es,
                                        int dt, int op) {
        std::vector<std::pair<void*, size_t>> v;
        for (auto& e : es) v.emplace_back(P(e.first), e.second);
        const uint64_t tag = c->next_collective_tag();
        return c->spawn([c, v, dt, op, tag] { c->all_reduce_bucketed_tagged(v, (DataType)dt, (ReduceOp)op, tag); });
      })
      .def("all_reduce_compressed_nb", [](std::shared_ptr<NexarClient> c, uint64_t p, size_t n, int dt, int op,
                                          std::shared_ptr<Compressor> comp, uint64_t residual) {
        const uint64_t tag = c->next_collective_tag();
        return c->spawn([c, p, n, dt, op, comp, residual, tag] {
          c->all_reduce_compressed_tagged(P(p), n, (DataType)dt, (ReduceOp)op, *comp, P(residual), tag);
        });
      })
      .def("peer_info", [](const NexarClient& c, Rank r) {
        // Direct link to communicator rank r (nexar's client.peer(rank)); raises UnknownPeer otherwise.
        if (r >= c.world_size() || !c.has_direct_peer(r))
          fail(Err::UnknownPeer, "unknown peer: rank " + std::to_string(r) + " has no direct connection");
        auto conn = c.mesh()->conn(c.mesh_rank(r));
        py::dict d;
        d["rank"] = r;
        d["mesh_rank"] = c.mesh_rank(r);
        d["alive"] = conn && conn->alive();
        d["encrypted"] = conn && conn->encrypted();
        return d;
      })
      .def("recv_message_from", [](NexarClient& c, Rank src, uint32_t tag, double timeout_s) {
        // The oldest data message with `tag` from `src` on the root
        // communicator (what send_message_to / send deliver).
        const Rank m = c.mesh_rank(src);
        const double t = timeout_s < 0 ? c.config().collective_timeout_s : timeout_s;
        Bytes b;
        {
          py::gil_scoped_release nogil;
          b = std::move(c.mesh()->box(m)->pop_data(tag, Clock::now() + std::chrono::microseconds((int64_t)(t * 1e6))).msg.payload);
        }
        return py::bytes(reinterpret_cast<const char*>(b.data()), b.size());
      }, py::arg("src"), py::arg("tag"), py::arg("timeout_s") = -1.0)
      .def("send_message_to", [](NexarClient& c, Rank dest, uint32_t tag, const py::bytes& payload, int prio) {
        // One framed data message to `dest` (received with recv_message_from(src, tag) or recv).
        const std::string s = payload;
        Message m = Message::data(tag, c.mesh()->rank(), Bytes(s.begin(), s.end()));
        py::gil_scoped_release nogil;
        c.send_message_to(dest, m, (Priority)prio);
      }, py::arg("dest"), py::arg("tag"), py::arg("payload"), py::arg("priority") = 0)
      .def("spawn_collective", [](std::shared_ptr<NexarClient> c, const std::string& op, py::tuple args) {
        // Generic non-blocking launcher for the other collectives. The
        // collective's tag is reserved here (call order), so concurrent
        // non-blocking collectives stay isolated.
        std::vector<uint64_t> a;
        for (auto x : args) a.push_back(x.cast<uint64_t>());
        auto sub = std::shared_ptr<NexarClient>(c);
        const uint64_t tag = c->next_collective_tag();
        auto fn = [sub, op, a, tag]() {
          NexarClient& cl = *sub;
          using namespace coll;
          auto b = [](uint64_t x) { return static_cast<uint8_t*>(P(x)); };
          if (op == "broadcast") broadcast(cl, b(a[0]), a[1] * dtype_size((DataType)a[2]), (Rank)a[3], tag);
          else if (op == "all_gather") ring_allgather(cl, b(a[0]), b(a[1]), a[2], (DataType)a[3], tag);
          else if (op == "reduce_scatter") ring_reduce_scatter(cl, b(a[0]), b(a[1]), a[2], (DataType)a[3], (ReduceOp)a[4], tag);
          else if (op == "reduce") reduce(cl, b(a[0]), a[1], (DataType)a[2], (ReduceOp)a[3], (Rank)a[4], tag);
          else if (op == "all_to_all") alltoall(cl, b(a[0]), b(a[1]), a[2], (DataType)a[3], tag);
          else if (op == "gather") gather(cl, b(a[0]), b(a[1]), a[2], (DataType)a[3], (Rank)a[4], tag);
          else if (op == "scatter") scatter(cl, b(a[0]), b(a[1]), a[2], (DataType)a[3], (Rank)a[4], tag);
          else if (op == "scan") scan(cl, b(a[0]), a[1], (DataType)a[2], (ReduceOp)a[3], false, tag);
          else if (op == "exclusive_scan") scan(cl, b(a[0]), a[1], (DataType)a[2], (ReduceOp)a[3], true, tag);
          else if (op == "all_reduce_rs_ag") rs_ag_allreduce(cl, b(a[0]), a[1], (DataType)a[2], (ReduceOp)a[3], tag);
          else if (op == "barrier") barrier(cl, cl.config().barrier_timeout_s);
          else fail(Err::CollectiveFailed, "unknown collective " + op);
        };
        return c->spawn(fn);
      })
      // communicator management
      .def("split", &NexarClient::split, GR())
      .def("rebuild_excluding", &NexarClient::rebuild_excluding, GR())
      .def("rebuild_adding", &NexarClient::rebuild_adding, py::arg("new_mesh_ranks"), py::arg("comm_id") = 0, GR())
      .def("dead_ranks", &NexarClient::dead_ranks)
      .def("wait_failure", [](NexarClient& c, double timeout) {
        auto mesh = c.mesh();
        uint64_t v = 0;
        {
          py::gil_scoped_release r;
          mesh->wait_failure(mesh->failure_version(), timeout, &v);
        }
        return c.dead_ranks();
      })
      .def("close", &NexarClient::close, GR());

  // ------------------------------------------------------------ recovery / elastic
  py::class_<RecoveryEvent>(m, "RecoveryEvent")
      .def_readonly("old_rank", &RecoveryEvent::old_rank)
      .def_readonly("new_rank", &RecoveryEvent::new_rank)
      .def_readonly("new_world_size", &RecoveryEvent::new_world_size)
      .def_readonly("dead_ranks", &RecoveryEvent::dead_ranks);
  py::class_<EventSubscription<RecoveryEvent>, std::shared_ptr<EventSubscription<RecoveryEvent>>>(
      m, "RecoveryEventReceiver")
      .def("recv", [](EventSubscription<RecoveryEvent>& s, double timeout) -> py::object {
        RecoveryEvent e;
        bool ok;
        {
          py::gil_scoped_release r;
          ok = s.recv(timeout, &e);
        }
        if (!ok) return py::none();
        return py::cast(e);
      }, py::arg("timeout_s") = -1.0)
      .def_property_readonly("pending", &EventSubscription<RecoveryEvent>::pending)
      .def_property_readonly("dropped", &EventSubscription<RecoveryEvent>::dropped);
  py::class_<RecoveryOrchestrator>(m, "RecoveryOrchestrator")
      .def(py::init([](std::shared_ptr<NexarClient> c, int policy) {
        return new RecoveryOrchestrator(c, (RecoveryPolicy)policy);
      }))
      .def_static("from_config", &RecoveryOrchestrator::from_config)
      .def("start", &RecoveryOrchestrator::start)
      .def("run", &RecoveryOrchestrator::run, GR())
      .def("subscribe", &RecoveryOrchestrator::subscribe)
      .def("shutdown", &RecoveryOrchestrator::shutdown, GR())
      .def("recover", &RecoveryOrchestrator::recover, GR())
      .def("client", &RecoveryOrchestrator::client)
      .def("error", &RecoveryOrchestrator::error)
      .def("next_event", [](RecoveryOrchestrator& o, double timeout) -> py::object {
        RecoveryEvent e;
        bool ok;
        {
          py::gil_scoped_release r;
          ok = o.next_event(timeout, &e);
        }
        if (!ok) return py::none();
        return py::cast(e);
      });
  py::class_<ElasticEvent>(m, "ElasticEvent")
      .def_readonly("epoch", &ElasticEvent::epoch)
      .def_readonly("new_rank", &ElasticEvent::new_rank)
      .def_readonly("new_world_size", &ElasticEvent::new_world_size)
      .def_readonly("joined", &ElasticEvent::joined)
      .def_readonly("left", &ElasticEvent::left);
  py::class_<EventSubscription<ElasticEvent>, std::shared_ptr<EventSubscription<ElasticEvent>>>(
      m, "ElasticEventReceiver")
      .def("recv", [](EventSubscription<ElasticEvent>& s, double timeout) -> py::object {
        ElasticEvent e;
        bool ok;
        {
          py::gil_scoped_release r;
          ok = s.recv(timeout, &e);
        }
        if (!ok) return py::none();
        return py::cast(e);
      }, py::arg("timeout_s") = -1.0)
      .def_property_readonly("pending", &EventSubscription<ElasticEvent>::pending)
      .def_property_readonly("dropped", &EventSubscription<ElasticEvent>::dropped);
  py::class_<ElasticManager>(m, "ElasticManager")
      .def(py::init<std::shared_ptr<NexarClient>, std::shared_ptr<SeedNode>, uint32_t, uint32_t, double>(),
           py::arg("client"), py::arg("seed") = nullptr, py::arg("min_world") = 1, py::arg("max_world") = 0,
           py::arg("timeout_s") = 60.0)
      .def("elastic_checkpoint", &ElasticManager::elastic_checkpoint, GR())
      .def("client", &ElasticManager::client)
      .def("remove_node", &ElasticManager::remove_node)
      .def("events", &ElasticManager::events)
      .def("subscribe", &ElasticManager::subscribe)
      .def_property_readonly("epoch", &ElasticManager::epoch)
      .def_static("join", [](const std::string& seed, const py::object& token, const Config& cfg, double timeout) {
        Bytes t = token.is_none() ? Bytes() : to_bytes(token.cast<py::bytes>());
        py::gil_scoped_release r;
        return ElasticManager::join(seed, t, cfg, timeout);
      }, py::arg("seed_addr"), py::arg("token") = py::none(), py::arg("config") = Config(), py::arg("timeout_s") = 60.0);
}
