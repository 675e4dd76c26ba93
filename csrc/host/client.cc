#include "client.h"

#include <algorithm>
#include <thread>

namespace nexar {

namespace {
constexpr uint32_t kMeshMagic = 0x4e584d31;  // "NXM1"
constexpr uint64_t kP2PTagBit = 1ull << 63;   // tag space of p2p send / recv (apart from tagged bytes)
enum RelayLane : uint8_t { kRelayTagged = 0, kRelayControl = 1, kRelayRaw = 2 };

uint64_t token_hash(const Bytes& t) { return t.empty() ? 0 : fnv1a_comm_id({t}); }

void send_handshake(Stream& io, Rank rank, uint32_t world, const Bytes& token) {
  Bytes b;
  put_u32(b, kMeshMagic);
  put_u32(b, rank);
  put_u32(b, world);
  put_u64(b, token_hash(token));
  io.write_all(b.data(), b.size());
}
Rank read_handshake(Stream& io, const Bytes& token) {
  uint8_t b[20];
  if (!io.read_exact(b, sizeof(b))) fail(Err::ConnectionFailed, "mesh handshake: connection closed");
  if ((uint32_t)get_le(b, 4) != kMeshMagic) fail(Err::ConnectionFailed, "mesh handshake: bad magic");
  if (get_le(b + 12, 8) != token_hash(token)) fail(Err::ClusterTokenMismatch, "cluster token mismatch: bootstrap authentication failed");
  return (Rank)get_le(b + 4, 4);
}
Clock::time_point deadline_in(double s) {
  return Clock::now() + std::chrono::microseconds((int64_t)(s * 1e6));
}
}  // namespace

// ============================================================ Mesh
Mesh::Mesh(Rank rank, uint32_t world, Config cfg, Bytes token, std::shared_ptr<BufferPool> pool)
    : rank_(rank), world_(world), cfg_(std::move(cfg)), token_(std::move(token)),
      pool_(pool ? std::move(pool) : BufferPool::with_profile(PoolProfile::Training)) {
  for (Rank r = 0; r < world; ++r) boxes_.push_back(std::make_shared<Mailbox>(r));
}

Mesh::~Mesh() {
  stop_health_monitor();
  std::map<Rank, std::unique_ptr<PeerRouter>> routers;
  {
    std::lock_guard<std::mutex> g(mu_);
    routers.swap(routers_);
  }
  routers.clear();  // joins reader threads
  if (listen_fd >= 0) close_fd(listen_fd);
}

void Mesh::grow(uint32_t new_world) {
  std::lock_guard<std::mutex> g(mu_);
  while (boxes_.size() < new_world) boxes_.push_back(std::make_shared<Mailbox>((Rank)boxes_.size()));
  if (new_world > world_) world_ = new_world;
}

std::shared_ptr<Stream> Mesh::dial(int fd) const {
  return tls() ? tls_client(fd, tls_id_, true, cfg_.collective_timeout_s) : plain_stream(fd);
}

std::shared_ptr<Stream> Mesh::answer(int fd) const {
  return tls() ? tls_server(fd, tls_id_, true, cfg_.collective_timeout_s) : plain_stream(fd);
}

void Mesh::add_connection(Rank r, std::shared_ptr<Stream> io) {
  auto conn = std::make_shared<PeerConnection>(r, std::move(io));
  std::shared_ptr<Mailbox> b;
  {
    std::lock_guard<std::mutex> g(mu_);
    if (r >= boxes_.size()) fail(Err::InvalidRank, "invalid rank " + std::to_string(r) + ": world size is " + std::to_string(boxes_.size()));
    b = boxes_[r];
    conns_[r] = conn;
  }
  std::weak_ptr<Mesh> weak = weak_from_this();
  auto router = std::make_unique<PeerRouter>(
      conn, b,
      [weak](const Message& m) {
        if (auto s = weak.lock()) s->on_relay(m);
      },
      [weak](Rank p) {
        if (auto s = weak.lock()) s->mark_dead(p, "connection lost");
      },
      pool_);
  std::lock_guard<std::mutex> g(mu_);
  routers_[r] = std::move(router);
}

bool Mesh::all_encrypted() const {
  std::lock_guard<std::mutex> g(mu_);
  if (conns_.empty()) return false;
  for (auto& kv : conns_)
    if (!kv.second->encrypted()) return false;
  return true;
}

bool Mesh::has_direct(Rank r) const {
  std::lock_guard<std::mutex> g(mu_);
  return conns_.count(r) != 0;
}

std::shared_ptr<Mailbox> Mesh::box(Rank r) const {
  std::lock_guard<std::mutex> g(mu_);
  if (r >= boxes_.size()) fail(Err::InvalidRank, "invalid rank " + std::to_string(r));
  return boxes_[r];
}

std::shared_ptr<PeerConnection> Mesh::conn(Rank r) const {
  std::lock_guard<std::mutex> g(mu_);
  auto it = conns_.find(r);
  return it == conns_.end() ? nullptr : it->second;
}

void Mesh::set_routing(const TopologyStrategy& t) {
  std::lock_guard<std::mutex> g(mu_);
  topo_ = t;
  sparse_ = t.is_sparse();
  if (sparse_) rt_ = build_routing_table(t, rank_, world_);
}

long long Mesh::next_hop(Rank dest) const {
  std::lock_guard<std::mutex> g(mu_);
  if (conns_.count(dest)) return dest;
  if (!sparse_) return -1;
  return rt_.route(dest);
}

static Bytes relay_payload(uint8_t lane, uint64_t comm, const void* p, size_t n) {
  Bytes b;
  b.reserve(9 + n);
  put_u8(b, lane);
  put_u64(b, comm);
  put_bytes(b, static_cast<const uint8_t*>(p), n);
  return b;
}

void Mesh::send_tagged(Rank dest, uint64_t comm, uint64_t tag, const void* p, size_t n) {
  if (auto c = conn(dest)) {
    c->send_raw_tagged(comm, tag, p, n);
    return;
  }
  const long long hop = next_hop(dest);
  if (hop < 0) fail(Err::UnknownPeer, "rank " + std::to_string(dest) + " not found in cluster");
  Message m = Message::relay(rank_, dest, tag, relay_payload(kRelayTagged, comm, p, n));
  send_message((Rank)hop, m, Priority::Bulk);
}

void Mesh::send_raw(Rank dest, uint64_t comm, const void* p, size_t n) {
  if (auto c = conn(dest)) {
    if (comm == 0) c->send_raw(p, n);
    else c->send_raw_comm(comm, p, n);
    return;
  }
  const long long hop = next_hop(dest);
  if (hop < 0) fail(Err::UnknownPeer, "rank " + std::to_string(dest) + " not found in cluster");
  send_message((Rank)hop, Message::relay(rank_, dest, 0, relay_payload(kRelayRaw, comm, p, n)), Priority::Bulk);
}

void Mesh::send_data(Rank dest, uint32_t tag, const void* p, size_t n) {
  if (auto c = conn(dest)) {
    c->send_data(tag, rank_, p, n, Priority::Bulk);
    return;
  }
  const auto* b = static_cast<const uint8_t*>(p);
  send_message(dest, Message::data(tag, rank_, Bytes(b, b + n)), Priority::Bulk);
}

void Mesh::send_message(Rank dest, const Message& m, Priority prio) {
  if (auto c = conn(dest)) {
    c->send_message(m, prio);
    return;
  }
  const long long hop = next_hop(dest);
  if (hop < 0) fail(Err::UnknownPeer, "rank " + std::to_string(dest) + " not found in cluster");
  Bytes body = encode_body(m);
  Message r = Message::relay(rank_, dest, 0, relay_payload(kRelayControl, 0, body.data(), body.size()));
  auto c = conn((Rank)hop);
  if (!c) fail(Err::UnknownPeer, "no connection to next hop " + std::to_string(hop));
  c->send_message(r, prio);
}

void Mesh::on_relay(const Message& m) {
  if (m.final_dest != rank_) {
    // Forward towards the destination; on failure retry once on the same hop,
    // then try an alternative neighbour (nexar/src/transport/relay.rs:323-376).
    long long hop = next_hop(m.final_dest);
    for (int attempt = 0; attempt < 3 && hop >= 0; ++attempt) {
      auto c = conn((Rank)hop);
      if (c) {
        try {
          c->send_message(m, Priority::Bulk);
          return;
        } catch (const NexarError&) {
        }
      }
      if (attempt >= 1) {
        std::lock_guard<std::mutex> g(mu_);
        hop = find_alternative_hop(topo_, rank_, m.final_dest, (Rank)hop, world_);
      }
    }
    NEXAR_LOG(LogLevel::Warn, "relay: dropping message for rank " + std::to_string(m.final_dest));
    return;
  }
  if (m.payload.size() < 9) return;
  const uint8_t lane = m.payload[0];
  const uint64_t comm = get_le(m.payload.data() + 1, 8);
  Bytes data(m.payload.begin() + 9, m.payload.end());
  auto b = box(m.src_rank);
  if (lane == kRelayTagged) {
    b->push(LaneKey{LaneKind::Tagged, comm, m.relay_tag}, Item{{}, std::move(data)});
  } else if (lane == kRelayRaw) {
    b->push(LaneKey{comm == 0 ? LaneKind::Raw : LaneKind::RawComm, comm, 0}, Item{{}, std::move(data)});
  } else {
    Message inner = decode_body(data.data(), data.size());
    LaneKey k{LaneKind::Control, 0, 0};
    if (inner.kind == MsgKind::Barrier || inner.kind == MsgKind::BarrierAck) k = LaneKey{LaneKind::Barrier, inner.comm_id, 0};
    else if (inner.kind == MsgKind::Data) k = LaneKey{LaneKind::Data, 0, 0};
    else if (inner.kind == MsgKind::Rpc) k = LaneKey{LaneKind::RpcRequest, 0, 0};
    else if (inner.kind == MsgKind::RpcResponse) k = LaneKey{LaneKind::RpcResponse, inner.req_id, 0};
    else if (inner.kind == MsgKind::Heartbeat) return;
    b->push(k, Item{std::move(inner), {}});
  }
}

void Mesh::start_health_monitor() {
  if (health_thr_.joinable()) return;
  health_stop_ = false;
  health_thr_ = std::thread([this] { health_loop(); });
}

void Mesh::stop_health_monitor() {
  health_stop_ = true;
  fcv_.notify_all();
  if (health_thr_.joinable()) health_thr_.join();
}

void Mesh::health_loop() {
  const double interval = std::max(0.01, cfg_.heartbeat_interval_s);
  while (!health_stop_) {
    std::vector<std::pair<Rank, std::shared_ptr<PeerConnection>>> peers;
    {
      std::lock_guard<std::mutex> g(mu_);
      for (auto& kv : conns_) peers.emplace_back(kv.first, kv.second);
    }
    const uint64_t ts = (uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(
                            std::chrono::system_clock::now().time_since_epoch()).count();
    for (auto& pc : peers) {
      {
        std::lock_guard<std::mutex> g(fmu_);
        if (dead_.count(pc.first)) continue;
      }
      try {
        pc.second->send_message(Message::heartbeat(ts), Priority::Critical);
      } catch (const NexarError& e) {
        mark_dead(pc.first, std::string("heartbeat send failed: ") + e.what());
        continue;
      }
      double seen = 0;
      {
        std::lock_guard<std::mutex> g(mu_);
        auto it = routers_.find(pc.first);
        if (it != routers_.end()) seen = it->second->last_seen_s();
      }
      if (seen > cfg_.heartbeat_timeout_s) mark_dead(pc.first, "no traffic for " + std::to_string(seen) + " s");
    }
    std::unique_lock<std::mutex> lk(fmu_);
    fcv_.wait_for(lk, std::chrono::duration<double>(interval), [this] { return health_stop_.load(); });
  }
}

void Mesh::mark_dead(Rank r, const std::string& why) {
  {
    std::lock_guard<std::mutex> g(fmu_);
    if (!dead_.insert(r).second) return;
    ++fversion_;
  }
  NEXAR_LOG(closed_ ? LogLevel::Debug : LogLevel::Info,
            "rank " + std::to_string(rank_) + ": peer " + std::to_string(r) + " marked dead (" + why + ")");
  if (auto b = box(r)) b->close(Err::PeerDisconnected, "peer " + std::to_string(r) + " disconnected unexpectedly");
  fcv_.notify_all();
}

std::vector<Rank> Mesh::dead_ranks() const {
  std::lock_guard<std::mutex> g(fmu_);
  return std::vector<Rank>(dead_.begin(), dead_.end());
}

uint64_t Mesh::failure_version() const {
  std::lock_guard<std::mutex> g(fmu_);
  return fversion_;
}

std::vector<Rank> Mesh::wait_failure(uint64_t seen, double timeout_s, uint64_t* version_out) {
  std::unique_lock<std::mutex> lk(fmu_);
  fcv_.wait_for(lk, std::chrono::duration<double>(timeout_s), [&] { return fversion_ != seen || health_stop_.load(); });
  if (version_out) *version_out = fversion_;
  return std::vector<Rank>(dead_.begin(), dead_.end());
}

void Mesh::close() {
  closed_ = true;
  std::vector<std::shared_ptr<PeerConnection>> cs;
  {
    std::lock_guard<std::mutex> g(mu_);
    for (auto& kv : conns_) cs.push_back(kv.second);
  }
  for (auto& c : cs) c->close();
  health_stop_ = true;
  fcv_.notify_all();
}

// ============================================================ handles
void CollectiveGroup::wait_all() {
  std::exception_ptr first;
  for (auto& h : hs_) {
    try {
      h.wait();
    } catch (...) {
      if (!first) first = std::current_exception();
    }
  }
  if (first) std::rethrow_exception(first);
}

// ============================================================ client
NexarClient::NexarClient(std::shared_ptr<Mesh> mesh, Rank rank, uint32_t world, uint64_t comm_id,
                         std::vector<Rank> rank_map, std::shared_ptr<DeviceAdapter> adapter)
    : mesh_(std::move(mesh)), rank_(rank), world_(world), comm_id_(comm_id), rank_map_(std::move(rank_map)),
      adapter_(adapter ? std::move(adapter) : std::make_shared<CpuAdapter>()),
      rpc_mu_(std::make_shared<std::mutex>()),
      rpc_registry_(std::make_shared<std::map<uint16_t, RpcHandler>>()) {}

Rank NexarClient::mesh_rank(Rank r) const {
  if (r >= world_) fail(Err::InvalidRank, "invalid rank " + std::to_string(r) + ": world size is " + std::to_string(world_));
  return rank_map_[r];
}

std::shared_ptr<NexarClient> NexarClient::from_worker_info(WorkerInfo info, const Config& cfg,
                                                          std::shared_ptr<BufferPool> pool) {
  auto mesh = std::make_shared<Mesh>(info.rank, info.world_size, cfg, info.token, std::move(pool));
  mesh->listen_fd = info.listen_fd;
  mesh->listen_addr = info.listen_addr;
  if (cfg.tls) {
    if (!info.tls.valid()) fail(Err::ConnectionFailed, "TLS is on but the seed issued no certificate (seed without TLS?)");
    mesh->set_tls(info.tls);
  }
  std::map<Rank, std::string> addr;
  for (auto& p : info.peers) addr[p.first] = p.second;
  const auto nbrs = build_neighbors(cfg.topology, info.rank, info.world_size);
  size_t expect_accept = 0;
  for (Rank p : nbrs) {
    if (p < info.rank) {
      auto hp = split_host_port(addr.at(p));
      auto io = mesh->dial(tcp_connect(hp.first, hp.second, 30.0));
      send_handshake(*io, info.rank, info.world_size, info.token);
      mesh->add_connection(p, io);
    } else {
      ++expect_accept;
    }
  }
  const auto t0 = Clock::now();
  while (expect_accept > 0) {
    if (seconds_since(t0) > 60.0) fail(Err::ClusterFormationTimeout, "mesh formation timed out");
    int fd = tcp_accept(info.listen_fd, 0.5);
    if (fd < 0) continue;
    Rank p;
    std::shared_ptr<Stream> io;
    try {
      io = mesh->answer(fd);  // owns fd from here on, also when it throws
      p = read_handshake(*io, info.token);
    } catch (const NexarError& e) {
      NEXAR_LOG(LogLevel::Warn, std::string("rejected mesh connection: ") + e.what());
      continue;
    }
    if (!nbrs.count(p) || p <= info.rank || mesh->has_direct(p)) continue;
    mesh->add_connection(p, io);
    --expect_accept;
  }
  mesh->set_routing(cfg.topology);
  mesh->start_health_monitor();
  std::vector<Rank> rm(info.world_size);
  for (Rank r = 0; r < info.world_size; ++r) rm[r] = r;
  return std::make_shared<NexarClient>(mesh, info.rank, info.world_size, 0, rm, nullptr);
}

std::vector<std::shared_ptr<NexarClient>> NexarClient::bootstrap_local(uint32_t world, const Config& cfg,
                                                                       std::shared_ptr<BufferPool> pool) {
  if (world == 0) fail(Err::InvalidRank, "world size must be >= 1");
  auto seed = SeedNode::bind_local(cfg.tls);
  std::vector<WorkerInfo> infos(world);
  std::vector<std::exception_ptr> errs(world + 1);
  std::thread seed_thr([&] {
    try {
      seed->form_cluster(world);
    } catch (...) {
      errs[world] = std::current_exception();
    }
  });
  std::vector<std::thread> ts;
  for (uint32_t i = 0; i < world; ++i) {
    ts.emplace_back([&, i] {
      try {
        infos[i] = WorkerNode::connect(seed->local_addr(), {}, "127.0.0.1", cfg.tls);
      } catch (...) {
        errs[i] = std::current_exception();
      }
    });
  }
  for (auto& t : ts) t.join();
  seed_thr.join();
  for (auto& e : errs)
    if (e) std::rethrow_exception(e);
  std::vector<std::shared_ptr<NexarClient>> clients(world);
  ts.clear();
  std::fill(errs.begin(), errs.end(), nullptr);
  for (uint32_t i = 0; i < world; ++i) {
    ts.emplace_back([&, i] {
      try {
        clients[infos[i].rank] = from_worker_info(infos[i], cfg, pool);
      } catch (...) {
        errs[i] = std::current_exception();
      }
    });
  }
  for (auto& t : ts) t.join();
  for (auto& e : errs)
    if (e) std::rethrow_exception(e);
  return clients;
}

std::shared_ptr<NexarClient> NexarClient::bootstrap_worker(const std::string& seed_addr, const Bytes& token,
                                                          const Config& cfg, const std::string& bind_host,
                                                          std::shared_ptr<BufferPool> pool) {
  WorkerInfo info = WorkerNode::connect(seed_addr, token, bind_host, cfg.tls);
  return from_worker_info(std::move(info), cfg, std::move(pool));
}

// ------------------------------------------------------------ p2p
void NexarClient::set_adapter(std::shared_ptr<DeviceAdapter> a) {
  adapter_ = a ? std::move(a) : std::make_shared<CpuAdapter>();
}

// Point to point moves the buffer through the adapter: staged to the host
// before sending, written back after receiving (nexar/src/client/async_client.rs:312-379).
// On the root communicator a message is a Data message (tag, source rank,
// payload), as the reference sends it, so send pairs with recv_message_from and
// send_message_to with recv; the payload is written straight from the caller's
// buffer and read straight into its own buffer (no encode / decode copies). A
// receive takes the oldest Data message with its tag (the reference takes the
// next one and fails on a tag mismatch). On a split / rebuilt communicator the
// message travels as a tagged frame keyed by the communicator id, so
// communicators that share links never see each other's messages (the
// reference's Data message has no communicator id).
void NexarClient::p2p_send(const void* ptr, size_t size, Rank dest, uint32_t tag) {
  const Rank m = mesh_rank(dest);
  if (comm_id_ == 0) mesh_->send_data(m, tag, ptr, size);
  else mesh_->send_tagged(m, comm_id_, kP2PTagBit | tag, ptr, size);
}

void NexarClient::send(const void* ptr, size_t size, Rank dest, uint32_t tag) {
  if (adapter_->host_addressable()) {
    p2p_send(ptr, size, dest, tag);
    return;
  }
  Bytes staged(size);
  adapter_->stage_for_send(ptr, size, staged.data());
  p2p_send(staged.data(), size, dest, tag);
}

Bytes NexarClient::recv_p2p(Rank src, uint32_t tag) {
  const Rank m = mesh_rank(src);
  auto dl = deadline_in(collective_timeout());
  if (comm_id_ == 0) return std::move(mesh_->box(m)->pop_data(tag, dl).msg.payload);
  return std::move(mesh_->box(m)->pop(LaneKey{LaneKind::Tagged, comm_id_, kP2PTagBit | tag}, dl).bytes);
}

void NexarClient::recv(void* ptr, size_t size, Rank src, uint32_t tag) {
  Bytes payload = recv_p2p(src, tag);
  if (payload.size() != size)
    fail(Err::BufferSizeMismatch, "buffer size mismatch: expected " + std::to_string(size) + " bytes, got " + std::to_string(payload.size()));
  if (adapter_->host_addressable()) std::memcpy(ptr, payload.data(), size);
  else adapter_->receive_to_device(payload.data(), size, ptr);
}

void NexarClient::send_iov(const std::vector<std::pair<const void*, size_t>>& iov, Rank dest, uint32_t tag) {
  size_t total = 0;
  for (auto& e : iov) total += e.second;
  Bytes b(total);
  adapter_->stage_for_send_iov(iov, b.data());
  p2p_send(b.data(), b.size(), dest, tag);
}

void NexarClient::recv_iov(const std::vector<std::pair<void*, size_t>>& iov, Rank src, uint32_t tag) {
  size_t total = 0;
  for (auto& e : iov) total += e.second;
  Bytes payload = recv_p2p(src, tag);
  if (payload.size() != total)
    fail(Err::BufferSizeMismatch, "buffer size mismatch: expected " + std::to_string(total) + " bytes, got " + std::to_string(payload.size()));
  adapter_->receive_to_device_iov(payload.data(), iov);
}

void NexarClient::send_bytes(Rank dest, const void* p, size_t n) { mesh_->send_raw(mesh_rank(dest), comm_id_, p, n); }

Bytes NexarClient::recv_bytes(Rank src) {
  LaneKey k = comm_id_ == 0 ? LaneKey{LaneKind::Raw, 0, 0} : LaneKey{LaneKind::RawComm, comm_id_, 0};
  return std::move(mesh_->box(mesh_rank(src))->pop(k, deadline_in(collective_timeout())).bytes);
}

void NexarClient::send_bytes_tagged(Rank dest, uint64_t tag, const void* p, size_t n) {
  mesh_->send_tagged(mesh_rank(dest), comm_id_, tag, p, n);
}

Bytes NexarClient::recv_bytes_tagged(Rank src, uint64_t tag, double timeout_s) {
  const double t = timeout_s < 0 ? collective_timeout() : timeout_s;
  return std::move(mesh_->box(mesh_rank(src))->pop(LaneKey{LaneKind::Tagged, comm_id_, tag}, deadline_in(t)).bytes);
}

void NexarClient::send_message_to(Rank dest, const Message& m, Priority prio) {
  mesh_->send_message(mesh_rank(dest), m, prio);
}

Message NexarClient::recv_control_from(Rank src, double timeout_s) {
  return std::move(mesh_->box(mesh_rank(src))->pop(LaneKey{LaneKind::Control, 0, 0}, deadline_in(timeout_s)).msg);
}

void NexarClient::coll_send(Rank dest, uint64_t tag, const void* p, size_t n, const char* op) {
  try {
    send_bytes_tagged(dest, tag, p, n);
  } catch (const NexarError& e) {
    throw collective_failed(op, dest, e.what());
  }
}

Bytes NexarClient::coll_recv(Rank src, uint64_t tag, const char* op) {
  try {
    return recv_bytes_tagged(src, tag);
  } catch (const NexarError& e) {
    throw collective_failed(op, src, e.what());
  }
}

// ------------------------------------------------------------ rpc
void NexarClient::register_rpc(uint16_t fn_id, RpcHandler h) {
  std::lock_guard<std::mutex> g(*rpc_mu_);
  (*rpc_registry_)[fn_id] = std::move(h);
}

Bytes NexarClient::rpc(Rank target, uint16_t fn_id, const Bytes& args, double timeout_s) {
  const double t = timeout_s < 0 ? config().rpc_timeout_s : timeout_s;
  const uint64_t id = (rpc_req_id_.fetch_add(1) << 8) | (mesh_->rank() & 0xff);
  try {
    send_message_to(target, Message::rpc(id, fn_id, args), Priority::Realtime);
  } catch (const NexarError& e) {
    fail(Err::RpcFailed, "RPC call to rank " + std::to_string(target) + " failed: " + e.what());
  }
  Message resp;
  try {
    resp = std::move(mesh_->box(mesh_rank(target))->pop(LaneKey{LaneKind::RpcResponse, id, 0}, deadline_in(t)).msg);
  } catch (const NexarError& e) {
    fail(Err::RpcFailed, "RPC call to rank " + std::to_string(target) + " failed: " + e.what());
  }
  // Response body: [status u8][payload]. status 1 = handler missing, 2 = handler error.
  if (resp.payload.empty()) fail(Err::RpcFailed, "RPC call to rank " + std::to_string(target) + " failed: empty response");
  const uint8_t st = resp.payload[0];
  Bytes body(resp.payload.begin() + 1, resp.payload.end());
  if (st == 1) fail(Err::RpcNotRegistered, "RPC handler not registered for fn_id=" + std::to_string(fn_id));
  if (st != 0)
    fail(Err::RpcFailed, "RPC call to rank " + std::to_string(target) + " failed: " + std::string(body.begin(), body.end()));
  return body;
}

Message NexarClient::recv_rpc_request(Rank src, double timeout_s) {
  const double t = timeout_s < 0 ? config().rpc_timeout_s : timeout_s;
  return std::move(mesh_->box(mesh_rank(src))->pop(LaneKey{LaneKind::RpcRequest, 0, 0}, deadline_in(t)).msg);
}

void NexarClient::handle_rpc_request(Rank src, const Message& req) {
  RpcHandler h;
  {
    std::lock_guard<std::mutex> g(*rpc_mu_);
    auto it = rpc_registry_->find(req.fn_id);
    if (it != rpc_registry_->end()) h = it->second;
  }
  Bytes out;
  if (!h) {
    out.push_back(1);
  } else {
    try {
      Bytes r = h(req.payload);
      out.push_back(0);
      out.insert(out.end(), r.begin(), r.end());
    } catch (const std::exception& e) {
      out.push_back(2);
      std::string w = e.what();
      out.insert(out.end(), w.begin(), w.end());
    }
  }
  send_message_to(src, Message::rpc_response(req.req_id, std::move(out)), Priority::Realtime);
}

void NexarClient::start_rpc_server() {
  if (rpc_thr_.joinable()) return;
  rpc_stop_ = false;
  std::weak_ptr<NexarClient> weak = weak_from_this();
  rpc_thr_ = std::thread([weak, this] {
    while (!rpc_stop_) {
      auto self = weak.lock();
      if (!self) return;
      bool any = false;
      for (Rank r = 0; r < world_ && !rpc_stop_; ++r) {
        if (r == rank_) continue;
        try {
          Message m = recv_rpc_request(r, 0.0);
          any = true;
          handle_rpc_request(r, m);
        } catch (const NexarError&) {
        }
      }
      if (!any) std::this_thread::sleep_for(std::chrono::microseconds(200));
    }
  });
}

void NexarClient::stop_rpc_server() {
  rpc_stop_ = true;
  if (rpc_thr_.joinable()) rpc_thr_.join();
}

// ------------------------------------------------------------ non-blocking
CollectiveHandle NexarClient::spawn(std::function<void()> fn) {
  auto self = shared_from_this();
  std::packaged_task<void()> task([self, fn = std::move(fn)] { fn(); });
  std::shared_future<void> f = task.get_future().share();
  std::thread(std::move(task)).detach();
  return CollectiveHandle(f);
}

// ------------------------------------------------------------ communicator management
std::shared_ptr<NexarClient> NexarClient::split(uint32_t color, uint32_t key) {
  // All ranks exchange [color u32][key u32][generation u64] (16 bytes) with a
  // ring all-gather, then group by color and order by (key, rank)
  // (nexar/src/client/split.rs:26-182).
  const uint64_t gen = split_generation_.load();
  uint8_t mine[16];
  for (int i = 0; i < 4; ++i) mine[i] = (color >> (8 * i)) & 0xff;
  for (int i = 0; i < 4; ++i) mine[4 + i] = (key >> (8 * i)) & 0xff;
  for (int i = 0; i < 8; ++i) mine[8 + i] = (gen >> (8 * i)) & 0xff;
  Bytes all(16 * world_);
  coll::ring_allgather(*this, mine, all.data(), 16, DataType::U8, next_collective_tag());
  std::vector<std::pair<uint32_t, Rank>> group;  // (key, rank)
  for (Rank r = 0; r < world_; ++r) {
    const uint8_t* e = all.data() + 16 * r;
    const uint32_t c = (uint32_t)get_le(e, 4), k = (uint32_t)get_le(e + 4, 4);
    const uint64_t g = get_le(e + 8, 8);
    if (g != gen)
      throw collective_failed("split", r, "split_generation mismatch: local=" + std::to_string(gen) + ", rank " +
                                              std::to_string(r) + "=" + std::to_string(g));
    if (c == color) group.emplace_back(k, r);
  }
  std::sort(group.begin(), group.end());
  split_generation_.fetch_add(1);
  Bytes p1, p2, p3;
  put_u64(p1, comm_id_);
  put_u64(p2, gen);
  put_u32(p3, color);
  const uint64_t cid = fnv1a_comm_id({p1, p2, p3});
  std::vector<Rank> rm;
  Rank me = 0;
  for (size_t i = 0; i < group.size(); ++i) {
    if (group[i].second == rank_) me = (Rank)i;
    rm.push_back(rank_map_[group[i].second]);
  }
  auto c = std::make_shared<NexarClient>(mesh_, me, (uint32_t)rm.size(), cid, rm, adapter_);
  c->rpc_mu_ = rpc_mu_;
  c->rpc_registry_ = rpc_registry_;
  return c;
}

std::shared_ptr<NexarClient> NexarClient::rebuild_excluding(const std::vector<Rank>& dead_in) {
  // Local, deterministic renumbering of the survivors; comm_id from the
  // parent's id, the rebuild generation and the sorted dead set
  // (nexar/src/client/rebuild.rs:29-121).
  std::vector<Rank> dead(dead_in.begin(), dead_in.end());
  std::sort(dead.begin(), dead.end());
  dead.erase(std::unique(dead.begin(), dead.end()), dead.end());
  if (std::binary_search(dead.begin(), dead.end(), rank_))
    fail(Err::Recovery, "recovery failed: this rank is in the dead set");
  std::vector<Rank> rm;
  Rank me = 0;
  for (Rank r = 0; r < world_; ++r) {
    if (std::binary_search(dead.begin(), dead.end(), r)) continue;
    if (r == rank_) me = (Rank)rm.size();
    rm.push_back(rank_map_[r]);
  }
  const uint64_t gen = rebuild_generation_.fetch_add(1);
  Bytes p1, p2, p3;
  put_u64(p1, comm_id_);
  put_u64(p2, gen);
  for (Rank d : dead) put_u32(p3, d);
  const uint64_t cid = fnv1a_comm_id({p1, p2, p3});
  auto c = std::make_shared<NexarClient>(mesh_, me, (uint32_t)rm.size(), cid, rm, adapter_);
  c->rpc_mu_ = rpc_mu_;
  c->rpc_registry_ = rpc_registry_;
  return c;
}

std::shared_ptr<NexarClient> NexarClient::rebuild_adding(const std::vector<Rank>& new_mesh_ranks, uint64_t comm_id) {
  std::vector<Rank> rm = rank_map_;
  for (Rank m : new_mesh_ranks) {
    if (m != mesh_->rank() && !mesh_->has_direct(m) && !mesh_->sparse())
      fail(Err::Elastic, "elastic scaling error: no connection to new rank " + std::to_string(m));
    rm.push_back(m);
  }
  const uint64_t gen = rebuild_generation_.fetch_add(1);
  Bytes p1, p2, p3;
  put_u64(p1, comm_id_);
  put_u64(p2, gen | (1ull << 62));
  for (Rank m : new_mesh_ranks) put_u32(p3, m);
  const uint64_t cid = comm_id ? comm_id : fnv1a_comm_id({p1, p2, p3});
  Rank me = 0;
  for (size_t i = 0; i < rm.size(); ++i)
    if (rm[i] == mesh_->rank()) me = (Rank)i;
  auto c = std::make_shared<NexarClient>(mesh_, me, (uint32_t)rm.size(), cid, rm, adapter_);
  c->rpc_mu_ = rpc_mu_;
  c->rpc_registry_ = rpc_registry_;
  return c;
}

std::vector<Rank> NexarClient::dead_ranks() const {
  std::vector<Rank> out;
  for (Rank m : mesh_->dead_ranks())
    for (Rank r = 0; r < world_; ++r)
      if (rank_map_[r] == m) out.push_back(r);
  std::sort(out.begin(), out.end());
  return out;
}

}  // namespace nexar
