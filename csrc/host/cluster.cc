#include "cluster.h"

#include <algorithm>
#include <deque>
#include <random>
#include <unistd.h>

namespace nexar {

// ------------------------------------------------------------------ topology
static uint32_t ring_distance(Rank a, Rank b, uint32_t world) {
  const uint32_t cw = (b + world - a) % world;
  const uint32_t ccw = (a + world - b) % world;
  return std::min(cw, ccw);
}

std::set<Rank> build_neighbors(const TopologyStrategy& s, Rank rank, uint32_t world) {
  std::set<Rank> n;
  switch (s.kind) {
    case TopologyKind::FullMesh:
      for (Rank r = 0; r < world; ++r)
        if (r != rank) n.insert(r);
      break;
    case TopologyKind::KRegular: {
      const uint32_t half = s.degree / 2;
      for (uint32_t d = 1; d <= half; ++d) {
        n.insert((rank + d) % world);
        n.insert((rank + world - d) % world);
      }
      n.erase(rank);
      break;
    }
    case TopologyKind::Hypercube: {
      if (world == 0 || (world & (world - 1)) != 0)
        fail(Err::Elastic, "Hypercube requires a power-of-2 world size, got " + std::to_string(world));
      for (uint32_t b = 0; (1u << b) < world; ++b) n.insert(rank ^ (1u << b));
      break;
    }
  }
  return n;
}

long long RoutingTable::route(Rank dest) const {
  if (neighbors.count(dest)) return dest;
  auto it = next_hop.find(dest);
  return it == next_hop.end() ? -1 : (long long)it->second;
}

RoutingTable build_routing_table(const TopologyStrategy& s, Rank rank, uint32_t world) {
  RoutingTable rt;
  rt.neighbors = build_neighbors(s, rank, world);
  if (s.kind == TopologyKind::FullMesh) return rt;
  for (Rank dest = 0; dest < world; ++dest) {
    if (dest == rank || rt.neighbors.count(dest)) continue;
    Rank hop = 0;
    if (s.kind == TopologyKind::KRegular) {
      uint32_t best = UINT32_MAX;
      for (Rank n : rt.neighbors) {  // ascending: ties go to the lower rank
        const uint32_t d = ring_distance(n, dest, world);
        if (d < best) {
          best = d;
          hop = n;
        }
      }
    } else {
      const uint32_t diff = rank ^ dest;
      const uint32_t hb = 31 - __builtin_clz(diff);
      hop = rank ^ (1u << hb);
    }
    rt.next_hop[dest] = hop;
  }
  return rt;
}

SpanningTree build_spanning_tree(const TopologyStrategy& s, Rank root, uint32_t world) {
  SpanningTree t;
  std::set<Rank> visited{root};
  std::deque<Rank> q{root};
  t.children[root] = {};
  while (!q.empty()) {
    const Rank node = q.front();
    q.pop_front();
    std::vector<Rank> kids;
    for (Rank n : build_neighbors(s, node, world))
      if (visited.insert(n).second) kids.push_back(n);
    std::sort(kids.begin(), kids.end());
    for (Rank c : kids) {
      t.parent[c] = node;
      t.children[c] = {};
      q.push_back(c);
    }
    auto& ch = t.children[node];
    ch.insert(ch.end(), kids.begin(), kids.end());
  }
  return t;
}

long long find_alternative_hop(const TopologyStrategy& s, Rank rank, Rank dest, Rank failed_hop, uint32_t world) {
  std::vector<Rank> cand;
  for (Rank n : build_neighbors(s, rank, world))
    if (n != failed_hop) cand.push_back(n);
  if (cand.empty()) return -1;
  long long best = -1;
  uint32_t best_d = UINT32_MAX;
  for (Rank n : cand) {
    uint32_t d = s.kind == TopologyKind::Hypercube ? (uint32_t)__builtin_popcount(n ^ dest)
                                                   : ring_distance(n, dest, world);
    if (n == dest) d = 0;
    if (d < best_d) {
      best_d = d;
      best = n;
    }
  }
  return best;
}

std::vector<Rank> optimal_ring_order(uint32_t world) {
  std::vector<Rank> v(world);
  for (Rank r = 0; r < world; ++r) v[r] = r;
  return v;
}

// ------------------------------------------------------------------ cluster map
void ClusterMap::add_peer(Rank r, const std::string& addr) {
  std::lock_guard<std::mutex> g(mu_);
  peers_[r] = PeerInfo{addr, 0, true};
  ++epoch_;
}
void ClusterMap::remove_peer(Rank r) {
  std::lock_guard<std::mutex> g(mu_);
  if (peers_.erase(r)) ++epoch_;
}
void ClusterMap::heartbeat(Rank r, double now_s) {
  std::lock_guard<std::mutex> g(mu_);
  auto it = peers_.find(r);
  if (it != peers_.end()) it->second.last_heartbeat_s = now_s;
}
std::vector<Rank> ClusterMap::alive_peers() const {
  std::lock_guard<std::mutex> g(mu_);
  std::vector<Rank> v;
  for (auto& kv : peers_)
    if (kv.second.alive) v.push_back(kv.first);
  return v;
}
std::vector<Rank> ClusterMap::check_timeouts(double now_s, double timeout_s) {
  std::lock_guard<std::mutex> g(mu_);
  std::vector<Rank> dead;
  for (auto& kv : peers_) {
    if (kv.second.alive && now_s - kv.second.last_heartbeat_s > timeout_s) {
      kv.second.alive = false;
      dead.push_back(kv.first);
    }
  }
  if (!dead.empty()) ++epoch_;
  return dead;
}
size_t ClusterMap::size() const {
  std::lock_guard<std::mutex> g(mu_);
  return peers_.size();
}
bool ClusterMap::contains(Rank r) const {
  std::lock_guard<std::mutex> g(mu_);
  return peers_.count(r) != 0;
}
std::string ClusterMap::addr(Rank r) const {
  std::lock_guard<std::mutex> g(mu_);
  auto it = peers_.find(r);
  return it == peers_.end() ? std::string() : it->second.addr;
}

// ------------------------------------------------------------------ tokens
Bytes random_token(size_t n) {
  std::random_device rd;
  Bytes t(n);
  for (auto& b : t) b = (uint8_t)rd();
  return t;
}

Bytes token_from_env() {
  const char* v = std::getenv("NEXAR_CLUSTER_TOKEN");
  if (!v || !*v) return {};
  return Bytes(v, v + std::strlen(v));
}

static std::string hex(const Bytes& b) {
  static const char* d = "0123456789abcdef";
  std::string s;
  for (uint8_t x : b) {
    s.push_back(d[x >> 4]);
    s.push_back(d[x & 15]);
  }
  return s;
}

// ------------------------------------------------------------------ seed
namespace {
constexpr double kTlsHandshakeTimeoutS = 10.0;
}

void SeedNode::use_ca(std::shared_ptr<ClusterCA> ca) {
  if (!ca_) fail(Err::Tls, "use_ca: the seed was bound without TLS");
  if (!ca) fail(Err::Tls, "use_ca: no CA");
  ca_ = std::move(ca);
  seed_id_ = ca_->issue("nexar-seed");
}

std::shared_ptr<Stream> SeedNode::accept_bootstrap(int fd) {
  if (!ca_) return plain_stream(fd);
  // Workers do not verify the seed (they hold no CA yet): the cluster token
  // in their Hello authenticates them, TLS keeps the token and the issued
  // key private (nexar/src/transport/tls.rs:179-298).
  return tls_server(fd, seed_id_, false, kTlsHandshakeTimeoutS);
}

std::shared_ptr<SeedNode> SeedNode::bind(const std::string& addr, const Bytes& token, bool tls) {
  auto hp = split_host_port(addr);
  std::shared_ptr<SeedNode> s(new SeedNode());
  if (tls) {
    s->ca_ = ClusterCA::generate();
    s->seed_id_ = s->ca_->issue("nexar-seed");
  }
  int port = 0;
  s->listen_fd_ = tcp_listen(hp.first, hp.second, &port);
  s->addr_ = hp.first + ":" + std::to_string(port);
  s->token_ = token;
  if (s->token_.empty()) {
    // No token given: generate one and log it (nexar/src/cluster/seed.rs:65-108).
    s->token_ = random_token();
    NEXAR_LOG(LogLevel::Warn, "NEXAR_CLUSTER_TOKEN not set; generated cluster token " + hex(s->token_));
  }
  return s;
}

std::shared_ptr<SeedNode> SeedNode::bind_local(bool tls) {
  std::shared_ptr<SeedNode> s(new SeedNode());
  if (tls) {
    s->ca_ = ClusterCA::generate();
    s->seed_id_ = s->ca_->issue("nexar-seed");
  }
  int port = 0;
  s->listen_fd_ = tcp_listen("127.0.0.1", 0, &port);
  s->addr_ = "127.0.0.1:" + std::to_string(port);
  return s;  // empty token: local mode, no authentication
}

SeedNode::~SeedNode() { close(); }

void SeedNode::close() {
  stop_ = true;
  if (listen_fd_ >= 0) {
    close_fd(listen_fd_);
    listen_fd_ = -1;
  }
  if (elastic_thr_.joinable()) elastic_thr_.join();
  std::lock_guard<std::mutex> g(mu_);
  pending_.clear();  // drops (closes) the bootstrap streams
}

PeerList SeedNode::form_cluster(uint32_t world) {
  const auto t0 = Clock::now();
  std::vector<std::shared_ptr<Stream>> ios;
  PeerList table;
  while (table.size() < world) {
    const double left = formation_timeout_s_ - seconds_since(t0);
    if (left <= 0) {
      fail(Err::ClusterFormationTimeout, "cluster formation timed out: " + std::to_string(table.size()) + "/" +
                                             std::to_string(world) + " nodes joined");
    }
    int fd = tcp_accept(listen_fd_, std::min(left, 0.5));
    if (fd < 0) continue;
    try {
      auto io = accept_bootstrap(fd);
      Message h = read_framed(*io);
      if (h.kind != MsgKind::Hello) fail(Err::DecodeFailed, "expected Hello");
      if (h.protocol_version != kProtocolVersion) {
        NEXAR_LOG(LogLevel::Warn, "rejecting worker with protocol version " + std::to_string(h.protocol_version));
        continue;
      }
      if (!token_.empty() && h.cluster_token != token_) {
        NEXAR_LOG(LogLevel::Warn, "rejecting worker: cluster token mismatch");
        continue;
      }
      table.emplace_back((Rank)table.size(), h.listen_addr);
      ios.push_back(io);
    } catch (const NexarError& e) {
      NEXAR_LOG(LogLevel::Warn, std::string("bad bootstrap connection: ") + e.what());
    }
  }
  for (uint32_t r = 0; r < world; ++r) {
    write_framed(*ios[r], Message::welcome(r, world, table));
    if (ca_) send_identity(*ios[r], ca_->issue("nexar-rank-" + std::to_string(r)));
  }
  ios.clear();
  table_ = table;
  next_rank_ = world;
  return table;
}

void SeedNode::accept_elastic(uint32_t max_world) {
  if (elastic_thr_.joinable()) return;
  elastic_thr_ = std::thread([this, max_world] {
    while (!stop_) {
      int fd = tcp_accept(listen_fd_, 0.2);
      if (fd < 0) continue;
      try {
        auto io = accept_bootstrap(fd);
        Message h = read_framed(*io);
        if (h.kind != MsgKind::Hello || h.protocol_version != kProtocolVersion ||
            (!token_.empty() && h.cluster_token != token_)) {
          continue;
        }
        std::lock_guard<std::mutex> g(mu_);
        if (max_world && next_rank_ >= max_world) continue;
        const Rank r = next_rank_++;
        PeerList table = table_;
        table.emplace_back(r, h.listen_addr);
        table_ = table;
        write_framed(*io, Message::welcome(r, (uint32_t)table.size(), table));
        if (ca_) send_identity(*io, ca_->issue("nexar-rank-" + std::to_string(r)));
        pending_.push_back(PendingJoin{r, h.listen_addr, io});
      } catch (const NexarError&) {
      }
    }
  });
}

std::vector<PendingJoin> SeedNode::take_pending_joins() {
  std::lock_guard<std::mutex> g(mu_);
  auto v = std::move(pending_);
  pending_.clear();
  return v;
}

// ------------------------------------------------------------------ worker
WorkerInfo WorkerNode::connect(const std::string& seed_addr, const Bytes& token, const std::string& bind_host,
                               bool tls) {
  WorkerInfo w;
  int port = 0;
  w.listen_fd = tcp_listen(bind_host, 0, &port);
  w.listen_addr = bind_host + ":" + std::to_string(port);
  w.token = token;
  auto hp = split_host_port(seed_addr);
  int fd = -1;
  double backoff = 0.5;
  for (int attempt = 0; attempt < 5 && fd < 0; ++attempt) {
    try {
      fd = tcp_connect(hp.first, hp.second, backoff);
    } catch (const NexarError&) {
      if (attempt == 4) {
        close_fd(w.listen_fd);
        throw;
      }
      backoff *= 2;
    }
  }
  try {
    const int raw = fd;
    fd = -1;  // the stream owns (and on failure closes) the socket
    auto io = tls ? tls_client(raw, TlsIdentity{}, false, kTlsHandshakeTimeoutS) : plain_stream(raw);
    write_framed(*io, Message::hello(token, w.listen_addr));
    Message m = read_framed(*io);
    if (m.kind != MsgKind::Welcome) fail(Err::DecodeFailed, "expected Welcome from seed");
    w.rank = m.rank;
    w.world_size = m.world_size;
    w.peers = m.peers;
    if (tls) w.tls = recv_identity(*io);
  } catch (...) {
    if (fd >= 0) close_fd(fd);
    close_fd(w.listen_fd);
    throw;
  }
  return w;
}

}  // namespace nexar
