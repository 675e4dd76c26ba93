// Cluster layer: sparse overlay topologies, membership map, seed/worker
// bootstrap.
//
// Topologies follow nexar/src/cluster/sparse.rs:6-254 (FullMesh, KRegular,
// Hypercube; neighbours, greedy routing, BFS spanning tree, alternative hops).
// Ties in the greedy KRegular routing are broken towards the lower rank so
// every rank computes the same table.
//
// Seed / worker follow nexar/src/cluster/{seed,worker}.rs: the seed assigns
// ranks in join order after checking the protocol version and the cluster
// token, then sends every worker a Welcome with the full peer table. Unlike
// the reference, workers advertise a real listen address (their mesh
// listener), so ranks in different processes can connect to each other.
#pragma once

#include <atomic>
#include <map>
#include <mutex>
#include <set>
#include <thread>

#include "tls.h"
#include "transport.h"

namespace nexar {

// ------------------------------------------------------------------ topology
std::set<Rank> build_neighbors(const TopologyStrategy& s, Rank rank, uint32_t world);

struct RoutingTable {
  std::set<Rank> neighbors;
  std::map<Rank, Rank> next_hop;
  // Direct neighbour, next hop, or -1 if unreachable.
  long long route(Rank dest) const;
  bool is_neighbor(Rank r) const { return neighbors.count(r) != 0; }
};
RoutingTable build_routing_table(const TopologyStrategy& s, Rank rank, uint32_t world);

struct SpanningTree {
  std::map<Rank, Rank> parent;
  std::map<Rank, std::vector<Rank>> children;
};
SpanningTree build_spanning_tree(const TopologyStrategy& s, Rank root, uint32_t world);
long long find_alternative_hop(const TopologyStrategy& s, Rank rank, Rank dest, Rank failed_hop,
                               uint32_t world);
std::vector<Rank> optimal_ring_order(uint32_t world);

// ------------------------------------------------------------------ cluster map
struct PeerInfo {
  std::string addr;
  double last_heartbeat_s = 0;
  bool alive = true;
};

// rank -> {addr, last heartbeat, alive}; the epoch bumps on every change
// (nexar/src/cluster/topology.rs:7-98).
class ClusterMap {
 public:
  void add_peer(Rank r, const std::string& addr);
  void remove_peer(Rank r);
  void heartbeat(Rank r, double now_s);
  std::vector<Rank> alive_peers() const;
  std::vector<Rank> check_timeouts(double now_s, double timeout_s);  // marks and returns newly dead
  uint64_t epoch() const { return epoch_; }
  size_t size() const;
  bool contains(Rank r) const;
  std::string addr(Rank r) const;

 private:
  mutable std::mutex mu_;
  std::map<Rank, PeerInfo> peers_;
  uint64_t epoch_ = 0;
};

// ------------------------------------------------------------------ seed / worker
struct PendingJoin {
  Rank rank;
  std::string listen_addr;
  std::shared_ptr<Stream> io;  // bootstrap connection, Welcome already sent
};

class SeedNode {
 public:
  // `token` empty = no authentication (bind_local in the reference). With
  // `tls` the seed creates the cluster CA, serves bootstrap over TLS and
  // hands every worker its certificate (see tls.h).
  static std::shared_ptr<SeedNode> bind(const std::string& addr, const Bytes& token, bool tls = false);
  static std::shared_ptr<SeedNode> bind_local(bool tls = false);
  bool tls() const { return ca_ != nullptr; }
  ~SeedNode();
  std::string local_addr() const { return addr_; }
  const Bytes& token() const { return token_; }
  void set_formation_timeout(double s) { formation_timeout_s_ = s; }
  // Replace the cluster CA of a TLS seed with a restored one (before
  // form_cluster); identities issued afterwards chain to it.
  void use_ca(std::shared_ptr<ClusterCA> ca);
  std::shared_ptr<ClusterCA> ca() const { return ca_; }

  // Accept `world` workers, assign ranks in join order, send every worker its
  // Welcome. Returns the peer table (rank -> listen addr).
  PeerList form_cluster(uint32_t world);
  // After formation: keep accepting joiners (ranks world, world+1, ...) up to
  // max_world in a background thread; they queue as pending joins.
  void accept_elastic(uint32_t max_world);
  std::vector<PendingJoin> take_pending_joins();
  void close();

 private:
  SeedNode() = default;
  std::shared_ptr<Stream> accept_bootstrap(int fd);
  std::shared_ptr<ClusterCA> ca_;
  TlsIdentity seed_id_;
  int listen_fd_ = -1;
  std::string addr_;
  Bytes token_;
  double formation_timeout_s_ = 60.0;
  PeerList table_;
  std::mutex mu_;
  std::vector<PendingJoin> pending_;
  std::atomic<bool> stop_{false};
  std::thread elastic_thr_;
  Rank next_rank_ = 0;
};

struct WorkerInfo {
  Rank rank = 0;
  uint32_t world_size = 0;
  PeerList peers;
  int listen_fd = -1;         // mesh listener (already bound)
  std::string listen_addr;
  Bytes token;
  TlsIdentity tls;            // issued by the seed when the cluster runs TLS
};

class WorkerNode {
 public:
  // Bind a mesh listener on `bind_host`, connect to the seed (5 attempts with
  // doubling backoff from 500 ms, like nexar/src/cluster/worker.rs:113),
  // send Hello, wait for Welcome.
  static WorkerInfo connect(const std::string& seed_addr, const Bytes& token,
                            const std::string& bind_host = "127.0.0.1", bool tls = false);
};

Bytes token_from_env();
Bytes random_token(size_t n = 32);

}  // namespace nexar
