#include "recovery.h"

#include <algorithm>

namespace nexar {

namespace {
uint64_t now_ns() {
  return (uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(
             std::chrono::system_clock::now().time_since_epoch()).count();
}

// Pop the next control message of `kind` from `src`, skipping unrelated
// control traffic, until the deadline; `interrupt()` aborts the wait.
bool wait_control(const std::shared_ptr<NexarClient>& c, Rank src, MsgKind kind, double timeout_s, Message* out,
                  const std::function<bool()>& interrupt) {
  const auto t0 = Clock::now();
  while (seconds_since(t0) < timeout_s) {
    if (interrupt && interrupt()) return false;
    try {
      Message m = c->recv_control_from(src, 0.05);
      if (m.kind == kind) {
        *out = std::move(m);
        return true;
      }
    } catch (const NexarError& e) {
      if (e.code() != Err::Timeout) throw;
    }
  }
  fail(Err::Recovery, "timeout waiting for " + std::string(msg_kind_name(kind)) + " from rank " + std::to_string(src));
}
}  // namespace

// ============================================================ recovery
RecoveryOrchestrator::RecoveryOrchestrator(std::shared_ptr<NexarClient> client, RecoveryPolicy policy)
    : client_(std::move(client)), policy_(policy) {}

std::unique_ptr<RecoveryOrchestrator> RecoveryOrchestrator::from_config(std::shared_ptr<NexarClient> client) {
  const RecoveryPolicy p = client->config().recovery_policy;
  return std::make_unique<RecoveryOrchestrator>(std::move(client), p);
}

RecoveryOrchestrator::~RecoveryOrchestrator() { shutdown(); }

void RecoveryOrchestrator::start() {
  if (thr_.joinable()) return;
  stop_ = false;
  thr_ = std::thread([this] { loop(); });
}

void RecoveryOrchestrator::run() {
  if (thr_.joinable()) fail(Err::Recovery, "run(): the watch loop already runs (start())");
  stop_ = false;
  loop();
}

void RecoveryOrchestrator::shutdown() {
  stop_ = true;
  cv_.notify_all();
  if (thr_.joinable()) thr_.join();
  channel_.close();
}

std::shared_ptr<NexarClient> RecoveryOrchestrator::client() const {
  std::lock_guard<std::mutex> g(mu_);
  return client_;
}

void RecoveryOrchestrator::emit(RecoveryEvent e) {
  channel_.emit(e);
  {
    std::lock_guard<std::mutex> g(mu_);
    events_.push_back(std::move(e));
  }
  cv_.notify_all();
}

bool RecoveryOrchestrator::next_event(double timeout_s, RecoveryEvent* out) {
  std::unique_lock<std::mutex> lk(mu_);
  if (!cv_.wait_for(lk, std::chrono::duration<double>(timeout_s), [&] { return !events_.empty(); })) return false;
  *out = events_.front();
  events_.pop_front();
  return true;
}

std::string RecoveryOrchestrator::error() const {
  std::lock_guard<std::mutex> g(mu_);
  return error_;
}

void RecoveryOrchestrator::loop() {
  auto mesh = client()->mesh();
  uint64_t seen = 0;
  while (!stop_) {
    uint64_t ver = 0;
    mesh->wait_failure(seen, 0.1, &ver);
    if (stop_) return;
    if (ver == seen) continue;
    seen = ver;
    std::vector<Rank> dead = client()->dead_ranks();
    if (dead.empty()) continue;
    try {
      if (policy_ == RecoveryPolicy::Abort) {
        fail(Err::Recovery, "recovery failed: node failure detected and policy is Abort");
      } else if (policy_ == RecoveryPolicy::Manual) {
        auto c = client();
        emit(RecoveryEvent{c->rank(), c->rank(), c->world_size(), dead});
      } else {
        recover(dead);
        seen = mesh->failure_version();
      }
    } catch (const std::exception& e) {
      {
        std::lock_guard<std::mutex> g(mu_);
        error_ = e.what();
      }
      cv_.notify_all();
      return;
    }
  }
}

std::vector<Rank> RecoveryOrchestrator::agree(const std::shared_ptr<NexarClient>& c, Rank leader,
                                              const std::set<Rank>& alive, const std::vector<Rank>& my_dead,
                                              uint64_t epoch, uint64_t seen_version, bool* interrupted) {
  auto mesh = c->mesh();
  auto interrupt = [&] { return mesh->failure_version() != seen_version; };
  const double timeout = c->config().recovery_timeout_s;
  *interrupted = false;
  if (c->rank() == leader) {
    std::set<Rank> uni(my_dead.begin(), my_dead.end());
    for (Rank src : alive) {
      if (src == leader) continue;
      auto it = votes_.find(src);
      if (it == votes_.end()) {
        Message m;
        if (!wait_control(c, src, MsgKind::RecoveryVote, timeout, &m, interrupt)) {
          *interrupted = true;
          return {};
        }
        it = votes_.emplace(src, m.dead_ranks).first;
      }
      uni.insert(it->second.begin(), it->second.end());
    }
    std::vector<Rank> agreed(uni.begin(), uni.end());
    for (Rank dst : alive)
      if (dst != leader) c->send_message_to(dst, Message::recovery_agreement(epoch, agreed), Priority::Critical);
    return agreed;
  }
  c->send_message_to(leader, Message::recovery_vote(epoch, my_dead), Priority::Critical);
  Message m;
  if (!wait_control(c, leader, MsgKind::RecoveryAgreement, timeout, &m, interrupt)) {
    *interrupted = true;
    return {};
  }
  return m.dead_ranks;
}

void RecoveryOrchestrator::recover(std::vector<Rank> dead_in) {
  std::set<Rank> dead(dead_in.begin(), dead_in.end());
  auto c = client();
  auto mesh = c->mesh();
  for (int attempt = 0; attempt < 16; ++attempt) {
    const uint64_t ver = mesh->failure_version();
    for (Rank r : c->dead_ranks()) dead.insert(r);
    std::set<Rank> alive;
    for (Rank r = 0; r < c->world_size(); ++r)
      if (!dead.count(r)) alive.insert(r);
    if (alive.empty()) fail(Err::Recovery, "recovery failed: no survivors remaining");
    const Rank leader = *alive.begin();
    bool interrupted = false;
    std::vector<Rank> agreed;
    try {
      agreed = agree(c, leader, alive, std::vector<Rank>(dead.begin(), dead.end()), now_ns(), ver, &interrupted);
    } catch (const NexarError& e) {
      if (e.code() == Err::PeerDisconnected || e.code() == Err::CollectiveFailed) {
        interrupted = true;  // someone else died mid-agreement: retry with the larger set
      } else {
        throw;
      }
    }
    if (interrupted) continue;
    votes_.clear();
    auto nc = c->rebuild_excluding(agreed);
    const Rank old = c->rank();
    {
      std::lock_guard<std::mutex> g(mu_);
      client_ = nc;
    }
    emit(RecoveryEvent{old, nc->rank(), nc->world_size(), agreed});
    return;
  }
  fail(Err::Recovery, "recovery failed: too many cascading failures");
}

// ============================================================ elastic
ElasticManager::ElasticManager(std::shared_ptr<NexarClient> client, std::shared_ptr<SeedNode> seed,
                               uint32_t min_world, uint32_t max_world, double timeout_s)
    : client_(std::move(client)), seed_(std::move(seed)), min_world_(min_world), max_world_(max_world),
      timeout_s_(timeout_s) {}

void ElasticManager::remove_node(Rank r) { pending_leave_.push_back(r); }

static uint64_t elastic_comm_id(uint64_t epoch, uint32_t new_world, const PeerList& joining,
                                const std::vector<Rank>& leaving) {
  Bytes a, b, cc;
  put_u64(a, epoch);
  put_u32(a, new_world);
  for (auto& j : joining) put_u32(b, j.first);
  for (Rank l : leaving) put_u32(cc, l);
  return fnv1a_comm_id({a, b, cc});
}

bool ElasticManager::elastic_checkpoint() {
  if (!client_) fail(Err::Elastic, "elastic scaling error: this rank has left the group");
  auto c = client_;
  ++epoch_;
  Message ack;
  const double timeout = timeout_s_;
  if (c->rank() != 0) {
    c->send_message_to(0, Message::elastic_checkpoint(epoch_), Priority::Critical);
    try {
      wait_control(c, 0, MsgKind::ElasticCheckpointAck, timeout, &ack, nullptr);
    } catch (const NexarError&) {
      fail(Err::ElasticTimeout, "elastic checkpoint timed out after " + std::to_string((int)(timeout * 1000)) +
                                    "ms (epoch " + std::to_string(epoch_) + ")");
    }
  } else {
    for (Rank r = 1; r < c->world_size(); ++r) {
      Message m;
      try {
        wait_control(c, r, MsgKind::ElasticCheckpoint, timeout, &m, nullptr);
      } catch (const NexarError&) {
        fail(Err::ElasticTimeout, "elastic checkpoint timed out after " + std::to_string((int)(timeout * 1000)) +
                                      "ms (epoch " + std::to_string(epoch_) + ")");
      }
    }
    PeerList joining;
    if (seed_) {
      for (auto& pj : seed_->take_pending_joins()) {
        joining.emplace_back(pj.rank, pj.listen_addr);  // dropping pj closes its bootstrap stream
      }
    }
    std::vector<Rank> leaving = pending_leave_;
    pending_leave_.clear();
    std::sort(leaving.begin(), leaving.end());
    leaving.erase(std::unique(leaving.begin(), leaving.end()), leaving.end());
    uint32_t new_world = c->world_size() + (uint32_t)joining.size() - (uint32_t)leaving.size();
    if (new_world < min_world_) {
      leaving.clear();  // refuse to shrink below the minimum
      new_world = c->world_size() + (uint32_t)joining.size();
    }
    if (max_world_ && new_world > max_world_) fail(Err::Elastic, "elastic scaling error: exceeds max world size");
    ack = Message::elastic_checkpoint_ack(epoch_, joining, leaving, new_world);
    for (Rank r = 1; r < c->world_size(); ++r) c->send_message_to(r, ack, Priority::Critical);
  }
  if (ack.joining.empty() && ack.leaving.empty()) return false;
  auto mesh = c->mesh();
  const uint64_t cid = elastic_comm_id(ack.epoch, ack.new_world_size, ack.joining, ack.leaving);
  std::vector<Rank> joined;
  if (!ack.joining.empty()) {
    Rank maxr = 0;
    for (auto& j : ack.joining) maxr = std::max(maxr, j.first);
    mesh->grow(maxr + 1);
    for (auto& j : ack.joining) {
      auto hp = split_host_port(j.second);
      auto io = mesh->dial(tcp_connect(hp.first, hp.second, timeout));
      Bytes h;
      put_u32(h, 0x4e584d31);
      put_u32(h, mesh->rank());
      put_u32(h, ack.new_world_size);
      put_u64(h, mesh->token().empty() ? 0 : fnv1a_comm_id({mesh->token()}));
      io->write_all(h.data(), h.size());
      mesh->add_connection(j.first, io);
      joined.push_back(j.first);
    }
    if (c->rank() == 0)
      for (auto& j : ack.joining) mesh->send_message(j.first, ack, Priority::Critical);
  }
  auto nc = joined.empty() ? c : c->rebuild_adding(joined, cid);
  const bool me_leaving = std::find(ack.leaving.begin(), ack.leaving.end(), c->rank()) != ack.leaving.end();
  if (!ack.leaving.empty()) {
    if (me_leaving) {
      events_.push_back(ElasticEvent{ack.epoch, 0, ack.new_world_size, joined, ack.leaving});
      channel_.emit(events_.back());
      client_ = nullptr;
      return true;
    }
    nc = nc->rebuild_excluding(ack.leaving);
  }
  client_ = nc;
  events_.push_back(ElasticEvent{ack.epoch, nc->rank(), nc->world_size(), joined, ack.leaving});
  channel_.emit(events_.back());
  return true;
}

std::shared_ptr<NexarClient> ElasticManager::join(const std::string& seed_addr, const Bytes& token, const Config& cfg,
                                                  double timeout_s) {
  WorkerInfo info = WorkerNode::connect(seed_addr, token, "127.0.0.1", cfg.tls);
  const Rank me = info.rank;
  auto mesh = std::make_shared<Mesh>(me, me + 1, cfg, token);
  mesh->listen_fd = info.listen_fd;
  mesh->listen_addr = info.listen_addr;
  if (cfg.tls) mesh->set_tls(info.tls);
  std::set<Rank> connected;
  bool have_ack = false;
  Message ack;
  const auto t0 = Clock::now();
  size_t expect = SIZE_MAX;
  while (connected.size() < expect) {
    if (seconds_since(t0) > timeout_s) fail(Err::ElasticTimeout, "elastic join timed out");
    int fd = tcp_accept(info.listen_fd, 0.05);
    if (fd >= 0) {
      try {
        auto io = mesh->answer(fd);
        uint8_t b[20];
        if (io->read_exact(b, sizeof(b)) && (uint32_t)get_le(b, 4) == 0x4e584d31) {
          const Rank p = (Rank)get_le(b + 4, 4);
          mesh->grow(std::max<uint32_t>(mesh->world(), p + 1));
          mesh->add_connection(p, io);
          connected.insert(p);
        }
      } catch (const NexarError& e) {
        NEXAR_LOG(LogLevel::Warn, std::string("rejected join connection: ") + e.what());
      }
    }
    if (!have_ack && connected.count(0)) {
      try {
        auto it = mesh->box(0)->pop(LaneKey{LaneKind::Control, 0, 0}, Clock::now());
        if (it.msg.kind == MsgKind::ElasticCheckpointAck) {
          ack = std::move(it.msg);
          have_ack = true;
          size_t higher = 0;
          for (auto& j : ack.joining)
            if (j.first > me) ++higher;
          expect = ack.new_world_size + ack.leaving.size() - 1 - higher;
          // dial co-joiners with a higher rank
          Rank maxr = me;
          for (auto& j : ack.joining) maxr = std::max(maxr, j.first);
          mesh->grow(maxr + 1);
          for (auto& j : ack.joining) {
            if (j.first <= me) continue;
            auto hp = split_host_port(j.second);
            auto cio = mesh->dial(tcp_connect(hp.first, hp.second, timeout_s));
            Bytes h;
            put_u32(h, 0x4e584d31);
            put_u32(h, me);
            put_u32(h, ack.new_world_size);
            put_u64(h, token.empty() ? 0 : fnv1a_comm_id({token}));
            cio->write_all(h.data(), h.size());
            mesh->add_connection(j.first, cio);
          }
        }
      } catch (const NexarError&) {
      }
    }
  }
  // Existing members (sorted mesh ranks) followed by the joiners.
  std::set<Rank> joiners;
  for (auto& j : ack.joining) joiners.insert(j.first);
  std::vector<Rank> existing;
  for (Rank p : connected)
    if (!joiners.count(p)) existing.push_back(p);
  std::vector<Rank> rm = existing;
  for (Rank j : joiners) rm.push_back(j);
  mesh->set_routing(TopologyStrategy{});
  mesh->start_health_monitor();
  Rank my = 0;
  for (size_t i = 0; i < rm.size(); ++i)
    if (rm[i] == me) my = (Rank)i;
  const uint64_t cid = elastic_comm_id(ack.epoch, ack.new_world_size, ack.joining, ack.leaving);
  auto c = std::make_shared<NexarClient>(mesh, my, (uint32_t)rm.size(), cid, rm, nullptr);
  if (!ack.leaving.empty()) return c->rebuild_excluding(ack.leaving);
  return c;
}

}  // namespace nexar
