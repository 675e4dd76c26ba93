// Failure recovery and elastic membership.
//
// RecoveryOrchestrator follows nexar/src/cluster/recovery.rs:16-355: it
// watches the mesh's failure list; policy Abort raises, Manual emits an event
// and keeps the communicator, Automatic runs an agreement round (leader =
// lowest surviving rank collects RecoveryVote{epoch, dead} from every
// survivor, broadcasts the union as RecoveryAgreement) and swaps in
// rebuild_excluding(agreed). A failure that arrives during the agreement
// restarts it with the larger dead set (cascading failures).
//
// ElasticManager follows nexar/src/cluster/elastic.rs: elastic_checkpoint()
// is a collective sync point. Every rank sends ElasticCheckpoint{epoch} to
// rank 0, which answers with ElasticCheckpointAck{joining, leaving,
// new_world_size}; then existing ranks connect to the joiners, the
// communicator is rebuilt with the joiners appended and the leavers removed.
// Joiners come from the seed's accept_elastic queue on rank 0.
#pragma once

#include <deque>
#include <map>

#include "client.h"
#include "events.h"

namespace nexar {

struct RecoveryEvent {
  Rank old_rank;
  Rank new_rank;
  uint32_t new_world_size;
  std::vector<Rank> dead_ranks;
};

class RecoveryOrchestrator {
 public:
  RecoveryOrchestrator(std::shared_ptr<NexarClient> client, RecoveryPolicy policy);
  static std::unique_ptr<RecoveryOrchestrator> from_config(std::shared_ptr<NexarClient> client);
  ~RecoveryOrchestrator();
  // Start the watch loop on a background thread.
  void start();
  // Run the watch loop on the calling thread until shutdown() (the
  // reference's `run`); throws if the loop already runs on start()'s thread.
  void run();
  // Broadcast receiver: sees every event emitted after this call.
  std::shared_ptr<EventSubscription<RecoveryEvent>> subscribe() { return channel_.subscribe(); }
  void shutdown();
  // Run one recovery synchronously for an observed dead set (used by run()).
  void recover(std::vector<Rank> dead);
  std::shared_ptr<NexarClient> client() const;
  // Next event, waiting up to timeout_s; false on timeout.
  bool next_event(double timeout_s, RecoveryEvent* out);
  // Error raised by the loop (Abort policy or a failed recovery), if any.
  std::string error() const;

 private:
  std::vector<Rank> agree(const std::shared_ptr<NexarClient>& c, Rank leader, const std::set<Rank>& alive,
                          const std::vector<Rank>& my_dead, uint64_t epoch, uint64_t seen_version,
                          bool* interrupted);
  void loop();
  void emit(RecoveryEvent e);
  mutable std::mutex mu_;
  std::condition_variable cv_;
  std::shared_ptr<NexarClient> client_;
  RecoveryPolicy policy_;
  std::deque<RecoveryEvent> events_;
  EventChannel<RecoveryEvent> channel_;
  std::string error_;
  // Leader side: the latest vote of each survivor, kept across agreement
  // attempts (a vote consumed by an attempt that a later failure interrupted
  // is not sent again by a voter that already knew every failure). Cleared
  // after a rebuild, which renumbers the ranks. Orchestrator thread only.
  std::map<Rank, std::vector<Rank>> votes_;
  std::thread thr_;
  std::atomic<bool> stop_{false};
};

struct ElasticEvent {
  uint64_t epoch;
  Rank new_rank;
  uint32_t new_world_size;
  std::vector<Rank> joined;  // mesh ranks
  std::vector<Rank> left;    // communicator ranks (old numbering)
};

class ElasticManager {
 public:
  // `seed` is non-null on the rank that hosts the seed (rank 0).
  ElasticManager(std::shared_ptr<NexarClient> client, std::shared_ptr<SeedNode> seed, uint32_t min_world,
                 uint32_t max_world, double timeout_s);
  // Collective sync point; returns true if membership changed. If this rank
  // left, client() becomes null.
  bool elastic_checkpoint();
  std::shared_ptr<NexarClient> client() const { return client_; }
  // Coordinator (rank 0): schedule a rank to leave at the next checkpoint.
  void remove_node(Rank r);
  std::vector<ElasticEvent> events() const { return events_; }
  // Broadcast receiver: sees every membership change after this call.
  std::shared_ptr<EventSubscription<ElasticEvent>> subscribe() { return channel_.subscribe(); }
  uint64_t epoch() const { return epoch_; }

  // Joiner side: connect to the seed, accept the existing ranks' connections,
  // wait for the checkpoint acknowledgement and build the grown communicator.
  static std::shared_ptr<NexarClient> join(const std::string& seed_addr, const Bytes& token, const Config& cfg,
                                           double timeout_s);

 private:
  std::shared_ptr<NexarClient> client_;
  std::shared_ptr<SeedNode> seed_;
  uint32_t min_world_, max_world_;
  double timeout_s_;
  uint64_t epoch_ = 0;
  std::vector<Rank> pending_leave_;
  std::vector<ElasticEvent> events_;
  EventChannel<ElasticEvent> channel_;
};

}  // namespace nexar
