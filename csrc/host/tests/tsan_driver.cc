// Native driver for a ThreadSanitizer build of the host control plane (no
// Python): every thread below is a rank of one in-process cluster, so TSAN
// sees the transport's router threads, the senders, the heartbeat monitor,
// the recovery orchestrator, the TLS streams and a device adapter shared by
// every rank's thread interleave for real.
//
//   g++ -std=c++17 -O1 -g -fsanitize=thread -I csrc/host csrc/host/<runtime .cc files>
//       csrc/host/tests/tsan_driver.cc -lssl -lcrypto -pthread -o tsan_driver
//   ./tsan_driver            (exit 0 and no "WARNING: ThreadSanitizer" report)
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <thread>
#include <vector>

#include "client.h"
#include "recovery.h"

using namespace nexar;

namespace {

void run_all(const std::vector<std::shared_ptr<NexarClient>>& cs, const std::function<void(NexarClient&)>& fn) {
  std::vector<std::thread> ts;
  for (auto& c : cs) ts.emplace_back([&, c] { fn(*c); });
  for (auto& t : ts) t.join();
}

int check(bool ok, const char* what) {
  if (!ok) {
    std::fprintf(stderr, "FAILED: %s\n", what);
    std::exit(1);
  }
  return 0;
}

void collectives(bool tls) {
  Config cfg;
  cfg.tls = tls;
  cfg.heartbeat_interval_s = 0.05;
  auto cs = NexarClient::bootstrap_local(4, cfg);
  std::vector<std::vector<float>> bufs(4, std::vector<float>(50000));
  run_all(cs, [&](NexarClient& c) {
    auto& b = bufs[c.rank()];
    for (auto& x : b) x = (float)(c.rank() + 1);
    c.all_reduce(b.data(), b.size(), DataType::F32, ReduceOp::Sum);
    std::vector<float> out(4 * 1000);
    c.all_gather(b.data(), out.data(), 1000, DataType::F32);
    std::vector<float> rs(b.size() / 4);
    c.reduce_scatter(b.data(), rs.data(), rs.size(), DataType::F32, ReduceOp::Sum);
    c.broadcast(b.data(), 1000, DataType::F32, 2);
    // two concurrent non-blocking all-reduces (tags taken at call time)
    const uint64_t t1 = c.next_collective_tag(), t2 = c.next_collective_tag();
    float* p = b.data();
    auto h1 = c.spawn([&c, p, t1] { c.all_reduce_tagged(p, 1000, DataType::F32, ReduceOp::Max, t1); });
    auto h2 = c.spawn([&c, p, t2] { c.all_reduce_tagged(p + 1000, 1000, DataType::F32, ReduceOp::Min, t2); });
    h1.wait();
    h2.wait();
    const Rank peer = (c.rank() + 1) % 4, from = (c.rank() + 3) % 4;
    std::vector<char> msg(1 << 16, (char)c.rank()), got(1 << 16);
    std::thread tx([&] { c.send(msg.data(), msg.size(), peer, 7); });
    c.recv(got.data(), got.size(), from, 7);
    tx.join();
    check(got[100] == (char)from, "p2p payload");
    c.barrier();
  });
  for (auto& b : bufs) check(b[5000] == 10.0f && b[0] == 10.0f, "all_reduce + broadcast + non-blocking results");
  for (auto& c : cs) c->close();
}

void recovery() {
  Config cfg;
  cfg.heartbeat_interval_s = 0.05;
  cfg.heartbeat_timeout_s = 0.5;
  cfg.recovery_timeout_s = 5.0;
  cfg.collective_timeout_s = 2.0;
  auto cs = NexarClient::bootstrap_local(4, cfg);
  std::vector<std::unique_ptr<RecoveryOrchestrator>> orch;
  for (int r = 0; r < 4; ++r)
    if (r != 2) orch.push_back(std::make_unique<RecoveryOrchestrator>(cs[r], RecoveryPolicy::Automatic));
  // A broadcast receiver drained on its own thread while the orchestrator
  // thread emits into it.
  auto sub = orch[0]->subscribe();
  std::atomic<bool> got{false};
  std::thread listener([&] {
    RecoveryEvent e;
    if (sub->recv(15.0, &e)) got = e.dead_ranks.size() == 1 && e.dead_ranks[0] == 2;
  });
  for (auto& o : orch) o->start();
  cs[2]->close();
  std::vector<std::shared_ptr<NexarClient>> survivors;
  for (auto& o : orch) {
    RecoveryEvent e;
    check(o->next_event(15.0, &e), "recovery event");
    survivors.push_back(o->client());
  }
  listener.join();
  check(got.load(), "subscribed recovery event");
  std::vector<std::vector<float>> bufs(3, std::vector<float>(64, 1.0f));
  run_all(survivors, [&](NexarClient& c) { c.all_reduce(bufs[c.rank()].data(), 64, DataType::F32, ReduceOp::Sum); });
  for (auto& b : bufs) check(b[0] == 3.0f, "all_reduce after recovery");
  for (auto& o : orch) o->shutdown();
  for (auto& c : survivors) c->close();
  for (auto& c : cs) c->close();
}

// An adapter whose buffers are not host-addressable (the staging paths of
// every collective and of p2p run), shared by all ranks' threads; it counts
// the bytes it stages from several threads at once.
class CountingStagingAdapter : public DeviceAdapter {
 public:
  std::string name() const override { return "staging-test"; }
  void stage_for_send(const void* ptr, size_t n, uint8_t* out) override {
    std::memcpy(out, ptr, n);
    staged += n;
  }
  void receive_to_device(const uint8_t* src, size_t n, void* ptr) override {
    std::memcpy(ptr, src, n);
    received += n;
  }
  void reduce_inplace(void* dst, const void* src, size_t count, DataType dt, ReduceOp op) override {
    reduce_slice(dst, src, count, dt, op);
  }
  std::atomic<uint64_t> staged{0}, received{0};
};

void staged_collectives() {
  Config cfg;
  cfg.heartbeat_interval_s = 0.05;
  auto cs = NexarClient::bootstrap_local(3, cfg);
  auto ad = std::make_shared<CountingStagingAdapter>();
  for (auto& c : cs) c->set_adapter(ad);
  std::vector<std::vector<float>> bufs(3, std::vector<float>(3000));
  run_all(cs, [&](NexarClient& c) {
    auto& b = bufs[c.rank()];
    for (auto& x : b) x = (float)(c.rank() + 1);
    c.all_reduce(b.data(), b.size(), DataType::F32, ReduceOp::Sum);
    std::vector<float> out(3 * 100), rs(1000), a2a(3 * 100);
    c.all_gather(b.data(), out.data(), 100, DataType::F32);
    c.reduce_scatter(b.data(), rs.data(), rs.size(), DataType::F32, ReduceOp::Sum);
    c.all_to_all(b.data(), a2a.data(), 100, DataType::F32);
    std::vector<float> g(c.rank() == 1 ? 300 : 0);
    c.gather(b.data(), c.rank() == 1 ? g.data() : nullptr, 100, DataType::F32, 1);
    c.scan(b.data(), 100, DataType::F32, ReduceOp::Sum);
    const Rank peer = (c.rank() + 1) % 3, from = (c.rank() + 2) % 3;
    std::vector<char> msg(4096, (char)c.rank()), got(4096);
    std::thread tx([&] { c.send(msg.data(), msg.size(), peer, 9); });
    c.recv(got.data(), got.size(), from, 9);
    tx.join();
    check(got[7] == (char)from, "staged p2p payload");
  });
  check(bufs[0][2000] == 6.0f, "staged all_reduce");
  check(ad->staged.load() > 0 && ad->received.load() > 0, "adapter used");
  for (auto& c : cs) c->close();
}

}  // namespace

int main() {
  collectives(false);
  collectives(true);
  staged_collectives();
  recovery();
  std::printf("tsan driver: ok\n");
  return 0;
}
