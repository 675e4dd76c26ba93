// Broadcast event channel: every subscriber receives every event emitted
// after it subscribed, in emission order, on its own queue (the semantics of
// the reference's tokio broadcast channels for RecoveryEvent / ElasticEvent,
// nexar/src/cluster/recovery.rs:56-81 and elastic.rs:102-132). A subscriber
// that falls more than `kMaxQueued` events behind loses the oldest ones.
#pragma once
#include <chrono>
#include <condition_variable>
#include <deque>
#include <memory>
#include <mutex>
#include <vector>

namespace nexar {

template <class E>
class EventSubscription {
 public:
  static constexpr size_t kMaxQueued = 1024;
  // Next event, waiting up to timeout_s (< 0: forever); false on timeout or
  // when the channel was closed and the queue is drained.
  bool recv(double timeout_s, E* out) {
    std::unique_lock<std::mutex> lk(mu_);
    auto ready = [&] { return !q_.empty() || closed_; };
    if (timeout_s < 0) {
      cv_.wait(lk, ready);
    } else if (!cv_.wait_for(lk, std::chrono::duration<double>(timeout_s), ready)) {
      return false;
    }
    if (q_.empty()) return false;
    *out = std::move(q_.front());
    q_.pop_front();
    return true;
  }
  size_t pending() const {
    std::lock_guard<std::mutex> lk(mu_);
    return q_.size();
  }
  size_t dropped() const {
    std::lock_guard<std::mutex> lk(mu_);
    return dropped_;
  }
  void push(const E& e) {
    {
      std::lock_guard<std::mutex> lk(mu_);
      if (q_.size() == kMaxQueued) {
        q_.pop_front();
        ++dropped_;
      }
      q_.push_back(e);
    }
    cv_.notify_all();
  }
  void close() {
    {
      std::lock_guard<std::mutex> lk(mu_);
      closed_ = true;
    }
    cv_.notify_all();
  }

 private:
  mutable std::mutex mu_;
  std::condition_variable cv_;
  std::deque<E> q_;
  size_t dropped_ = 0;
  bool closed_ = false;
};

template <class E>
class EventChannel {
 public:
  std::shared_ptr<EventSubscription<E>> subscribe() {
    auto s = std::make_shared<EventSubscription<E>>();
    std::lock_guard<std::mutex> lk(mu_);
    if (closed_) s->close();
    subs_.push_back(s);
    return s;
  }
  void emit(const E& e) {
    std::vector<std::shared_ptr<EventSubscription<E>>> live;
    {
      std::lock_guard<std::mutex> lk(mu_);
      std::vector<std::weak_ptr<EventSubscription<E>>> keep;
      for (auto& w : subs_)
        if (auto s = w.lock()) {
          live.push_back(s);
          keep.push_back(w);
        }
      subs_.swap(keep);
    }
    for (auto& s : live) s->push(e);
  }
  void close() {
    std::vector<std::shared_ptr<EventSubscription<E>>> live;
    {
      std::lock_guard<std::mutex> lk(mu_);
      closed_ = true;
      for (auto& w : subs_)
        if (auto s = w.lock()) live.push_back(s);
    }
    for (auto& s : live) s->close();
  }

 private:
  std::mutex mu_;
  std::vector<std::weak_ptr<EventSubscription<E>>> subs_;
  bool closed_ = false;
};

}  // namespace nexar
