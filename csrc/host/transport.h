// TCP transport: sockets, the per-peer send side and the per-peer receive
// demultiplexer.
//
// One TCP connection per pair of ranks carries every kind of traffic. Each
// frame starts with a kind byte, as each QUIC stream does in the reference
// (nexar/src/transport/connection.rs:30-35):
//   0x01 framed message   [len u64][8-byte header + body]
//   0x02 raw              [len u64][payload]
//   0x03 raw + comm_id    [comm_id u64][len u64][payload]
//   0x04 raw + tag        [tag u64][len u64][payload]
//   0x05 raw + comm + tag [comm_id u64][tag u64][len u64][payload]   (new)
// Kind 0x05 is an addition: tagged traffic of a split/rebuilt communicator
// carries its comm_id, so two communicators sharing a connection can never
// consume each other's tagged messages. The root communicator (comm_id 0)
// uses 0x04 exactly as the reference does.
//
// Receive side: one reader thread per connection parses frames and files
// them into the source rank's Mailbox under a lane key, mirroring the
// reference's router lanes (nexar/src/transport/router.rs:33-234):
// control, barrier (per comm_id), heartbeat (own lane, see below), rpc
// requests, rpc responses (per req_id), data, raw, raw-per-comm and tagged
// (per comm_id, tag). Heartbeats only refresh the peer's last-seen time, so
// they can never be mistaken for a barrier message (the reference routes them
// to the control lane that barriers read, router.rs:377-392).
#pragma once

#include <atomic>
#include <condition_variable>
#include <deque>
#include <functional>
#include <map>
#include <mutex>
#include <string>
#include <thread>
#include <typeindex>
#include <unordered_map>

#include "tls.h"
#include "buffer_pool.h"
#include "wire.h"

namespace nexar {

enum FrameKind : uint8_t {
  kFrameMessage = 0x01, kFrameRaw = 0x02, kFrameRawComm = 0x03, kFrameRawTagged = 0x04,
  kFrameRawCommTagged = 0x05,
};

// ------------------------------------------------------------------ sockets
std::pair<std::string, int> split_host_port(const std::string& addr);
int tcp_listen(const std::string& host, int port, int* bound_port);
int tcp_accept(int listen_fd, double timeout_s);  // -1 on timeout
int tcp_connect(const std::string& host, int port, double timeout_s);
void write_all(int fd, const void* p, size_t n);
// a then b with one sendmsg per attempt (header + payload of a frame).
void write_pair(int fd, const void* a, size_t na, const void* b, size_t nb);
bool read_exact(int fd, void* p, size_t n);  // false on EOF
size_t read_some(int fd, void* p, size_t n);  // >= 1 byte, 0 on EOF / error
void close_fd(int fd);

// Read/write one framed message (kind 0x01) on a bootstrap socket.
void write_framed(int fd, const Message& m, Priority prio = Priority::Critical);
void write_framed(Stream& s, const Message& m, Priority prio = Priority::Critical);
Message read_framed(Stream& s);
Message read_framed(int fd);

// ------------------------------------------------------------------ mailbox
enum class LaneKind : uint8_t {
  Control = 0, Barrier = 1, RpcRequest = 2, RpcResponse = 3, Data = 4, Raw = 5, RawComm = 6,
  Tagged = 7, RelayControl = 8,
};
struct LaneKey {
  LaneKind kind;
  uint64_t a = 0;  // comm_id / req_id
  uint64_t b = 0;  // tag
  bool operator<(const LaneKey& o) const {
    if (kind != o.kind) return kind < o.kind;
    if (a != o.a) return a < o.a;
    return b < o.b;
  }
};

struct Item {
  Message msg;   // message lanes
  Bytes bytes;   // raw lanes
};

// Per-source-rank set of lanes with blocking, deadline-bounded receive.
class Mailbox {
 public:
  explicit Mailbox(Rank src) : src_(src) {}
  void push(const LaneKey& k, Item it);
  // Pop the oldest item of lane k; throws Timeout on deadline, the close
  // error once the lane is empty and the mailbox is closed.
  Item pop(const LaneKey& k, Clock::time_point deadline);
  // Pop the oldest Data message whose tag matches.
  Item pop_data(uint32_t tag, Clock::time_point deadline);
  void close(Err code, const std::string& why);
  void reopen();
  bool closed() const;
  size_t pending() const;
  Rank src() const { return src_; }

 private:
  // Spin on version_ for a short window before sleeping on cv_: a reply
  // that arrives within microseconds is taken without a futex sleep / wake.
  // Returns once version_ moved away from `seen` or at `until`.
  void spin_until_changed(uint64_t seen, Clock::time_point until) const;

  Rank src_;
  mutable std::mutex mu_;
  std::condition_variable cv_;
  std::map<LaneKey, std::deque<Item>> lanes_;
  std::atomic<uint64_t> version_{0};  // bumped by every push and close
  int waiters_ = 0;                   // threads asleep on cv_ (guarded by mu_)
  bool closed_ = false;
  Err close_code_ = Err::PeerDisconnected;
  std::string close_msg_;
};

// ------------------------------------------------------------------ connection
class PeerConnection {
 public:
  // Takes ownership of the stream (and its socket).
  PeerConnection(Rank peer, std::shared_ptr<Stream> io) : peer_(peer), io_(std::move(io)) {}
  ~PeerConnection();
  Rank peer() const { return peer_; }
  int fd() const { return io_->fd(); }
  bool encrypted() const { return io_->encrypted(); }
  // Reader side (the router thread): false on EOF or error.
  bool read_exact(void* p, size_t n) { return io_->read_exact(p, n); }
  size_t read_some(void* p, size_t n) { return io_->read_some(p, n); }

  void send_message(const Message& m, Priority prio);
  void send_raw(const void* p, size_t n);
  void send_raw_comm(uint64_t comm_id, const void* p, size_t n);
  void send_raw_tagged(uint64_t comm_id, uint64_t tag, const void* p, size_t n);
  // One Data message (wire kind 9: tag, source rank, payload blob), framed
  // and encoded exactly as send_message(Message::data(...)) would, with the
  // payload written straight from `p` (no encode copy).
  void send_data(uint32_t tag, Rank src, const void* p, size_t n, Priority prio);
  // Shut the socket down (fault injection / teardown); the reader sees EOF.
  void close();
  bool alive() const { return alive_.load(); }

  // Type-indexed extension slot for accelerated transports
  // (nexar/src/transport/connection.rs:85-117).
  template <typename T> void add_extension(std::shared_ptr<T> ext) {
    std::lock_guard<std::mutex> g(ext_mu_);
    ext_[std::type_index(typeid(T))] = ext;
  }
  template <typename T> std::shared_ptr<T> extension() const {
    std::lock_guard<std::mutex> g(ext_mu_);
    auto it = ext_.find(std::type_index(typeid(T)));
    return it == ext_.end() ? nullptr : std::static_pointer_cast<T>(it->second);
  }

 private:
  void send_frame(uint8_t kind, const uint64_t* prefix, int nprefix, const void* p, size_t n);
  Rank peer_;
  std::shared_ptr<Stream> io_;
  std::mutex write_mu_;
  std::atomic<bool> alive_{true};
  mutable std::mutex ext_mu_;
  std::unordered_map<std::type_index, std::shared_ptr<void>> ext_;
};

// Reader thread for one connection; payloads it reads are allocated from
// `pool` (see PoolScope in buffer_pool.h) when one is given.
class PeerRouter {
 public:
  using RelayFn = std::function<void(const Message&)>;
  using DisconnectFn = std::function<void(Rank)>;
  PeerRouter(std::shared_ptr<PeerConnection> conn, std::shared_ptr<Mailbox> box, RelayFn on_relay,
             DisconnectFn on_disconnect, std::shared_ptr<BufferPool> pool = nullptr);
  ~PeerRouter();
  void stop();
  double last_seen_s() const;  // seconds since the last frame from this peer

 private:
  void run();
  void dispatch(Message&& m);
  std::shared_ptr<PeerConnection> conn_;
  std::shared_ptr<Mailbox> box_;
  RelayFn on_relay_;
  DisconnectFn on_disconnect_;
  std::shared_ptr<BufferPool> pool_;
  std::atomic<int64_t> last_seen_ns_;
  std::thread thr_;
};

}  // namespace nexar
