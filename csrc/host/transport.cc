#include "transport.h"

#include <sys/uio.h>

#include <algorithm>
#include <cstdlib>

#include <arpa/inet.h>
#include <cerrno>
#include <fcntl.h>
#include <netdb.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <poll.h>
#include <sys/socket.h>
#include <unistd.h>

namespace nexar {

// ------------------------------------------------------------------ sockets
std::pair<std::string, int> split_host_port(const std::string& addr) {
  const size_t c = addr.rfind(':');
  if (c == std::string::npos) fail(Err::ConnectionFailed, "address '" + addr + "' is not host:port");
  return {addr.substr(0, c), std::atoi(addr.c_str() + c + 1)};
}

static void tune(int fd) {
  int one = 1;
  setsockopt(fd, IPPROTO_TCP, TCP_NODELAY, &one, sizeof(one));
  int buf = 8 << 20;
  setsockopt(fd, SOL_SOCKET, SO_SNDBUF, &buf, sizeof(buf));
  setsockopt(fd, SOL_SOCKET, SO_RCVBUF, &buf, sizeof(buf));
}

static sockaddr_in resolve(const std::string& host, int port) {
  sockaddr_in sa{};
  sa.sin_family = AF_INET;
  sa.sin_port = htons((uint16_t)port);
  std::string h = host.empty() || host == "localhost" ? "127.0.0.1" : host;
  if (inet_pton(AF_INET, h.c_str(), &sa.sin_addr) != 1) {
    addrinfo hints{}, *res = nullptr;
    hints.ai_family = AF_INET;
    if (getaddrinfo(h.c_str(), nullptr, &hints, &res) != 0 || !res)
      fail(Err::ConnectionFailed, "cannot resolve host '" + host + "'");
    sa.sin_addr = reinterpret_cast<sockaddr_in*>(res->ai_addr)->sin_addr;
    freeaddrinfo(res);
  }
  return sa;
}

int tcp_listen(const std::string& host, int port, int* bound_port) {
  int fd = ::socket(AF_INET, SOCK_STREAM | SOCK_CLOEXEC, 0);
  if (fd < 0) fail(Err::Io, "socket() failed");
  int one = 1;
  setsockopt(fd, SOL_SOCKET, SO_REUSEADDR, &one, sizeof(one));
  sockaddr_in sa = resolve(host, port);
  if (::bind(fd, reinterpret_cast<sockaddr*>(&sa), sizeof(sa)) != 0) {
    ::close(fd);
    fail(Err::Io, "bind(" + host + ":" + std::to_string(port) + ") failed: " + strerror(errno));
  }
  if (::listen(fd, 256) != 0) {
    ::close(fd);
    fail(Err::Io, "listen() failed");
  }
  socklen_t len = sizeof(sa);
  getsockname(fd, reinterpret_cast<sockaddr*>(&sa), &len);
  if (bound_port) *bound_port = ntohs(sa.sin_port);
  return fd;
}

int tcp_accept(int listen_fd, double timeout_s) {
  pollfd p{listen_fd, POLLIN, 0};
  const int ms = timeout_s < 0 ? -1 : (int)(timeout_s * 1000);
  int r = ::poll(&p, 1, ms);
  if (r <= 0) return -1;
  int fd = ::accept4(listen_fd, nullptr, nullptr, SOCK_CLOEXEC);
  if (fd >= 0) tune(fd);
  return fd;
}

int tcp_connect(const std::string& host, int port, double timeout_s) {
  sockaddr_in sa = resolve(host, port);
  const auto t0 = Clock::now();
  double backoff = 0.02;
  while (true) {
    int fd = ::socket(AF_INET, SOCK_STREAM | SOCK_CLOEXEC, 0);
    if (fd < 0) fail(Err::Io, "socket() failed");
    if (::connect(fd, reinterpret_cast<sockaddr*>(&sa), sizeof(sa)) == 0) {
      tune(fd);
      return fd;
    }
    ::close(fd);
    if (seconds_since(t0) > timeout_s)
      fail(Err::ConnectionFailed, "connect to " + host + ":" + std::to_string(port) + " timed out");
    std::this_thread::sleep_for(std::chrono::duration<double>(backoff));
    backoff = std::min(backoff * 2, 0.5);
  }
}

void write_all(int fd, const void* p, size_t n) {
  const char* c = static_cast<const char*>(p);
  while (n > 0) {
    ssize_t w = ::send(fd, c, n, MSG_NOSIGNAL);
    if (w < 0) {
      if (errno == EINTR) continue;
      fail(Err::PeerDisconnected, std::string("send failed: ") + strerror(errno));
    }
    c += w;
    n -= (size_t)w;
  }
}

void write_pair(int fd, const void* a, size_t na, const void* b, size_t nb) {
  iovec v[2] = {{const_cast<void*>(a), na}, {const_cast<void*>(b), nb}};
  int first = 0;
  while (first < 2) {
    msghdr m{};
    m.msg_iov = v + first;
    m.msg_iovlen = 2 - first;
    ssize_t w = ::sendmsg(fd, &m, MSG_NOSIGNAL);
    if (w < 0) {
      if (errno == EINTR) continue;
      fail(Err::PeerDisconnected, std::string("send failed: ") + strerror(errno));
    }
    size_t left = (size_t)w;
    while (first < 2 && left >= v[first].iov_len) {
      left -= v[first].iov_len;
      ++first;
    }
    if (first < 2) {
      v[first].iov_base = static_cast<char*>(v[first].iov_base) + left;
      v[first].iov_len -= left;
    }
  }
}

size_t read_some(int fd, void* p, size_t n) {
  while (true) {
    ssize_t r = ::recv(fd, p, n, 0);
    if (r > 0) return (size_t)r;
    if (r < 0 && errno == EINTR) continue;
    return 0;
  }
}

bool read_exact(int fd, void* p, size_t n) {
  char* c = static_cast<char*>(p);
  while (n > 0) {
    ssize_t r = ::recv(fd, c, n, 0);
    if (r == 0) return false;
    if (r < 0) {
      if (errno == EINTR) continue;
      return false;
    }
    c += r;
    n -= (size_t)r;
  }
  return true;
}

void close_fd(int fd) {
  if (fd >= 0) {
    ::shutdown(fd, SHUT_RDWR);
    ::close(fd);
  }
}

void write_framed(int fd, const Message& m, Priority prio) {
  Bytes enc = encode_message(m, prio);
  Bytes frame;
  frame.reserve(9 + enc.size());
  frame.push_back(kFrameMessage);
  put_u64(frame, enc.size());
  frame.insert(frame.end(), enc.begin(), enc.end());
  write_all(fd, frame.data(), frame.size());
}

void write_framed(Stream& st, const Message& m, Priority prio) {
  Bytes enc = encode_message(m, prio);
  Bytes frame;
  frame.reserve(9 + enc.size());
  frame.push_back(kFrameMessage);
  put_u64(frame, enc.size());
  frame.insert(frame.end(), enc.begin(), enc.end());
  st.write_all(frame.data(), frame.size());
}

Message read_framed(Stream& st) {
  uint8_t kind = 0;
  if (!st.read_exact(&kind, 1)) fail(Err::PeerDisconnected, "connection closed");
  if (kind != kFrameMessage) fail(Err::DecodeFailed, "expected a framed message");
  uint8_t lb[8];
  if (!st.read_exact(lb, 8)) fail(Err::PeerDisconnected, "connection closed");
  const uint64_t len = get_le(lb, 8);
  if (len > kMaxMessageBytes) fail(Err::DecodeFailed, "message too large");
  Bytes b(len);
  if (len && !st.read_exact(b.data(), len)) fail(Err::PeerDisconnected, "connection closed");
  return decode_message(b.data(), b.size());
}

Message read_framed(int fd) {
  uint8_t kind = 0;
  if (!read_exact(fd, &kind, 1)) fail(Err::PeerDisconnected, "connection closed");
  if (kind != kFrameMessage) fail(Err::DecodeFailed, "expected a framed message");
  uint8_t lb[8];
  if (!read_exact(fd, lb, 8)) fail(Err::PeerDisconnected, "connection closed");
  const uint64_t len = get_le(lb, 8);
  if (len > kMaxMessageBytes) fail(Err::DecodeFailed, "message too large");
  Bytes b(len);
  if (len && !read_exact(fd, b.data(), len)) fail(Err::PeerDisconnected, "connection closed");
  return decode_message(b.data(), b.size());
}

// ------------------------------------------------------------------ mailbox
namespace {
// Spin window of a waiting pop (NEXAR_SPIN_US, default 50 us; 0 turns it off).
std::chrono::microseconds mailbox_spin() {
  static const std::chrono::microseconds v = [] {
    const char* e = std::getenv("NEXAR_SPIN_US");
    long us = e && *e ? std::strtol(e, nullptr, 10) : 50;
    return std::chrono::microseconds(us < 0 ? 0 : us);
  }();
  return v;
}

inline void cpu_relax() {
#if defined(__x86_64__) || defined(__i386__)
  __builtin_ia32_pause();
#endif
}
}  // namespace

void Mailbox::spin_until_changed(uint64_t seen, Clock::time_point until) const {
  for (uint32_t i = 1; version_.load(std::memory_order_acquire) == seen; ++i) {
    cpu_relax();
    if ((i & 63) == 0 && Clock::now() >= until) return;
  }
}

void Mailbox::push(const LaneKey& k, Item it) {
  bool wake;
  {
    std::lock_guard<std::mutex> g(mu_);
    lanes_[k].push_back(std::move(it));
    version_.fetch_add(1, std::memory_order_release);
    wake = waiters_ > 0;
  }
  if (wake) cv_.notify_all();
}

Item Mailbox::pop(const LaneKey& k, Clock::time_point deadline) {
  const auto spin_end = std::min(deadline, Clock::now() + mailbox_spin());
  std::unique_lock<std::mutex> lk(mu_);
  while (true) {
    auto it = lanes_.find(k);
    if (it != lanes_.end() && !it->second.empty()) {
      Item v = std::move(it->second.front());
      it->second.pop_front();
      if (it->second.empty()) lanes_.erase(it);  // lanes do not accumulate over long runs
      return v;
    }
    if (closed_) fail(close_code_, close_msg_);
    if (Clock::now() < spin_end) {
      const uint64_t seen = version_.load(std::memory_order_acquire);
      lk.unlock();
      spin_until_changed(seen, spin_end);
      lk.lock();
      continue;
    }
    ++waiters_;
    const auto st = cv_.wait_until(lk, deadline);
    --waiters_;
    if (st == std::cv_status::timeout) {
      auto it2 = lanes_.find(k);
      if (it2 != lanes_.end() && !it2->second.empty()) continue;
      if (closed_) fail(close_code_, close_msg_);
      fail(Err::Timeout, "timed out waiting for rank " + std::to_string(src_));
    }
  }
}

Item Mailbox::pop_data(uint32_t tag, Clock::time_point deadline) {
  const LaneKey k{LaneKind::Data, 0, 0};
  const auto spin_end = std::min(deadline, Clock::now() + mailbox_spin());
  std::unique_lock<std::mutex> lk(mu_);
  while (true) {
    auto it = lanes_.find(k);
    if (it != lanes_.end()) {
      for (auto q = it->second.begin(); q != it->second.end(); ++q) {
        if (q->msg.tag == tag) {
          Item v = std::move(*q);
          it->second.erase(q);
          if (it->second.empty()) lanes_.erase(it);
          return v;
        }
      }
    }
    if (closed_) fail(close_code_, close_msg_);
    if (Clock::now() < spin_end) {
      const uint64_t seen = version_.load(std::memory_order_acquire);
      lk.unlock();
      spin_until_changed(seen, spin_end);
      lk.lock();
      continue;
    }
    ++waiters_;
    const auto st = cv_.wait_until(lk, deadline);
    --waiters_;
    if (st == std::cv_status::timeout) {
      if (closed_) fail(close_code_, close_msg_);
      fail(Err::Timeout, "timed out waiting for data (tag " + std::to_string(tag) + ") from rank " +
                             std::to_string(src_));
    }
  }
}

void Mailbox::close(Err code, const std::string& why) {
  {
    std::lock_guard<std::mutex> g(mu_);
    if (closed_) return;
    closed_ = true;
    close_code_ = code;
    close_msg_ = why;
    version_.fetch_add(1, std::memory_order_release);
  }
  cv_.notify_all();
}

void Mailbox::reopen() {
  std::lock_guard<std::mutex> g(mu_);
  closed_ = false;
}

bool Mailbox::closed() const {
  std::lock_guard<std::mutex> g(mu_);
  return closed_;
}

size_t Mailbox::pending() const {
  std::lock_guard<std::mutex> g(mu_);
  size_t n = 0;
  for (auto& kv : lanes_) n += kv.second.size();
  return n;
}

// ------------------------------------------------------------------ connection
PeerConnection::~PeerConnection() { close(); }

void PeerConnection::send_frame(uint8_t kind, const uint64_t* prefix, int nprefix, const void* p, size_t n) {
  if (!alive_) fail(Err::PeerDisconnected, "peer " + std::to_string(peer_) + " disconnected unexpectedly");
  if (n > kMaxMessageBytes) fail(Err::EncodeFailed, "payload exceeds the 4 GiB limit");
  uint8_t hdr[1 + 8 * 3];
  size_t h = 0;
  hdr[h++] = kind;
  for (int i = 0; i < nprefix; ++i) {
    for (int j = 0; j < 8; ++j) hdr[h++] = (prefix[i] >> (8 * j)) & 0xff;
  }
  std::lock_guard<std::mutex> g(write_mu_);
  try {
    io_->write_pair(hdr, h, p, n);
  } catch (const NexarError&) {
    alive_ = false;
    throw NexarError(Err::PeerDisconnected, "peer " + std::to_string(peer_) + " disconnected unexpectedly");
  }
}

void PeerConnection::send_message(const Message& m, Priority prio) {
  Bytes enc = encode_message(m, prio);
  uint64_t len = enc.size();
  send_frame(kFrameMessage, &len, 1, enc.data(), enc.size());
}
void PeerConnection::send_data(uint32_t tag, Rank src, const void* p, size_t n, Priority prio) {
  if (!alive_) fail(Err::PeerDisconnected, "peer " + std::to_string(peer_) + " disconnected unexpectedly");
  constexpr size_t kBody = kDataPrefixBytes - kHeaderSize;  // kind, tag, src, blob length
  if (n + kBody > 0xffffffffull) fail(Err::EncodeFailed, "message body exceeds u32::MAX bytes");
  uint8_t hdr[1 + 8 + kDataPrefixBytes];
  size_t h = 0;
  hdr[h++] = kFrameMessage;
  const uint64_t frame_len = kDataPrefixBytes + n;
  for (int j = 0; j < 8; ++j) hdr[h++] = (frame_len >> (8 * j)) & 0xff;
  h += encode_data_prefix(tag, src, n, prio, hdr + h);
  std::lock_guard<std::mutex> g(write_mu_);
  try {
    io_->write_pair(hdr, h, p, n);
  } catch (const NexarError&) {
    alive_ = false;
    throw NexarError(Err::PeerDisconnected, "peer " + std::to_string(peer_) + " disconnected unexpectedly");
  }
}

void PeerConnection::send_raw(const void* p, size_t n) {
  uint64_t len = n;
  send_frame(kFrameRaw, &len, 1, p, n);
}
void PeerConnection::send_raw_comm(uint64_t comm_id, const void* p, size_t n) {
  uint64_t pre[2] = {comm_id, n};
  send_frame(kFrameRawComm, pre, 2, p, n);
}
void PeerConnection::send_raw_tagged(uint64_t comm_id, uint64_t tag, const void* p, size_t n) {
  if (comm_id == 0) {
    uint64_t pre[2] = {tag, n};
    send_frame(kFrameRawTagged, pre, 2, p, n);
  } else {
    uint64_t pre[3] = {comm_id, tag, n};
    send_frame(kFrameRawCommTagged, pre, 3, p, n);
  }
}

void PeerConnection::close() {
  if (alive_.exchange(false)) io_->shutdown();
}

// ------------------------------------------------------------------ router
static int64_t now_ns() {
  return std::chrono::duration_cast<std::chrono::nanoseconds>(Clock::now().time_since_epoch()).count();
}

PeerRouter::PeerRouter(std::shared_ptr<PeerConnection> conn, std::shared_ptr<Mailbox> box, RelayFn on_relay,
                       DisconnectFn on_disconnect, std::shared_ptr<BufferPool> pool)
    : conn_(std::move(conn)), box_(std::move(box)), on_relay_(std::move(on_relay)),
      on_disconnect_(std::move(on_disconnect)), pool_(std::move(pool)), last_seen_ns_(now_ns()) {
  thr_ = std::thread([this] { run(); });
}

PeerRouter::~PeerRouter() { stop(); }

void PeerRouter::stop() {
  conn_->close();
  if (thr_.joinable()) {
    if (thr_.get_id() == std::this_thread::get_id()) thr_.detach();
    else thr_.join();
  }
}

double PeerRouter::last_seen_s() const { return (now_ns() - last_seen_ns_.load()) / 1e9; }

void PeerRouter::dispatch(Message&& m) {
  switch (m.kind) {
    case MsgKind::Heartbeat:
      return;  // last_seen already refreshed
    case MsgKind::Barrier:
    case MsgKind::BarrierAck: {
      LaneKey k{LaneKind::Barrier, m.comm_id, 0};
      box_->push(k, Item{std::move(m), {}});
      return;
    }
    case MsgKind::Rpc:
      box_->push(LaneKey{LaneKind::RpcRequest, 0, 0}, Item{std::move(m), {}});
      return;
    case MsgKind::RpcResponse: {
      LaneKey k{LaneKind::RpcResponse, m.req_id, 0};
      box_->push(k, Item{std::move(m), {}});
      return;
    }
    case MsgKind::Data:
      box_->push(LaneKey{LaneKind::Data, 0, 0}, Item{std::move(m), {}});
      return;
    case MsgKind::Relay:
      if (on_relay_) on_relay_(m);
      return;
    default:
      box_->push(LaneKey{LaneKind::Control, 0, 0}, Item{std::move(m), {}});
      return;
  }
}

namespace {
// Buffered reads for the router: frame headers and small payloads come out
// of one 64 KB buffer filled by single reads (one system call per burst of
// small frames instead of three per frame); payloads of half the buffer or
// more are read straight into their destination.
class FrameReader {
 public:
  explicit FrameReader(PeerConnection& c) : c_(c), buf_(kCap) {}
  bool read_exact(void* p, size_t n) {
    uint8_t* d = static_cast<uint8_t*>(p);
    const size_t have = end_ - pos_;
    if (have >= n) {
      std::memcpy(d, buf_.data() + pos_, n);
      pos_ += n;
      return true;
    }
    std::memcpy(d, buf_.data() + pos_, have);
    pos_ = end_ = 0;
    d += have;
    n -= have;
    if (n >= kCap / 2) return c_.read_exact(d, n);
    while (n > 0) {
      const size_t r = c_.read_some(buf_.data(), kCap);
      if (r == 0) return false;
      const size_t take = std::min(r, n);
      std::memcpy(d, buf_.data(), take);
      d += take;
      n -= take;
      pos_ = take;
      end_ = r;
    }
    return true;
  }

 private:
  static constexpr size_t kCap = 64 << 10;
  PeerConnection& c_;
  Bytes buf_;
  size_t pos_ = 0, end_ = 0;
};
}  // namespace

void PeerRouter::run() {
  const Rank peer = conn_->peer();
  PoolScope scope(pool_.get());  // payload buffers come from the mesh's pool
  FrameReader in(*conn_);
  try {
    while (true) {
      uint8_t kind;
      if (!in.read_exact(&kind, 1)) break;
      uint64_t pre[3] = {0, 0, 0};
      int np = 0;
      switch (kind) {
        case kFrameMessage: case kFrameRaw: np = 1; break;
        case kFrameRawComm: case kFrameRawTagged: np = 2; break;
        case kFrameRawCommTagged: np = 3; break;
        default:
          NEXAR_LOG(LogLevel::Error, "unknown frame kind " + std::to_string(kind) + " from rank " + std::to_string(peer));
          goto done;
      }
      uint8_t buf[24];
      if (!in.read_exact(buf, 8 * np)) break;
      for (int i = 0; i < np; ++i) pre[i] = get_le(buf + 8 * i, 8);
      const uint64_t len = pre[np - 1];
      if (len > kMaxMessageBytes) {
        NEXAR_LOG(LogLevel::Error, "oversized frame from rank " + std::to_string(peer));
        break;
      }
      if (kind == kFrameMessage && len >= kDataPrefixBytes) {
        // Data messages (p2p send / recv) are parsed from their fixed prefix
        // and the payload is read straight into its own buffer; any other
        // message is reassembled and decoded whole.
        uint8_t head[kDataPrefixBytes];
        if (!in.read_exact(head, kDataPrefixBytes)) break;
        uint32_t tag = 0;
        Rank src = 0;
        uint64_t plen = 0;
        if (decode_data_prefix(head, len, &tag, &src, &plen)) {
          Bytes data(plen);
          if (plen && !in.read_exact(data.data(), plen)) break;
          last_seen_ns_ = now_ns();
          dispatch(Message::data(tag, src, std::move(data)));
          continue;
        }
        Bytes whole(len);
        std::memcpy(whole.data(), head, kDataPrefixBytes);
        if (!in.read_exact(whole.data() + kDataPrefixBytes, len - kDataPrefixBytes)) break;
        last_seen_ns_ = now_ns();
        Message m;
        try {
          m = decode_message(whole.data(), whole.size());
        } catch (const NexarError& e) {
          NEXAR_LOG(LogLevel::Warn, std::string("dropping undecodable message: ") + e.what());
          continue;
        }
        dispatch(std::move(m));
        continue;
      }
      Bytes payload(len);
      if (len && !in.read_exact(payload.data(), len)) break;
      last_seen_ns_ = now_ns();
      switch (kind) {
        case kFrameMessage: {
          Message m;
          try {
            m = decode_message(payload.data(), payload.size());
          } catch (const NexarError& e) {
            NEXAR_LOG(LogLevel::Warn, std::string("dropping undecodable message: ") + e.what());
            continue;
          }
          dispatch(std::move(m));
          break;
        }
        case kFrameRaw:
          box_->push(LaneKey{LaneKind::Raw, 0, 0}, Item{{}, std::move(payload)});
          break;
        case kFrameRawComm:
          box_->push(LaneKey{LaneKind::RawComm, pre[0], 0}, Item{{}, std::move(payload)});
          break;
        case kFrameRawTagged:
          box_->push(LaneKey{LaneKind::Tagged, 0, pre[0]}, Item{{}, std::move(payload)});
          break;
        case kFrameRawCommTagged:
          box_->push(LaneKey{LaneKind::Tagged, pre[0], pre[1]}, Item{{}, std::move(payload)});
          break;
      }
    }
  } catch (const std::exception& e) {
    NEXAR_LOG(LogLevel::Warn, std::string("router for rank ") + std::to_string(peer) + " stopped: " + e.what());
  }
done:
  box_->close(Err::PeerDisconnected, "peer " + std::to_string(peer) + " disconnected unexpectedly");
  conn_->close();
  if (on_disconnect_) on_disconnect_(peer);
}

}  // namespace nexar
