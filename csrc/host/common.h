// Base layer of the host runtime: wire enums, errors, configuration, logging.
//
// DataType / ReduceOp / Priority keep the reference's codes
// (nexar/src/types.rs:13-98). NexarError keeps the reference's variant set
// (nexar/src/error.rs:6-105) as numeric codes. Config keeps the reference's
// fields, defaults and NEXAR_* environment names (nexar/src/config.rs:12-228).
#pragma once

#include <chrono>
#include <cstdint>
#include <cstring>
#include <functional>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace nexar {

using Rank = uint32_t;

// Allocator that leaves bytes uninitialised on value-less construction:
// `Bytes b(n)` / `b.resize(n)` do not zero-fill (receive buffers are written
// in full by the socket read; zeroing a 16 MB payload costs as much as a
// tenth of its transfer). `Bytes b(n, 0)` / `assign(n, 0)` still zero.
// Storage comes from pool_allocate (buffer_pool.cc): a thread inside a
// PoolScope (the receive routers) draws buffers of 16 KiB and more from its
// BufferPool's tiers, and they return to their tier when freed on any thread.
void* pool_allocate(size_t bytes);
void pool_deallocate(void* p) noexcept;
template <class T>
struct NoInitAllocator : std::allocator<T> {
  using value_type = T;
  template <class U> struct rebind { using other = NoInitAllocator<U>; };
  NoInitAllocator() noexcept = default;
  template <class U> NoInitAllocator(const NoInitAllocator<U>&) noexcept {}
  T* allocate(size_t n) { return static_cast<T*>(pool_allocate(n * sizeof(T))); }
  void deallocate(T* p, size_t) noexcept { pool_deallocate(p); }
  template <class U> void construct(U* p) noexcept { ::new (static_cast<void*>(p)) U; }
  template <class U, class... A> void construct(U* p, A&&... a) { ::new (static_cast<void*>(p)) U(std::forward<A>(a)...); }
};
template <class T, class U>
bool operator==(const NoInitAllocator<T>&, const NoInitAllocator<U>&) noexcept { return true; }
template <class T, class U>
bool operator!=(const NoInitAllocator<T>&, const NoInitAllocator<U>&) noexcept { return false; }

using Bytes = std::vector<uint8_t, NoInitAllocator<uint8_t>>;
using Clock = std::chrono::steady_clock;

constexpr uint16_t kProtocolVersion = 1;

enum class DataType : uint8_t {
  F32 = 0, F64 = 1, F16 = 2, BF16 = 3, I8 = 4, I32 = 5, I64 = 6, U8 = 7, U32 = 8, U64 = 9,
  F8E4M3 = 10, F8E5M2 = 11,
};
inline size_t dtype_size(DataType d) {
  switch (d) {
    case DataType::F32: case DataType::I32: case DataType::U32: return 4;
    case DataType::F64: case DataType::I64: case DataType::U64: return 8;
    case DataType::F16: case DataType::BF16: return 2;
    default: return 1;
  }
}
const char* dtype_name(DataType d);

enum class ReduceOp : uint8_t { Sum = 0, Prod = 1, Min = 2, Max = 3 };
const char* op_name(ReduceOp op);

enum class Priority : uint8_t { Critical = 0, Realtime = 1, Bulk = 2 };

// ------------------------------------------------------------------ errors
enum class Err : int {
  Ok = 0, ConnectionFailed = 1, PeerDisconnected = 2, UnknownPeer = 3, ProtocolMismatch = 4,
  DecodeFailed = 5, EncodeFailed = 6, BarrierTimeout = 7, ClusterFormationTimeout = 8,
  UnsupportedDType = 9, BufferSizeMismatch = 10, InvalidRank = 11, Transport = 12, Tls = 13,
  Io = 14, RpcNotRegistered = 15, RpcFailed = 16, DeviceError = 17, CollectiveFailed = 18,
  Cancelled = 19, ClusterTokenMismatch = 20, IndivisibleCount = 21, LockPoisoned = 22,
  Recovery = 23, ElasticTimeout = 24, Elastic = 25, Timeout = 26,
};

class NexarError : public std::runtime_error {
 public:
  NexarError(Err code, const std::string& msg) : std::runtime_error(msg), code_(code) {}
  Err code() const { return code_; }
 private:
  Err code_;
};

[[noreturn]] inline void fail(Err code, const std::string& msg) { throw NexarError(code, msg); }
NexarError collective_failed(const std::string& op, Rank rank, const std::string& reason);

// ------------------------------------------------------------------ config
enum class RecoveryPolicy : uint8_t { Automatic = 0, Manual = 1, Abort = 2 };

enum class TopologyKind : uint8_t { FullMesh = 0, KRegular = 1, Hypercube = 2 };
struct TopologyStrategy {
  TopologyKind kind = TopologyKind::FullMesh;
  uint32_t degree = 0;  // KRegular only
  bool is_sparse() const { return kind != TopologyKind::FullMesh; }
  std::string to_string() const;
};
// "full_mesh" | "k_regular:N" | "hypercube" (nexar/src/cluster/sparse.rs parse_topology)
TopologyStrategy parse_topology(const std::string& s);

struct Config {
  TopologyStrategy topology;
  double collective_timeout_s = 30.0;
  double barrier_timeout_s = 30.0;
  double rpc_timeout_s = 30.0;
  uint64_t large_msg_bytes = 8ull << 20;
  // All-reduces up to this size use recursive doubling (log2 N exchanges of
  // the whole buffer) instead of the ring's 2(N-1) steps (new; 0 disables).
  uint64_t small_msg_bytes = 256ull << 10;
  uint64_t pipeline_segment_bytes = 2ull << 20;
  uint32_t ring_max_world = 8;
  bool enable_tcp_bulk_sidecar = true;
  bool encrypt_bulk_transport = true;
  // TLS 1.3 with a per-cluster CA on every host link (bootstrap and mesh).
  // Off by default: the default deployment is one box over loopback.
  bool tls = false;
  uint64_t compressed_allreduce_max_bytes = 4ull << 30;
  double heartbeat_interval_s = 1.0;
  double heartbeat_timeout_s = 5.0;
  double recovery_timeout_s = 30.0;
  bool elastic_enabled = false;
  uint32_t elastic_min_world_size = 1;
  uint32_t elastic_max_world_size = 0;
  double elastic_checkpoint_timeout_s = 60.0;
  RecoveryPolicy recovery_policy = RecoveryPolicy::Automatic;
  // Device knobs (new; consumed by the CUDA runtime through the Python layer).
  uint64_t ar_oneshot_max = 256ull << 10;
  uint64_t device_wait_timeout_us = 10'000'000;

  static Config from_env();
};

// ------------------------------------------------------------------ logging
enum class LogLevel : int { Error = 0, Warn = 1, Info = 2, Debug = 3 };
LogLevel log_level();
void log_msg(LogLevel lvl, const std::string& msg);
#define NEXAR_LOG(lvl, expr)                                          \
  do {                                                                \
    if ((int)(lvl) <= (int)::nexar::log_level()) {                    \
      ::nexar::log_msg((lvl), (expr));                                \
    }                                                                 \
  } while (0)

// ------------------------------------------------------------------ little-endian helpers
inline void put_u8(Bytes& b, uint8_t v) { b.push_back(v); }
inline void put_u16(Bytes& b, uint16_t v) { for (int i = 0; i < 2; ++i) b.push_back((v >> (8 * i)) & 0xff); }
inline void put_u32(Bytes& b, uint32_t v) { for (int i = 0; i < 4; ++i) b.push_back((v >> (8 * i)) & 0xff); }
inline void put_u64(Bytes& b, uint64_t v) { for (int i = 0; i < 8; ++i) b.push_back((v >> (8 * i)) & 0xff); }
inline void put_bytes(Bytes& b, const uint8_t* p, size_t n) { b.insert(b.end(), p, p + n); }
inline void put_blob(Bytes& b, const Bytes& v) { put_u64(b, v.size()); put_bytes(b, v.data(), v.size()); }
inline void put_str(Bytes& b, const std::string& s) {
  put_u64(b, s.size());
  put_bytes(b, reinterpret_cast<const uint8_t*>(s.data()), s.size());
}
inline uint64_t get_le(const uint8_t* p, int n) {
  uint64_t v = 0;
  for (int i = 0; i < n; ++i) v |= (uint64_t)p[i] << (8 * i);
  return v;
}

class Reader {
 public:
  Reader(const uint8_t* p, size_t n) : p_(p), n_(n) {}
  explicit Reader(const Bytes& b) : p_(b.data()), n_(b.size()) {}
  uint8_t u8() { need(1); return p_[off_++]; }
  uint16_t u16() { need(2); uint16_t v = (uint16_t)get_le(p_ + off_, 2); off_ += 2; return v; }
  uint32_t u32() { need(4); uint32_t v = (uint32_t)get_le(p_ + off_, 4); off_ += 4; return v; }
  uint64_t u64() { need(8); uint64_t v = get_le(p_ + off_, 8); off_ += 8; return v; }
  Bytes blob() {
    uint64_t n = u64();
    need(n);
    Bytes v(p_ + off_, p_ + off_ + n);
    off_ += n;
    return v;
  }
  std::string str() {
    uint64_t n = u64();
    need(n);
    std::string s(reinterpret_cast<const char*>(p_ + off_), n);
    off_ += n;
    return s;
  }
  size_t remaining() const { return n_ - off_; }
  bool done() const { return off_ == n_; }

 private:
  void need(uint64_t k) {
    if (k > n_ - off_) fail(Err::DecodeFailed, "truncated message: need " + std::to_string(k) +
                                                   " bytes, have " + std::to_string(n_ - off_));
  }
  const uint8_t* p_;
  size_t n_;
  size_t off_ = 0;
};

// FNV-1a 64 over byte parts; never returns 0 (reserved for the root
// communicator). Same constants as nexar/src/client/hash.rs:6-20.
uint64_t fnv1a_comm_id(const std::vector<Bytes>& parts);

inline double seconds_since(Clock::time_point t0) {
  return std::chrono::duration<double>(Clock::now() - t0).count();
}

}  // namespace nexar
