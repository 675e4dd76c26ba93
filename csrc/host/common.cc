#include "common.h"

#include <cstdio>
#include <cstdlib>
#include <mutex>

namespace nexar {

const char* dtype_name(DataType d) {
  switch (d) {
    case DataType::F32: return "f32";
    case DataType::F64: return "f64";
    case DataType::F16: return "f16";
    case DataType::BF16: return "bf16";
    case DataType::I8: return "i8";
    case DataType::I32: return "i32";
    case DataType::I64: return "i64";
    case DataType::U8: return "u8";
    case DataType::U32: return "u32";
    case DataType::U64: return "u64";
    case DataType::F8E4M3: return "f8e4m3";
    case DataType::F8E5M2: return "f8e5m2";
  }
  return "?";
}

const char* op_name(ReduceOp op) {
  switch (op) {
    case ReduceOp::Sum: return "sum";
    case ReduceOp::Prod: return "prod";
    case ReduceOp::Min: return "min";
    case ReduceOp::Max: return "max";
  }
  return "?";
}

NexarError collective_failed(const std::string& op, Rank rank, const std::string& reason) {
  return NexarError(Err::CollectiveFailed, op + " failed at rank " + std::to_string(rank) + ": " + reason);
}

std::string TopologyStrategy::to_string() const {
  switch (kind) {
    case TopologyKind::FullMesh: return "full_mesh";
    case TopologyKind::KRegular: return "k_regular:" + std::to_string(degree);
    case TopologyKind::Hypercube: return "hypercube";
  }
  return "?";
}

TopologyStrategy parse_topology(const std::string& s) {
  TopologyStrategy t;
  if (s == "full_mesh" || s.empty()) return t;
  if (s == "hypercube") {
    t.kind = TopologyKind::Hypercube;
    return t;
  }
  const std::string pfx = "k_regular:";
  if (s.compare(0, pfx.size(), pfx) == 0) {
    char* end = nullptr;
    unsigned long d = std::strtoul(s.c_str() + pfx.size(), &end, 10);
    if (end && *end == 0 && d > 0) {
      t.kind = TopologyKind::KRegular;
      t.degree = (uint32_t)d;
      return t;
    }
  }
  fail(Err::Elastic, "invalid topology string: '" + s + "'");
}

namespace {
const char* env(const char* k) {
  const char* v = std::getenv(k);
  return (v && *v) ? v : nullptr;
}
double env_f(const char* k, double d) {
  const char* v = env(k);
  return v ? std::atof(v) : d;
}
uint64_t env_u(const char* k, uint64_t d) {
  const char* v = env(k);
  return v ? std::strtoull(v, nullptr, 10) : d;
}
bool env_b(const char* k, bool d) {
  const char* v = env(k);
  if (!v) return d;
  std::string s(v);
  return s == "1" || s == "true" || s == "TRUE" || s == "yes";
}
}  // namespace

Config Config::from_env() {
  Config c;
  c.collective_timeout_s = env_f("NEXAR_COLLECTIVE_TIMEOUT_SECS", c.collective_timeout_s);
  c.barrier_timeout_s = env_f("NEXAR_BARRIER_TIMEOUT_SECS", c.barrier_timeout_s);
  c.rpc_timeout_s = env_f("NEXAR_RPC_TIMEOUT_SECS", c.rpc_timeout_s);
  c.large_msg_bytes = env_u("NEXAR_LARGE_MSG_BYTES", c.large_msg_bytes);
  c.small_msg_bytes = env_u("NEXAR_SMALL_MSG_BYTES", c.small_msg_bytes);
  c.pipeline_segment_bytes = env_u("NEXAR_PIPELINE_SEGMENT_BYTES", c.pipeline_segment_bytes);
  c.ring_max_world = (uint32_t)env_u("NEXAR_RING_MAX_WORLD", c.ring_max_world);
  c.enable_tcp_bulk_sidecar = env_b("NEXAR_ENABLE_TCP_BULK_SIDECAR", c.enable_tcp_bulk_sidecar);
  c.tls = env_b("NEXAR_TLS", c.tls);
  c.encrypt_bulk_transport = env_b("NEXAR_ENCRYPT_BULK_TRANSPORT", c.encrypt_bulk_transport);
  c.compressed_allreduce_max_bytes = env_u("NEXAR_COMPRESSED_ALLREDUCE_MAX_BYTES", c.compressed_allreduce_max_bytes);
  c.heartbeat_interval_s = env_f("NEXAR_HEARTBEAT_INTERVAL_SECS", c.heartbeat_interval_s);
  c.heartbeat_timeout_s = env_f("NEXAR_HEARTBEAT_TIMEOUT_SECS", c.heartbeat_timeout_s);
  c.recovery_timeout_s = env_f("NEXAR_RECOVERY_TIMEOUT_SECS", c.recovery_timeout_s);
  if (const char* t = env("NEXAR_TOPOLOGY")) c.topology = parse_topology(t);
  c.elastic_enabled = env_b("NEXAR_ELASTIC_ENABLED", c.elastic_enabled);
  c.elastic_min_world_size = (uint32_t)env_u("NEXAR_ELASTIC_MIN_WORLD_SIZE", c.elastic_min_world_size);
  c.elastic_max_world_size = (uint32_t)env_u("NEXAR_ELASTIC_MAX_WORLD_SIZE", c.elastic_max_world_size);
  c.elastic_checkpoint_timeout_s = env_f("NEXAR_ELASTIC_CHECKPOINT_TIMEOUT_SECS", c.elastic_checkpoint_timeout_s);
  if (const char* p = env("NEXAR_RECOVERY_POLICY")) {
    std::string s(p);
    if (s == "manual") c.recovery_policy = RecoveryPolicy::Manual;
    else if (s == "abort") c.recovery_policy = RecoveryPolicy::Abort;
    else c.recovery_policy = RecoveryPolicy::Automatic;
  }
  c.ar_oneshot_max = env_u("NEXAR_AR_ONESHOT_MAX", c.ar_oneshot_max);
  c.device_wait_timeout_us = env_u("NEXAR_DEVICE_WAIT_TIMEOUT_US", c.device_wait_timeout_us);
  return c;
}

LogLevel log_level() {
  static LogLevel lvl = [] {
    const char* v = std::getenv("NEXAR_LOG_LEVEL");
    if (!v) return LogLevel::Warn;
    std::string s(v);
    if (s == "error") return LogLevel::Error;
    if (s == "info") return LogLevel::Info;
    if (s == "debug") return LogLevel::Debug;
    return LogLevel::Warn;
  }();
  return lvl;
}

void log_msg(LogLevel lvl, const std::string& msg) {
  static std::mutex mu;
  static const char* names[] = {"ERROR", "WARN", "INFO", "DEBUG"};
  std::lock_guard<std::mutex> g(mu);
  std::fprintf(stderr, "[nexar %s] %s\n", names[(int)lvl], msg.c_str());
}

uint64_t fnv1a_comm_id(const std::vector<Bytes>& parts) {
  uint64_t h = 0xcbf29ce484222325ull;
  for (const auto& p : parts)
    for (uint8_t b : p) {
      h ^= b;
      h *= 0x100000001b3ull;
    }
  return h == 0 ? 1 : h;
}

}  // namespace nexar
