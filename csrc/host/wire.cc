#include "wire.h"

namespace nexar {

void Header::encode(uint8_t out[kHeaderSize]) const {
  for (int i = 0; i < 4; ++i) out[i] = (payload_length >> (8 * i)) & 0xff;
  out[4] = priority;
  out[5] = message_type;
  out[6] = 0;
  out[7] = 0;
}

bool Header::decode(const uint8_t in[kHeaderSize], Header* h) {
  if (in[5] != 0) return false;  // only Control is defined
  h->payload_length = (uint32_t)get_le(in, 4);
  h->priority = in[4];
  h->message_type = in[5];
  return true;
}

const char* msg_kind_name(MsgKind k) {
  static const char* names[] = {"Hello", "Welcome", "Barrier", "BarrierAck", "Heartbeat", "NodeJoined",
                                "NodeLeft", "Rpc", "RpcResponse", "Data", "RdmaEndpoint", "SplitRequest",
                                "RecoveryVote", "RecoveryAgreement", "ElasticCheckpoint",
                                "ElasticCheckpointAck", "Relay"};
  const unsigned i = (unsigned)k;
  return i < sizeof(names) / sizeof(names[0]) ? names[i] : "?";
}

bool Message::operator==(const Message& o) const {
  return kind == o.kind && protocol_version == o.protocol_version && capabilities == o.capabilities &&
         cluster_token == o.cluster_token && listen_addr == o.listen_addr && rank == o.rank &&
         world_size == o.world_size && peers == o.peers && ca_cert == o.ca_cert && node_cert == o.node_cert &&
         node_key == o.node_key && addr == o.addr && epoch == o.epoch && comm_id == o.comm_id &&
         dead_ranks == o.dead_ranks && joining == o.joining && leaving == o.leaving &&
         new_world_size == o.new_world_size && timestamp_ns == o.timestamp_ns && req_id == o.req_id &&
         fn_id == o.fn_id && payload == o.payload && tag == o.tag && src_rank == o.src_rank && lid == o.lid &&
         qpn == o.qpn && psn == o.psn && gid == o.gid && color == o.color && key == o.key &&
         final_dest == o.final_dest && relay_tag == o.relay_tag;
}

#define MK(K) Message m; m.kind = MsgKind::K
Message Message::hello(const Bytes& token, const std::string& la, uint64_t caps) {
  MK(Hello); m.protocol_version = kProtocolVersion; m.capabilities = caps; m.cluster_token = token;
  m.listen_addr = la; return m;
}
Message Message::welcome(Rank r, uint32_t w, const PeerList& p) { MK(Welcome); m.rank = r; m.world_size = w; m.peers = p; return m; }
Message Message::barrier(uint64_t e, uint64_t c) { MK(Barrier); m.epoch = e; m.comm_id = c; return m; }
Message Message::barrier_ack(uint64_t e, uint64_t c) { MK(BarrierAck); m.epoch = e; m.comm_id = c; return m; }
Message Message::heartbeat(uint64_t ts) { MK(Heartbeat); m.timestamp_ns = ts; return m; }
Message Message::node_joined(Rank r, const std::string& a) { MK(NodeJoined); m.rank = r; m.addr = a; return m; }
Message Message::node_left(Rank r) { MK(NodeLeft); m.rank = r; return m; }
Message Message::rpc(uint64_t id, uint16_t f, Bytes p) { MK(Rpc); m.req_id = id; m.fn_id = f; m.payload = std::move(p); return m; }
Message Message::rpc_response(uint64_t id, Bytes p) { MK(RpcResponse); m.req_id = id; m.payload = std::move(p); return m; }
Message Message::data(uint32_t t, Rank s, Bytes p) { MK(Data); m.tag = t; m.src_rank = s; m.payload = std::move(p); return m; }
Message Message::split_request(uint32_t c, uint32_t k) { MK(SplitRequest); m.color = c; m.key = k; return m; }
Message Message::recovery_vote(uint64_t e, std::vector<Rank> d) { MK(RecoveryVote); m.epoch = e; m.dead_ranks = std::move(d); return m; }
Message Message::recovery_agreement(uint64_t e, std::vector<Rank> d) { MK(RecoveryAgreement); m.epoch = e; m.dead_ranks = std::move(d); return m; }
Message Message::elastic_checkpoint(uint64_t e) { MK(ElasticCheckpoint); m.epoch = e; return m; }
Message Message::elastic_checkpoint_ack(uint64_t e, PeerList j, std::vector<Rank> l, uint32_t w) {
  MK(ElasticCheckpointAck); m.epoch = e; m.joining = std::move(j); m.leaving = std::move(l); m.new_world_size = w; return m;
}
Message Message::relay(Rank s, Rank d, uint64_t t, Bytes p) {
  MK(Relay); m.src_rank = s; m.final_dest = d; m.relay_tag = t; m.payload = std::move(p); return m;
}
#undef MK

namespace {
void put_peers(Bytes& b, const PeerList& v) {
  put_u64(b, v.size());
  for (const auto& e : v) {
    put_u32(b, e.first);
    put_str(b, e.second);
  }
}
PeerList get_peers(Reader& r) {
  uint64_t n = r.u64();
  if (n > r.remaining()) fail(Err::DecodeFailed, "peer list length exceeds message");
  PeerList v;
  v.reserve(n);
  for (uint64_t i = 0; i < n; ++i) {
    Rank rk = r.u32();
    v.emplace_back(rk, r.str());
  }
  return v;
}
void put_ranks(Bytes& b, const std::vector<Rank>& v) {
  put_u64(b, v.size());
  for (Rank x : v) put_u32(b, x);
}
std::vector<Rank> get_ranks(Reader& r) {
  uint64_t n = r.u64();
  if (n * 4 > r.remaining()) fail(Err::DecodeFailed, "rank list length exceeds message");
  std::vector<Rank> v(n);
  for (auto& x : v) x = r.u32();
  return v;
}
}  // namespace

Bytes encode_body(const Message& m) {
  Bytes b;
  b.reserve(32 + m.payload.size());
  put_u8(b, (uint8_t)m.kind);
  switch (m.kind) {
    case MsgKind::Hello:
      put_u16(b, m.protocol_version); put_u64(b, m.capabilities); put_blob(b, m.cluster_token); put_str(b, m.listen_addr);
      break;
    case MsgKind::Welcome:
      put_u32(b, m.rank); put_u32(b, m.world_size); put_peers(b, m.peers);
      put_blob(b, m.ca_cert); put_blob(b, m.node_cert); put_blob(b, m.node_key);
      break;
    case MsgKind::Barrier:
    case MsgKind::BarrierAck:
      put_u64(b, m.epoch); put_u64(b, m.comm_id);
      break;
    case MsgKind::Heartbeat: put_u64(b, m.timestamp_ns); break;
    case MsgKind::NodeJoined: put_u32(b, m.rank); put_str(b, m.addr); break;
    case MsgKind::NodeLeft: put_u32(b, m.rank); break;
    case MsgKind::Rpc: put_u64(b, m.req_id); put_u16(b, m.fn_id); put_blob(b, m.payload); break;
    case MsgKind::RpcResponse: put_u64(b, m.req_id); put_blob(b, m.payload); break;
    case MsgKind::Data: put_u32(b, m.tag); put_u32(b, m.src_rank); put_blob(b, m.payload); break;
    case MsgKind::RdmaEndpoint: put_u16(b, m.lid); put_u32(b, m.qpn); put_u32(b, m.psn); put_blob(b, m.gid); break;
    case MsgKind::SplitRequest: put_u32(b, m.color); put_u32(b, m.key); break;
    case MsgKind::RecoveryVote:
    case MsgKind::RecoveryAgreement:
      put_u64(b, m.epoch); put_ranks(b, m.dead_ranks);
      break;
    case MsgKind::ElasticCheckpoint: put_u64(b, m.epoch); break;
    case MsgKind::ElasticCheckpointAck:
      put_u64(b, m.epoch); put_peers(b, m.joining); put_ranks(b, m.leaving); put_u32(b, m.new_world_size);
      break;
    case MsgKind::Relay:
      put_u32(b, m.src_rank); put_u32(b, m.final_dest); put_u64(b, m.relay_tag); put_blob(b, m.payload);
      break;
  }
  return b;
}

Message decode_body(const uint8_t* p, size_t n) {
  Reader r(p, n);
  Message m;
  const uint8_t k = r.u8();
  if (k > (uint8_t)MsgKind::Relay) fail(Err::DecodeFailed, "unknown message variant " + std::to_string(k));
  m.kind = (MsgKind)k;
  switch (m.kind) {
    case MsgKind::Hello:
      m.protocol_version = r.u16(); m.capabilities = r.u64(); m.cluster_token = r.blob(); m.listen_addr = r.str();
      break;
    case MsgKind::Welcome:
      m.rank = r.u32(); m.world_size = r.u32(); m.peers = get_peers(r);
      m.ca_cert = r.blob(); m.node_cert = r.blob(); m.node_key = r.blob();
      break;
    case MsgKind::Barrier:
    case MsgKind::BarrierAck:
      m.epoch = r.u64(); m.comm_id = r.u64();
      break;
    case MsgKind::Heartbeat: m.timestamp_ns = r.u64(); break;
    case MsgKind::NodeJoined: m.rank = r.u32(); m.addr = r.str(); break;
    case MsgKind::NodeLeft: m.rank = r.u32(); break;
    case MsgKind::Rpc: m.req_id = r.u64(); m.fn_id = r.u16(); m.payload = r.blob(); break;
    case MsgKind::RpcResponse: m.req_id = r.u64(); m.payload = r.blob(); break;
    case MsgKind::Data: m.tag = r.u32(); m.src_rank = r.u32(); m.payload = r.blob(); break;
    case MsgKind::RdmaEndpoint: m.lid = r.u16(); m.qpn = r.u32(); m.psn = r.u32(); m.gid = r.blob(); break;
    case MsgKind::SplitRequest: m.color = r.u32(); m.key = r.u32(); break;
    case MsgKind::RecoveryVote:
    case MsgKind::RecoveryAgreement:
      m.epoch = r.u64(); m.dead_ranks = get_ranks(r);
      break;
    case MsgKind::ElasticCheckpoint: m.epoch = r.u64(); break;
    case MsgKind::ElasticCheckpointAck:
      m.epoch = r.u64(); m.joining = get_peers(r); m.leaving = get_ranks(r); m.new_world_size = r.u32();
      break;
    case MsgKind::Relay:
      m.src_rank = r.u32(); m.final_dest = r.u32(); m.relay_tag = r.u64(); m.payload = r.blob();
      break;
  }
  if (!r.done()) fail(Err::DecodeFailed, "trailing bytes after message body");
  return m;
}

Bytes encode_message(const Message& m, Priority prio) {
  Bytes body = encode_body(m);
  if (body.size() > 0xffffffffull) fail(Err::EncodeFailed, "message body exceeds u32::MAX bytes");
  Header h;
  h.payload_length = (uint32_t)body.size();
  h.priority = (uint8_t)prio;
  Bytes out(kHeaderSize);
  h.encode(out.data());
  out.insert(out.end(), body.begin(), body.end());
  return out;
}

size_t encode_data_prefix(uint32_t tag, Rank src, uint64_t payload_len, Priority prio, uint8_t* out) {
  Header h;
  h.payload_length = (uint32_t)(kDataPrefixBytes - kHeaderSize + payload_len);
  h.priority = (uint8_t)prio;
  h.encode(out);
  size_t o = kHeaderSize;
  out[o++] = (uint8_t)MsgKind::Data;
  for (int i = 0; i < 4; ++i) out[o++] = (tag >> (8 * i)) & 0xff;
  for (int i = 0; i < 4; ++i) out[o++] = (src >> (8 * i)) & 0xff;
  for (int i = 0; i < 8; ++i) out[o++] = (payload_len >> (8 * i)) & 0xff;
  return o;
}

bool decode_data_prefix(const uint8_t* p, uint64_t msg_len, uint32_t* tag, Rank* src, uint64_t* payload_len) {
  Header h;
  if (!Header::decode(p, &h)) return false;
  if (p[kHeaderSize] != (uint8_t)MsgKind::Data) return false;
  const uint64_t plen = get_le(p + kHeaderSize + 9, 8);
  if ((uint64_t)h.payload_length + kHeaderSize != msg_len || plen + kDataPrefixBytes != msg_len) return false;
  *tag = (uint32_t)get_le(p + kHeaderSize + 1, 4);
  *src = (Rank)get_le(p + kHeaderSize + 5, 4);
  *payload_len = plen;
  return true;
}

Message decode_message(const uint8_t* p, size_t n) {
  if (n < kHeaderSize) fail(Err::DecodeFailed, "buffer shorter than the 8-byte header");
  Header h;
  if (!Header::decode(p, &h)) fail(Err::DecodeFailed, "unknown message type in header");
  if ((uint64_t)h.payload_length + kHeaderSize != n)
    fail(Err::DecodeFailed, "header length " + std::to_string(h.payload_length) + " does not match buffer " +
                                std::to_string(n - kHeaderSize));
  return decode_body(p + kHeaderSize, h.payload_length);
}

}  // namespace nexar
