// Wire protocol: 8-byte frame header and the control-message union.
//
// Header layout follows nexar/src/protocol/header.rs:21-48:
//   [0..4) payload length u32 LE, [4] priority, [5] message type (0 = Control),
//   [6..8) reserved (zero).
// The message set follows nexar/src/protocol/message.rs:9-114 (17 variants).
// The reference serialises with rkyv; this runtime uses its own explicit
// little-endian encoding ([variant u8] then the fields in declaration order,
// vectors and strings as [len u64][bytes]), which needs no schema library.
#pragma once
#include <string>
#include <utility>
#include <vector>

#include "common.h"

namespace nexar {

constexpr size_t kHeaderSize = 8;
constexpr uint64_t kMaxMessageBytes = 4ull << 30;  // nexar/src/transport/router.rs:20

struct Header {
  uint32_t payload_length = 0;
  uint8_t priority = 0;
  uint8_t message_type = 0;  // 0 = Control
  void encode(uint8_t out[kHeaderSize]) const;
  static bool decode(const uint8_t in[kHeaderSize], Header* h);
};

enum class MsgKind : uint8_t {
  Hello = 0, Welcome = 1, Barrier = 2, BarrierAck = 3, Heartbeat = 4, NodeJoined = 5,
  NodeLeft = 6, Rpc = 7, RpcResponse = 8, Data = 9, RdmaEndpoint = 10, SplitRequest = 11,
  RecoveryVote = 12, RecoveryAgreement = 13, ElasticCheckpoint = 14, ElasticCheckpointAck = 15,
  Relay = 16,
};
const char* msg_kind_name(MsgKind k);

using PeerList = std::vector<std::pair<Rank, std::string>>;

struct Message {
  MsgKind kind = MsgKind::Heartbeat;
  // Hello
  uint16_t protocol_version = 0;
  uint64_t capabilities = 0;
  Bytes cluster_token;
  std::string listen_addr;
  // Welcome / NodeJoined / NodeLeft
  Rank rank = 0;
  uint32_t world_size = 0;
  PeerList peers;
  Bytes ca_cert, node_cert, node_key;
  std::string addr;
  // Barrier / BarrierAck / Recovery* / Elastic*
  uint64_t epoch = 0;
  uint64_t comm_id = 0;
  std::vector<Rank> dead_ranks;
  PeerList joining;
  std::vector<Rank> leaving;
  uint32_t new_world_size = 0;
  // Heartbeat
  uint64_t timestamp_ns = 0;
  // Rpc / RpcResponse
  uint64_t req_id = 0;
  uint16_t fn_id = 0;
  Bytes payload;
  // Data
  uint32_t tag = 0;
  Rank src_rank = 0;
  // RdmaEndpoint
  uint16_t lid = 0;
  uint32_t qpn = 0, psn = 0;
  Bytes gid;
  // SplitRequest
  uint32_t color = 0, key = 0;
  // Relay
  Rank final_dest = 0;
  uint64_t relay_tag = 0;

  bool operator==(const Message& o) const;

  static Message hello(const Bytes& token, const std::string& listen_addr, uint64_t caps = 0);
  static Message welcome(Rank rank, uint32_t world, const PeerList& peers);
  static Message barrier(uint64_t epoch, uint64_t comm_id);
  static Message barrier_ack(uint64_t epoch, uint64_t comm_id);
  static Message heartbeat(uint64_t ts_ns);
  static Message node_joined(Rank r, const std::string& addr);
  static Message node_left(Rank r);
  static Message rpc(uint64_t req_id, uint16_t fn_id, Bytes payload);
  static Message rpc_response(uint64_t req_id, Bytes payload);
  static Message data(uint32_t tag, Rank src, Bytes payload);
  static Message split_request(uint32_t color, uint32_t key);
  static Message recovery_vote(uint64_t epoch, std::vector<Rank> dead);
  static Message recovery_agreement(uint64_t epoch, std::vector<Rank> dead);
  static Message elastic_checkpoint(uint64_t epoch);
  static Message elastic_checkpoint_ack(uint64_t epoch, PeerList joining, std::vector<Rank> leaving,
                                        uint32_t new_world);
  static Message relay(Rank src, Rank final_dest, uint64_t tag, Bytes payload);
};

// Body only (no header).
Bytes encode_body(const Message& m);
Message decode_body(const uint8_t* p, size_t n);
// Header + body; throws EncodeFailed above the 4 GiB limit.
Bytes encode_message(const Message& m, Priority prio);
// Parse header + body from one contiguous buffer (length checked).
Message decode_message(const uint8_t* p, size_t n);

// The fixed part of an encoded Data message ahead of its payload: the 8-byte
// header, the variant byte, tag (u32), source rank (u32) and the payload's
// blob length (u64). Data messages are written and parsed in two pieces (this
// prefix, then the payload in place) so a p2p payload is never copied into or
// out of an encode buffer; the bytes are those encode_message produces.
constexpr size_t kDataPrefixBytes = kHeaderSize + 1 + 4 + 4 + 8;
size_t encode_data_prefix(uint32_t tag, Rank src, uint64_t payload_len, Priority prio, uint8_t* out);
// True if `p` (kDataPrefixBytes long) starts a well-formed Data message whose
// encoding is `msg_len` bytes in total; fills tag, source and payload length.
bool decode_data_prefix(const uint8_t* p, uint64_t msg_len, uint32_t* tag, Rank* src, uint64_t* payload_len);

}  // namespace nexar
