// Host collective algorithms over the TCP mesh (the CPU data path and the
// oracle the device kernels are tested against).
//
// Algorithms follow nexar/src/collective/*.rs: ring / recursive
// halving-doubling / pipelined ring all-reduce (dispatch at
// allreduce.rs:21-55), RS+AG all-reduce, bucketed and compressed all-reduce,
// ring all-gather and reduce-scatter, flat / binary-tree / BFS-tree broadcast,
// binomial reduce, pairwise all-to-all, flat gather / scatter, Hillis-Steele
// scan and two-phase / dissemination barrier. Every step uses its own tag
// (step_tag(t, s) = t*1000 + s, helpers.rs:76-78) on the communicator's
// tagged lanes.
//
// Differences: reduce_scatter leaves chunk r on rank r (the reference's ring
// leaves chunk (r+1) mod N, reduce_scatter.rs:73-77); the pipelined ring
// overlaps the reduction of segment k with the transfer of segment k+1
// (the reference runs them back to back, pipelined_allreduce.rs:142-176); the
// compressed all-reduce zeroes its dense buffer for every peer (the reference
// reuses it unzeroed, compressed_allreduce.rs:90,105).
#include <algorithm>
#include <future>

#include "client.h"

namespace nexar {
namespace coll {

size_t ceil_log2(uint32_t n) {
  if (n <= 1) return 0;
  return 32 - __builtin_clz(n - 1);
}

uint64_t step_tag(uint64_t base, uint64_t step) { return base * 1000ull + step; }

ChunkLayout::ChunkLayout(size_t count, uint32_t world) : base(count / world), remainder(count % world) {
  offsets.resize(world);
  size_t off = 0;
  for (uint32_t i = 0; i < world; ++i) {
    offsets[i] = off;
    off += chunk(i);
  }
}

static void check_len(const Bytes& b, size_t expect, const char* op, Rank src) {
  if (b.size() != expect)
    throw collective_failed(op, src, "buffer size mismatch: expected " + std::to_string(expect) + " bytes, got " +
                                         std::to_string(b.size()));
}

// Segment tags of the pipelined ring collectives: [63:48] outer & 0xFFFF,
// [47:32] step, [31:16] segment, [15:0] phase (the pipelined all-reduce's
// packing, nexar/src/collective/pipelined_allreduce.rs:27-29; reduce-scatter
// uses phase 2, all-gather phase 3).
static uint64_t seg_tag(uint64_t tag, uint64_t step, uint64_t seg, uint64_t phase) {
  return ((tag & 0xffffull) << 48) | ((step & 0xffffull) << 32) | ((seg & 0xffffull) << 16) | (phase & 0xffffull);
}

// ------------------------------------------------------------------ all-reduce
void ring_allreduce(NexarClient& c, uint8_t* buf, size_t count, DataType dt, ReduceOp op, uint64_t tag) {
  const uint32_t N = c.world_size();
  if (N <= 1 || count == 0) return;
  const Rank r = c.rank();
  const size_t es = dtype_size(dt);
  ChunkLayout L(count, N);
  const Rank next = (r + 1) % N, prev = (r + N - 1) % N;
  uint64_t step = 0;
  // reduce-scatter phase: after it, chunk (r+1) mod N is complete on rank r
  for (uint32_t s = 0; s + 1 < N; ++s, ++step) {
    const uint32_t send_c = (r + N - s) % N, recv_c = (r + N - s - 1) % N;
    c.coll_send(next, step_tag(tag, step), buf + L.offset(send_c) * es, L.chunk(send_c) * es, "allreduce");
    Bytes in = c.coll_recv(prev, step_tag(tag, step), "allreduce");
    check_len(in, L.chunk(recv_c) * es, "allreduce", prev);
    reduce_slice(buf + L.offset(recv_c) * es, in.data(), L.chunk(recv_c), dt, op);
  }
  // all-gather phase
  for (uint32_t s = 0; s + 1 < N; ++s, ++step) {
    const uint32_t send_c = (r + 1 + N - s) % N, recv_c = (r + N - s) % N;
    c.coll_send(next, step_tag(tag, step), buf + L.offset(send_c) * es, L.chunk(send_c) * es, "allreduce");
    Bytes in = c.coll_recv(prev, step_tag(tag, step), "allreduce");
    check_len(in, L.chunk(recv_c) * es, "allreduce", prev);
    std::memcpy(buf + L.offset(recv_c) * es, in.data(), in.size());
  }
}

void halving_doubling_allreduce(NexarClient& c, uint8_t* buf, size_t count, DataType dt, ReduceOp op, uint64_t tag) {
  const uint32_t N = c.world_size();
  if (N <= 1 || count == 0) return;
  const Rank r = c.rank();
  const size_t es = dtype_size(dt);
  uint32_t p2 = 1;
  while (p2 * 2 <= N) p2 *= 2;
  const uint32_t excess = N - p2;
  size_t step = 0;
  bool active = true;
  // fold the excess ranks into the power-of-two group
  if (r < excess) {
    Bytes in = c.coll_recv(r + p2, step_tag(tag, step), "allreduce");
    check_len(in, count * es, "allreduce", r + p2);
    reduce_slice(buf, in.data(), count, dt, op);
  } else if (r >= p2) {
    c.coll_send(r - p2, step_tag(tag, step), buf, count * es, "allreduce");
    active = false;
  }
  ++step;
  const uint32_t log2 = (uint32_t)__builtin_ctz(p2);
  if (active) {
    size_t start = 0, len = count;
    std::vector<std::pair<size_t, size_t>> hist;
    for (uint32_t round = 0; round < log2; ++round) {
      const Rank partner = r ^ (1u << round);
      const size_t half = len / 2, rem = len - half;
      size_t send_s, send_l, keep_s, keep_l;
      if (r < partner) {
        send_s = start + half; send_l = rem; keep_s = start; keep_l = half;
      } else {
        send_s = start; send_l = half; keep_s = start + half; keep_l = rem;
      }
      const uint64_t t = step_tag(tag, step + round);
      c.coll_send(partner, t, buf + send_s * es, send_l * es, "allreduce");
      Bytes in = c.coll_recv(partner, t, "allreduce");
      check_len(in, keep_l * es, "allreduce", partner);
      reduce_slice(buf + keep_s * es, in.data(), keep_l, dt, op);
      hist.emplace_back(start, len);
      start = keep_s;
      len = keep_l;
    }
    const size_t ag_base = step + log2;
    for (int round = (int)log2 - 1; round >= 0; --round) {
      const Rank partner = r ^ (1u << round);
      const uint64_t t = step_tag(tag, ag_base + (log2 - 1 - round));
      c.coll_send(partner, t, buf + start * es, len * es, "allreduce");
      Bytes in = c.coll_recv(partner, t, "allreduce");
      const size_t rl = in.size() / es;
      if (r < partner) {
        std::memcpy(buf + (start + len) * es, in.data(), in.size());
      } else {
        start -= rl;
        std::memcpy(buf + start * es, in.data(), in.size());
      }
      len += rl;
      (void)hist;
    }
  }
  // unfold: the power-of-two partners return the result
  const uint64_t t_out = step_tag(tag, 999);
  if (r < excess) {
    c.coll_send(r + p2, t_out, buf, count * es, "allreduce");
  } else if (r >= p2) {
    Bytes in = c.coll_recv(r - p2, t_out, "allreduce");
    check_len(in, count * es, "allreduce", r - p2);
    std::memcpy(buf, in.data(), in.size());
  }
}

// Latency-optimal all-reduce for small messages: log2(p) exchanges of the
// whole buffer with rank ^ 2^k (recursive doubling), against 2(N-1) steps of
// the ring. Ranks beyond the largest power of two fold their buffer into a
// partner first and receive the result last. Each pair computes
// mine op theirs on both sides; IEEE add, mul, min and max are commutative, so
// every rank ends with the same bits.
void recursive_doubling_allreduce(NexarClient& c, uint8_t* buf, size_t count, DataType dt, ReduceOp op,
                                  uint64_t tag) {
  const uint32_t N = c.world_size();
  if (N <= 1 || count == 0) return;
  const Rank r = c.rank();
  const size_t nb = count * dtype_size(dt);
  uint32_t p2 = 1;
  while (p2 * 2 <= N) p2 *= 2;
  const uint32_t excess = N - p2;
  if (r < excess) {
    Bytes in = c.coll_recv(r + p2, step_tag(tag, 0), "allreduce");
    check_len(in, nb, "allreduce", r + p2);
    reduce_slice(buf, in.data(), count, dt, op);
  } else if (r >= p2) {
    c.coll_send(r - p2, step_tag(tag, 0), buf, nb, "allreduce");
  }
  if (r < p2) {
    const uint32_t log2 = (uint32_t)__builtin_ctz(p2);
    for (uint32_t round = 0; round < log2; ++round) {
      const Rank partner = r ^ (1u << round);
      const uint64_t t = step_tag(tag, 1 + round);
      c.coll_send(partner, t, buf, nb, "allreduce");
      Bytes in = c.coll_recv(partner, t, "allreduce");
      check_len(in, nb, "allreduce", partner);
      reduce_slice(buf, in.data(), count, dt, op);
    }
  }
  const uint64_t t_out = step_tag(tag, 999);
  if (r < excess) {
    c.coll_send(r + p2, t_out, buf, nb, "allreduce");
  } else if (r >= p2) {
    Bytes in = c.coll_recv(r - p2, t_out, "allreduce");
    check_len(in, nb, "allreduce", r - p2);
    std::memcpy(buf, in.data(), nb);
  }
}

// Large all-reduce: the ring's 2(N-1) steps (N-1 reduce-scatter steps, then
// N-1 all-gather steps over the same ChunkLayout) run as one pipeline of
// segments. The chunk received at stage t is the chunk sent at stage t+1, so
// each received segment is reduced (or stored) in place and forwarded at once:
// the last reduce-scatter stage feeds the first all-gather stage directly.
// Every chunk is reduced along the ring in the same order as the unpipelined
// ring and then copied, so all ranks end with the same bits. Segment tags use
// the reference's packing (nexar/src/collective/pipelined_allreduce.rs:27-29)
// with the stage in the low field.
void pipelined_ring_allreduce(NexarClient& c, uint8_t* buf, size_t count, DataType dt, ReduceOp op, uint64_t tag) {
  const uint32_t N = c.world_size();
  if (N <= 1 || count == 0) return;
  const Rank r = c.rank();
  const size_t es = dtype_size(dt);
  const size_t seg = std::max<size_t>(1, c.config().pipeline_segment_bytes / es);
  ChunkLayout L(count, N);
  const Rank next = (r + 1) % N, prev = (r + N - 1) % N;
  const uint32_t stages = 2 * (N - 1);
  auto recv_chunk = [&](uint32_t t) -> uint32_t {
    return t < N - 1 ? (r + 2 * N - t - 1) % N : (r + 2 * N - (t - (N - 1))) % N;
  };
  auto send_segments = [&](uint32_t t, uint32_t chunk) {
    const size_t len = L.chunk(chunk);
    for (size_t k = 0, off = 0; off < len; ++k, off += seg)
      c.coll_send(next, seg_tag(tag, 0, k, t), buf + (L.offset(chunk) + off) * es, std::min(seg, len - off) * es,
                  "allreduce");
  };
  send_segments(0, r);
  for (uint32_t t = 0; t < stages; ++t) {
    const uint32_t rc = recv_chunk(t);
    const size_t len = L.chunk(rc);
    for (size_t k = 0, off = 0; off < len; ++k, off += seg) {
      const size_t m = std::min(seg, len - off);
      Bytes in = c.coll_recv(prev, seg_tag(tag, 0, k, t), "allreduce");
      check_len(in, m * es, "allreduce", prev);
      uint8_t* dst = buf + (L.offset(rc) + off) * es;
      if (t < N - 1) reduce_slice(dst, in.data(), m, dt, op);
      else std::memcpy(dst, in.data(), m * es);
      if (t + 1 < stages) c.coll_send(next, seg_tag(tag, 0, k, t + 1), dst, m * es, "allreduce");
    }
  }
}

void rs_ag_allreduce(NexarClient& c, uint8_t* buf, size_t count, DataType dt, ReduceOp op, uint64_t tag) {
  // Reduce-scatter then all-gather on the ChunkLayout ("ZeRO-style"); distinct
  // tags for the two halves (2t and 2t+1, rs_ag_allreduce.rs:26-128).
  const uint32_t N = c.world_size();
  if (N <= 1 || count == 0) return;
  const Rank r = c.rank();
  const size_t es = dtype_size(dt);
  ChunkLayout L(count, N);
  const Rank next = (r + 1) % N, prev = (r + N - 1) % N;
  const uint64_t t_rs = tag * 2, t_ag = tag * 2 + 1;
  for (uint32_t s = 0; s + 1 < N; ++s) {
    const uint32_t send_c = (r + N - s - 1) % N, recv_c = (r + N - s - 2) % N;
    c.coll_send(next, step_tag(t_rs, s), buf + L.offset(send_c) * es, L.chunk(send_c) * es, "allreduce_rs_ag");
    Bytes in = c.coll_recv(prev, step_tag(t_rs, s), "allreduce_rs_ag");
    check_len(in, L.chunk(recv_c) * es, "allreduce_rs_ag", prev);
    reduce_slice(buf + L.offset(recv_c) * es, in.data(), L.chunk(recv_c), dt, op);
  }
  // rank r now owns chunk r
  for (uint32_t s = 0; s + 1 < N; ++s) {
    const uint32_t send_c = (r + N - s) % N, recv_c = (r + N - s - 1) % N;
    c.coll_send(next, step_tag(t_ag, s), buf + L.offset(send_c) * es, L.chunk(send_c) * es, "allreduce_rs_ag");
    Bytes in = c.coll_recv(prev, step_tag(t_ag, s), "allreduce_rs_ag");
    check_len(in, L.chunk(recv_c) * es, "allreduce_rs_ag", prev);
    std::memcpy(buf + L.offset(recv_c) * es, in.data(), in.size());
  }
}

// ------------------------------------------------------------------ all-gather / reduce-scatter
void ring_allgather(NexarClient& c, const uint8_t* send, uint8_t* recv, size_t count, DataType dt, uint64_t tag) {
  const uint32_t N = c.world_size();
  const Rank r = c.rank();
  const size_t es = dtype_size(dt), nb = count * es;
  if (send != recv + r * nb) std::memmove(recv + r * nb, send, nb);
  if (N <= 1) return;
  if (nb * N <= c.config().small_msg_bytes && !c.is_sparse()) {
    // Small: direct exchange over the full mesh, the same bytes as the ring
    // in one hop instead of N-1.
    for (uint32_t s = 1; s < N; ++s)
      c.coll_send((r + s) % N, step_tag(tag, 0), recv + r * nb, nb, "allgather");
    for (uint32_t s = 1; s < N; ++s) {
      const Rank src = (r + N - s) % N;
      Bytes in = c.coll_recv(src, step_tag(tag, 0), "allgather");
      check_len(in, nb, "allgather", src);
      std::memcpy(recv + src * nb, in.data(), nb);
    }
    return;
  }
  const Rank next = (r + 1) % N, prev = (r + N - 1) % N;
  const size_t seg = std::max<size_t>(1, c.config().pipeline_segment_bytes / es);
  if (count >= 2 * seg) {
    // Pipelined: each received segment is stored and forwarded at once.
    const size_t nseg = (count + seg - 1) / seg;
    for (size_t k = 0; k < nseg; ++k) {
      const size_t off = k * seg, m = std::min(seg, count - off);
      c.coll_send(next, seg_tag(tag, 0, k, 3), recv + r * nb + off * es, m * es, "allgather");
    }
    for (uint32_t s = 0; s + 1 < N; ++s) {
      const uint32_t recv_i = (r + N - s - 1) % N;
      for (size_t k = 0; k < nseg; ++k) {
        const size_t off = k * seg, m = std::min(seg, count - off);
        Bytes in = c.coll_recv(prev, seg_tag(tag, s, k, 3), "allgather");
        check_len(in, m * es, "allgather", prev);
        uint8_t* dst = recv + recv_i * nb + off * es;
        std::memcpy(dst, in.data(), m * es);
        if (s + 2 < N) c.coll_send(next, seg_tag(tag, s + 1, k, 3), dst, m * es, "allgather");
      }
    }
    return;
  }
  for (uint32_t s = 0; s + 1 < N; ++s) {
    const uint32_t send_i = (r + N - s) % N, recv_i = (r + N - s - 1) % N;
    c.coll_send(next, step_tag(tag, s), recv + send_i * nb, nb, "allgather");
    Bytes in = c.coll_recv(prev, step_tag(tag, s), "allgather");
    check_len(in, nb, "allgather", prev);
    std::memcpy(recv + recv_i * nb, in.data(), nb);
  }
}

void ring_reduce_scatter(NexarClient& c, const uint8_t* send, uint8_t* recv, size_t count, DataType dt, ReduceOp op,
                         uint64_t tag) {
  const uint32_t N = c.world_size();
  const Rank r = c.rank();
  const size_t es = dtype_size(dt), nb = count * es;
  if (N <= 1) {
    std::memmove(recv, send, nb);
    return;
  }
  if (nb * N <= c.config().small_msg_bytes && !c.is_sparse()) {
    // Small: every rank sends block j to rank j directly (the ring's bytes in
    // one hop) and reduces the blocks it receives in rank order.
    for (uint32_t s = 1; s < N; ++s) {
      const Rank dst = (r + s) % N;
      c.coll_send(dst, step_tag(tag, 0), send + dst * nb, nb, "reduce_scatter");
    }
    std::vector<Bytes> got(N);
    for (uint32_t s = 1; s < N; ++s) {
      const Rank src = (r + N - s) % N;
      got[src] = c.coll_recv(src, step_tag(tag, 0), "reduce_scatter");
      check_len(got[src], nb, "reduce_scatter", src);
    }
    Bytes acc(nb);
    for (Rank p = 0; p < N; ++p) {
      const uint8_t* blk = p == r ? send + r * nb : got[p].data();
      if (p == 0) std::memcpy(acc.data(), blk, nb);
      else reduce_slice(acc.data(), blk, count, dt, op);
    }
    std::memcpy(recv, acc.data(), nb);
    return;
  }
  const Rank next = (r + 1) % N, prev = (r + N - 1) % N;
  const size_t seg = std::max<size_t>(1, c.config().pipeline_segment_bytes / es);
  if (count >= 2 * seg) {
    // Pipelined: every segment of a partial sum is forwarded as soon as it is
    // reduced, so receiving, reducing and sending overlap across ring steps.
    const size_t nseg = (count + seg - 1) / seg;
    const uint32_t first = (r + N - 1) % N;
    for (size_t k = 0; k < nseg; ++k) {
      const size_t off = k * seg, m = std::min(seg, count - off);
      c.coll_send(next, seg_tag(tag, 0, k, 2), send + (first * count + off) * es, m * es, "reduce_scatter");
    }
    if (recv != send + r * nb) std::memmove(recv, send + r * nb, nb);
    for (uint32_t s = 0; s + 1 < N; ++s) {
      const uint32_t recv_i = (r + N - s - 2) % N;
      for (size_t k = 0; k < nseg; ++k) {
        const size_t off = k * seg, m = std::min(seg, count - off);
        Bytes in = c.coll_recv(prev, seg_tag(tag, s, k, 2), "reduce_scatter");
        check_len(in, m * es, "reduce_scatter", prev);
        if (s + 2 == N) {
          reduce_slice(recv + off * es, in.data(), m, dt, op);
        } else {
          reduce_slice(in.data(), send + (recv_i * count + off) * es, m, dt, op);
          c.coll_send(next, seg_tag(tag, s + 1, k, 2), in.data(), m * es, "reduce_scatter");
        }
      }
    }
    return;
  }
  // Start one chunk "behind" so the final accumulated chunk is chunk r. The
  // partial sum travels: step 0 sends this rank's own chunk straight from
  // `send`; every later step forwards the chunk received (and reduced) in the
  // step before, so no copy of the whole send buffer is made.
  Bytes acc;
  for (uint32_t s = 0; s + 1 < N; ++s) {
    const uint32_t send_i = (r + N - s - 1) % N, recv_i = (r + N - s - 2) % N;
    const uint8_t* out = s == 0 ? send + send_i * nb : acc.data();
    c.coll_send(next, step_tag(tag, s), out, nb, "reduce_scatter");
    Bytes in = c.coll_recv(prev, step_tag(tag, s), "reduce_scatter");
    check_len(in, nb, "reduce_scatter", prev);
    if (s + 2 == N) {  // recv_i == r: the last partial lands in the output
      if (recv != send + r * nb) std::memmove(recv, send + r * nb, nb);
      reduce_slice(recv, in.data(), count, dt, op);
    } else {
      reduce_slice(in.data(), send + recv_i * nb, count, dt, op);
      acc = std::move(in);
    }
  }
}

// ------------------------------------------------------------------ broadcast / reduce
void broadcast(NexarClient& c, uint8_t* buf, size_t nbytes, Rank root, uint64_t tag) {
  const uint32_t N = c.world_size();
  if (N <= 1) return;
  const Rank r = c.rank();
  if (root >= N) fail(Err::InvalidRank, "invalid rank " + std::to_string(root) + ": world size is " + std::to_string(N));
  if (c.is_sparse() && c.comm_id() == 0) {
    // BFS spanning tree over the overlay (nexar/src/collective/broadcast.rs:99-148).
    SpanningTree t = build_spanning_tree(c.config().topology, root, N);
    if (r != root) {
      Bytes in = c.coll_recv(t.parent.at(r), tag, "broadcast");
      check_len(in, nbytes, "broadcast", t.parent.at(r));
      std::memcpy(buf, in.data(), nbytes);
    }
    for (Rank ch : t.children[r]) c.coll_send(ch, tag, buf, nbytes, "broadcast");
    return;
  }
  if (N < 4) {
    // flat: root sends to everyone
    if (r == root) {
      for (Rank p = 0; p < N; ++p)
        if (p != root) c.coll_send(p, tag, buf, nbytes, "broadcast");
    } else {
      Bytes in = c.coll_recv(root, tag, "broadcast");
      check_len(in, nbytes, "broadcast", root);
      std::memcpy(buf, in.data(), nbytes);
    }
    return;
  }
  // binary tree on logical ranks (root relabelled 0)
  const uint32_t lr = (r + N - root) % N;
  if (lr != 0) {
    const Rank parent = ((lr - 1) / 2 + root) % N;
    Bytes in = c.coll_recv(parent, tag, "broadcast");
    check_len(in, nbytes, "broadcast", parent);
    std::memcpy(buf, in.data(), nbytes);
  }
  for (uint32_t ch : {2 * lr + 1, 2 * lr + 2})
    if (ch < N) c.coll_send((ch + root) % N, tag, buf, nbytes, "broadcast");
}

void reduce(NexarClient& c, uint8_t* buf, size_t count, DataType dt, ReduceOp op, Rank root, uint64_t tag) {
  // Binomial tree towards the root on logical ranks (reduce.rs:14-99); works
  // for any world size (missing partners are skipped).
  const uint32_t N = c.world_size();
  if (N <= 1) return;
  if (root >= N) fail(Err::InvalidRank, "invalid rank " + std::to_string(root) + ": world size is " + std::to_string(N));
  const size_t es = dtype_size(dt);
  const uint32_t lr = (c.rank() + N - root) % N;
  Bytes acc(buf, buf + count * es);
  for (uint32_t mask = 1; mask < N; mask <<= 1) {
    if (lr & mask) {
      c.coll_send(((lr - mask) + root) % N, step_tag(tag, mask), acc.data(), acc.size(), "reduce");
      break;
    }
    const uint32_t src = lr + mask;
    if (src < N) {
      Bytes in = c.coll_recv((src + root) % N, step_tag(tag, mask), "reduce");
      check_len(in, acc.size(), "reduce", (src + root) % N);
      reduce_slice(acc.data(), in.data(), count, dt, op);
    }
  }
  if (lr == 0) std::memcpy(buf, acc.data(), acc.size());
}

// ------------------------------------------------------------------ all-to-all / gather / scatter
void alltoall(NexarClient& c, const uint8_t* send, uint8_t* recv, size_t count, DataType dt, uint64_t tag) {
  const uint32_t N = c.world_size();
  const Rank r = c.rank();
  const size_t nb = count * dtype_size(dt);
  std::memmove(recv + r * nb, send + r * nb, nb);
  // Pairwise order (step s: to r+s, from r-s). Every block is posted before
  // the first receive: peers' router threads drain their sockets, so the
  // sends cannot block on a peer that is itself sending, and the exchange
  // costs one network hop instead of N-1.
  for (uint32_t s = 1; s < N; ++s) {
    const Rank dst = (r + s) % N;
    c.coll_send(dst, step_tag(tag, s), send + dst * nb, nb, "alltoall");
  }
  for (uint32_t s = 1; s < N; ++s) {
    const Rank src = (r + N - s) % N;
    Bytes in = c.coll_recv(src, step_tag(tag, s), "alltoall");
    check_len(in, nb, "alltoall", src);
    std::memcpy(recv + src * nb, in.data(), nb);
  }
}

void gather(NexarClient& c, const uint8_t* send, uint8_t* recv, size_t count, DataType dt, Rank root, uint64_t tag) {
  const uint32_t N = c.world_size();
  const Rank r = c.rank();
  const size_t nb = count * dtype_size(dt);
  if (root >= N) fail(Err::InvalidRank, "invalid rank " + std::to_string(root));
  if (r != root) {
    c.coll_send(root, tag, send, nb, "gather");
    return;
  }
  std::memmove(recv + r * nb, send, nb);
  for (Rank p = 0; p < N; ++p) {
    if (p == root) continue;
    Bytes in = c.coll_recv(p, tag, "gather");
    check_len(in, nb, "gather", p);
    std::memcpy(recv + p * nb, in.data(), nb);
  }
}

void scatter(NexarClient& c, const uint8_t* send, uint8_t* recv, size_t count, DataType dt, Rank root, uint64_t tag) {
  const uint32_t N = c.world_size();
  const Rank r = c.rank();
  const size_t nb = count * dtype_size(dt);
  if (root >= N) fail(Err::InvalidRank, "invalid rank " + std::to_string(root));
  if (r == root) {
    for (Rank p = 0; p < N; ++p)
      if (p != root) c.coll_send(p, tag, send + p * nb, nb, "scatter");
    std::memmove(recv, send + r * nb, nb);
    return;
  }
  Bytes in = c.coll_recv(root, tag, "scatter");
  check_len(in, nb, "scatter", root);
  std::memcpy(recv, in.data(), nb);
}

// ------------------------------------------------------------------ scan
void scan(NexarClient& c, uint8_t* buf, size_t count, DataType dt, ReduceOp op, bool exclusive, uint64_t tag) {
  // Hillis-Steele over ranks: round k sends the running value to rank+2^k
  // and folds in the value from rank-2^k (scan.rs:13-80). The exclusive
  // form shifts the inclusive result one rank to the right; rank 0 gets the
  // op's identity (scan.rs:89-150).
  const uint32_t N = c.world_size();
  const Rank r = c.rank();
  const size_t nb = count * dtype_size(dt);
  Bytes acc(buf, buf + nb);
  for (uint32_t d = 1, k = 0; d < N; d <<= 1, ++k) {
    if (r + d < N) c.coll_send(r + d, step_tag(tag, k), acc.data(), nb, "scan");
    if (r >= d) {
      Bytes in = c.coll_recv(r - d, step_tag(tag, k), "scan");
      check_len(in, nb, "scan", r - d);
      // acc = in op acc (earlier ranks on the left)
      reduce_slice(in.data(), acc.data(), count, dt, op);
      acc.swap(in);
    }
  }
  if (!exclusive) {
    std::memcpy(buf, acc.data(), nb);
    return;
  }
  const uint64_t t = step_tag(tag, 999);
  if (r + 1 < N) c.coll_send(r + 1, t, acc.data(), nb, "exclusive_scan");
  if (r == 0) {
    fill_identity(buf, count, dt, op);
  } else {
    Bytes in = c.coll_recv(r - 1, t, "exclusive_scan");
    check_len(in, nb, "exclusive_scan", r - 1);
    std::memcpy(buf, in.data(), nb);
  }
}

// ------------------------------------------------------------------ barrier
static void expect_barrier(const Message& m, MsgKind k, uint64_t epoch, uint64_t comm, Rank from) {
  if (m.kind != k || m.epoch != epoch || m.comm_id != comm)
    throw collective_failed("barrier", from, std::string("expected ") + msg_kind_name(k) + "(epoch=" +
                                                 std::to_string(epoch) + ", comm_id=" + std::to_string(comm) +
                                                 "), got " + msg_kind_name(m.kind) + "(epoch=" + std::to_string(m.epoch) + ")");
}

void barrier(NexarClient& c, double timeout_s) {
  // world < 5: two-phase through rank 0; otherwise dissemination in
  // ceil(log2 N) rounds (nexar/src/collective/barrier.rs:9-212). Barrier
  // messages have their own per-comm lane, so heartbeats cannot interfere.
  const uint32_t N = c.world_size();
  if (N <= 1) return;
  const uint64_t epoch = c.next_barrier_epoch();
  const uint64_t comm = c.comm_id();
  const Rank r = c.rank();
  auto mesh = c.mesh();
  auto recv_b = [&](Rank from) {
    try {
      return std::move(mesh->box(c.mesh_rank(from))
                           ->pop(LaneKey{LaneKind::Barrier, comm, 0},
                                 Clock::now() + std::chrono::microseconds((int64_t)(timeout_s * 1e6)))
                           .msg);
    } catch (const NexarError& e) {
      if (e.code() == Err::Timeout)
        throw collective_failed("barrier", from, "timed out waiting for barrier(epoch=" + std::to_string(epoch) + ") after " +
                                                     std::to_string((int64_t)(timeout_s * 1000)) + "ms");
      throw collective_failed("barrier", from, e.what());
    }
  };
  auto send_b = [&](Rank to, const Message& m) {
    try {
      c.send_message_to(to, m, Priority::Critical);
    } catch (const NexarError& e) {
      throw collective_failed("barrier", to, e.what());
    }
  };
  if (N < 5) {
    if (r == 0) {
      for (Rank p = 1; p < N; ++p) expect_barrier(recv_b(p), MsgKind::Barrier, epoch, comm, p);
      for (Rank p = 1; p < N; ++p) send_b(p, Message::barrier_ack(epoch, comm));
    } else {
      send_b(0, Message::barrier(epoch, comm));
      expect_barrier(recv_b(0), MsgKind::BarrierAck, epoch, comm, 0);
    }
    return;
  }
  const size_t rounds = ceil_log2(N);
  for (size_t k = 0; k < rounds; ++k) {
    const uint32_t d = 1u << k;
    send_b((r + d) % N, Message::barrier(epoch, comm));
    expect_barrier(recv_b((r + N - d) % N), MsgKind::Barrier, epoch, comm, (r + N - d) % N);
  }
}

// ------------------------------------------------------------------ compressed
void compressed_allreduce(NexarClient& c, uint8_t* buf, size_t count, DataType dt, ReduceOp op, Compressor& comp,
                          uint8_t* residual, uint64_t tag) {
  // Compress locally with error feedback, ring-forward the compressed blobs
  // N-1 times (an all-gather of variable-size blobs), then decompress every
  // rank's blob into a zeroed dense buffer and reduce in rank order, so all
  // ranks produce identical results (compressed_allreduce.rs:29-113).
  const uint32_t N = c.world_size();
  const Rank r = c.rank();
  const size_t es = dtype_size(dt), nb = count * es;
  if ((uint64_t)N * nb * 2 > c.config().compressed_allreduce_max_bytes)
    throw collective_failed("compressed_allreduce", r, "world_size * bytes * 2 exceeds compressed_allreduce_max_bytes");
  CompressedTensor mine = comp.compress(buf, count, dt, residual);
  std::vector<Bytes> blobs(N);
  blobs[r] = mine.data;
  const Rank next = (r + 1) % N, prev = (r + N - 1) % N;
  for (uint32_t s = 0; s + 1 < N; ++s) {
    const uint32_t send_i = (r + N - s) % N, recv_i = (r + N - s - 1) % N;
    c.coll_send(next, step_tag(tag, s), blobs[send_i].data(), blobs[send_i].size(), "compressed_allreduce");
    blobs[recv_i] = c.coll_recv(prev, step_tag(tag, s), "compressed_allreduce");
  }
  Bytes dense(nb);
  for (uint32_t p = 0; p < N; ++p) {
    CompressedTensor ct;
    ct.data = std::move(blobs[p]);
    ct.original_count = count;
    ct.dtype = dt;
    if (p == 0) {
      std::memset(buf, 0, nb);
      comp.decompress(ct, buf);
    } else {
      std::memset(dense.data(), 0, nb);
      comp.decompress(ct, dense.data());
      reduce_slice(buf, dense.data(), count, dt, op);
    }
  }
}

}  // namespace coll

// ============================================================ client wrappers
namespace {
template <typename F> void with_staging(NexarClient& c, void* ptr, size_t nbytes, F&& f) {
  auto ad = c.adapter();
  if (ad->host_addressable()) {
    f(static_cast<uint8_t*>(ptr));
    return;
  }
  Bytes tmp(nbytes);
  ad->stage_for_send(ptr, nbytes, tmp.data());
  f(tmp.data());
  ad->receive_to_device(tmp.data(), nbytes, ptr);
}

// Out-of-place form: `send` (send_bytes) is staged in, `recv` (recv_bytes)
// written back after the algorithm; a null buffer or zero size is skipped
// (gather's and scatter's non-root sides).
template <typename F>
void with_staging2(NexarClient& c, const void* send, size_t send_bytes, void* recv, size_t recv_bytes, F&& f) {
  auto ad = c.adapter();
  if (ad->host_addressable()) {
    f(static_cast<const uint8_t*>(send), static_cast<uint8_t*>(recv));
    return;
  }
  Bytes in, out;
  const uint8_t* s = nullptr;
  uint8_t* r = nullptr;
  if (send && send_bytes) {
    in.resize(send_bytes);
    ad->stage_for_send(send, send_bytes, in.data());
    s = in.data();
  }
  if (recv && recv_bytes) {
    out.resize(recv_bytes);
    r = out.data();
  }
  f(s, r);
  if (r) ad->receive_to_device(out.data(), recv_bytes, recv);
}
}  // namespace

void NexarClient::all_reduce_tagged(void* ptr, size_t count, DataType dt, ReduceOp op, uint64_t tag) {
  const size_t nb = count * dtype_size(dt);
  with_staging(*this, ptr, nb, [&](uint8_t* b) {
    // dispatch (nexar/src/collective/allreduce.rs:21-55)
    if (nb >= config().large_msg_bytes) coll::pipelined_ring_allreduce(*this, b, count, dt, op, tag);
    else if (nb <= config().small_msg_bytes) coll::recursive_doubling_allreduce(*this, b, count, dt, op, tag);
    else if (world_ <= config().ring_max_world || count < world_) coll::ring_allreduce(*this, b, count, dt, op, tag);
    else coll::halving_doubling_allreduce(*this, b, count, dt, op, tag);
  });
}

void NexarClient::all_reduce(void* ptr, size_t count, DataType dt, ReduceOp op) {
  all_reduce_tagged(ptr, count, dt, op, next_collective_tag());
}

void NexarClient::all_reduce_rs_ag(void* ptr, size_t count, DataType dt, ReduceOp op) {
  const uint64_t tag = next_collective_tag();
  with_staging(*this, ptr, count * dtype_size(dt), [&](uint8_t* b) { coll::rs_ag_allreduce(*this, b, count, dt, op, tag); });
}

void NexarClient::all_reduce_bucketed(const std::vector<std::pair<void*, size_t>>& entries, DataType dt, ReduceOp op) {
  all_reduce_bucketed_tagged(entries, dt, op, next_collective_tag());
}

void NexarClient::all_reduce_bucketed_tagged(const std::vector<std::pair<void*, size_t>>& entries, DataType dt,
                                             ReduceOp op, uint64_t tag) {
  // Gather the (ptr, count) list into one buffer, one all-reduce, scatter back
  // (nexar/src/collective/bucketed_allreduce.rs:23-75).
  const size_t es = dtype_size(dt);
  size_t total = 0;
  for (auto& e : entries) total += e.second;
  Bytes flat(total * es);
  size_t off = 0;
  for (auto& e : entries) {
    adapter_->stage_for_send(e.first, e.second * es, flat.data() + off);
    off += e.second * es;
  }
  if (total * es >= config().large_msg_bytes) coll::pipelined_ring_allreduce(*this, flat.data(), total, dt, op, tag);
  else if (total * es <= config().small_msg_bytes) coll::recursive_doubling_allreduce(*this, flat.data(), total, dt, op, tag);
  else coll::ring_allreduce(*this, flat.data(), total, dt, op, tag);
  off = 0;
  for (auto& e : entries) {
    adapter_->receive_to_device(flat.data() + off, e.second * es, e.first);
    off += e.second * es;
  }
}

void NexarClient::all_reduce_compressed(void* ptr, size_t count, DataType dt, ReduceOp op, Compressor& comp, void* residual) {
  all_reduce_compressed_tagged(ptr, count, dt, op, comp, residual, next_collective_tag());
}

void NexarClient::all_reduce_compressed_tagged(void* ptr, size_t count, DataType dt, ReduceOp op, Compressor& comp,
                                               void* residual, uint64_t tag) {
  with_staging(*this, ptr, count * dtype_size(dt), [&](uint8_t* b) {
    coll::compressed_allreduce(*this, b, count, dt, op, comp, static_cast<uint8_t*>(residual), tag);
  });
}

void NexarClient::broadcast(void* ptr, size_t count, DataType dt, Rank root) {
  const uint64_t tag = next_collective_tag();
  const size_t nb = count * dtype_size(dt);
  with_staging(*this, ptr, nb, [&](uint8_t* b) { coll::broadcast(*this, b, nb, root, tag); });
}

void NexarClient::all_gather(const void* send, void* recv, size_t count, DataType dt) {
  const uint64_t tag = next_collective_tag();
  const size_t nb = count * dtype_size(dt);
  with_staging2(*this, send, nb, recv, nb * world_, [&](const uint8_t* s, uint8_t* r) {
    coll::ring_allgather(*this, s, r, count, dt, tag);
  });
}

void NexarClient::reduce_scatter(const void* send, void* recv, size_t count, DataType dt, ReduceOp op) {
  const uint64_t tag = next_collective_tag();
  const size_t nb = count * dtype_size(dt);
  with_staging2(*this, send, nb * world_, recv, nb, [&](const uint8_t* s, uint8_t* r) {
    coll::ring_reduce_scatter(*this, s, r, count, dt, op, tag);
  });
}

void NexarClient::reduce(void* ptr, size_t count, DataType dt, ReduceOp op, Rank root) {
  const uint64_t tag = next_collective_tag();
  with_staging(*this, ptr, count * dtype_size(dt), [&](uint8_t* b) { coll::reduce(*this, b, count, dt, op, root, tag); });
}

void NexarClient::all_to_all(const void* send, void* recv, size_t count, DataType dt) {
  const uint64_t tag = next_collective_tag();
  const size_t nb = count * dtype_size(dt) * world_;
  with_staging2(*this, send, nb, recv, nb, [&](const uint8_t* s, uint8_t* r) { coll::alltoall(*this, s, r, count, dt, tag); });
}

void NexarClient::gather(const void* send, void* recv, size_t count, DataType dt, Rank root) {
  const uint64_t tag = next_collective_tag();
  const size_t nb = count * dtype_size(dt);
  // Only the root's receive buffer (count x world) is written.
  with_staging2(*this, send, nb, rank_ == root ? recv : nullptr, nb * world_, [&](const uint8_t* s, uint8_t* r) {
    coll::gather(*this, s, r, count, dt, root, tag);
  });
}

void NexarClient::scatter(const void* send, void* recv, size_t count, DataType dt, Rank root) {
  const uint64_t tag = next_collective_tag();
  const size_t nb = count * dtype_size(dt);
  // Only the root's send buffer (count x world) is read.
  with_staging2(*this, rank_ == root ? send : nullptr, nb * world_, recv, nb, [&](const uint8_t* s, uint8_t* r) {
    coll::scatter(*this, s, r, count, dt, root, tag);
  });
}

void NexarClient::scan(void* ptr, size_t count, DataType dt, ReduceOp op) {
  const uint64_t tag = next_collective_tag();
  with_staging(*this, ptr, count * dtype_size(dt), [&](uint8_t* b) { coll::scan(*this, b, count, dt, op, false, tag); });
}

void NexarClient::exclusive_scan(void* ptr, size_t count, DataType dt, ReduceOp op) {
  const uint64_t tag = next_collective_tag();
  with_staging(*this, ptr, count * dtype_size(dt), [&](uint8_t* b) { coll::scan(*this, b, count, dt, op, true, tag); });
}

void NexarClient::barrier() { coll::barrier(*this, config().barrier_timeout_s); }
void NexarClient::barrier_with_timeout(double timeout_s) { coll::barrier(*this, timeout_s); }

}  // namespace nexar
