// Tiered host buffer pool (nexar/src/transport/buffer_pool.rs:5-354).
//
// Four tiers (small 64 KiB, large 8 MiB, huge 64 MiB, giant 256 MiB), each a
// bounded free list filled lazily. checkout(len) returns a zeroed buffer of
// exactly `len` bytes from the smallest tier that fits (or a one-off
// allocation above the giant tier); dropping the PooledBuf returns it to its
// tier unless the tier is full or the buffer grew past 4x the tier capacity.
// Profiles: Training (256/32/16/4 buffers) and Inference (256/16/4/0).
//
// The client's receive path uses the pool the way the reference's routers
// read frames into pooled buffers (nexar/src/transport/router.rs:408-458):
// every router thread of a mesh runs inside a PoolScope of the mesh's pool,
// so the payload buffers it allocates (16 KiB and more) are tier blocks, and
// a block returns to its tier's free list when the consumer frees the
// payload. Large receives then reuse memory that is already mapped instead of
// faulting in fresh pages for every message.
#pragma once
#include <memory>
#include <mutex>

#include "common.h"

namespace nexar {

enum class PoolProfile : uint8_t { Training = 0, Inference = 1 };
struct TierConfig {
  size_t count;
  size_t capacity;
};
enum class PoolTier : uint8_t { Small = 0, Large = 1, Huge = 2, Giant = 3, Unpooled = 4 };

class BufferPool;

class PooledBuf {
 public:
  PooledBuf(Bytes b, std::shared_ptr<BufferPool> pool, PoolTier tier)
      : buf_(std::move(b)), pool_(std::move(pool)), tier_(tier) {}
  PooledBuf(PooledBuf&&) = default;
  PooledBuf& operator=(PooledBuf&&) = default;
  ~PooledBuf();
  uint8_t* data() { return buf_.data(); }
  size_t size() const { return buf_.size(); }
  PoolTier tier() const { return tier_; }
  Bytes& bytes() { return buf_; }

 private:
  Bytes buf_;
  std::shared_ptr<BufferPool> pool_;
  PoolTier tier_;
};

class BufferPool : public std::enable_shared_from_this<BufferPool> {
 public:
  static constexpr size_t kSmall = 64 << 10, kLarge = 8 << 20, kHuge = 64 << 20, kGiant = 256 << 20;
  // Receive allocations below this size come from the system allocator.
  static constexpr size_t kPoolMinBytes = 16 << 10;
  static std::shared_ptr<BufferPool> with_profile(PoolProfile p);
  static std::shared_ptr<BufferPool> with_config(size_t small_count, size_t small_cap);
  static std::shared_ptr<BufferPool> from_tiers(TierConfig s, TierConfig l, TierConfig h, TierConfig g);
  PooledBuf checkout(size_t len);
  PoolTier tier_for_size(size_t len) const;
  size_t free_count(PoolTier t) const;
  void return_buf(Bytes&& b, PoolTier t);

  // Receive-path blocks (see PoolScope): a block of the tier that fits
  // `bytes` (reused from the free list when one is there), or nullptr above
  // the giant tier. give_block takes a block back (on any thread).
  void* take_block(size_t bytes);
  void give_block(void* block) noexcept;
  // Blocks handed out since creation: served from a free list / newly mapped.
  size_t blocks_reused(PoolTier t) const;
  size_t blocks_fresh(PoolTier t) const;

  // Pools are made by the factories above, whose shared pointers defer the
  // destruction until every receive block has come back.
  ~BufferPool();

 private:
  friend struct PoolDeleter;
  BufferPool() = default;
  void orphan() noexcept;  // the last shared owner is gone: free once no block is out
  TierConfig tiers_[4];
  std::vector<Bytes> free_[4];
  std::vector<void*> free_blocks_[4];
  size_t reused_[4] = {0, 0, 0, 0}, fresh_[4] = {0, 0, 0, 0};
  size_t live_blocks_ = 0;
  bool orphaned_ = false;
  mutable std::mutex mu_;
};

// While alive, Bytes of kPoolMinBytes or more allocated on this thread come
// from `pool`'s tiers (nullptr: the system allocator).
class PoolScope {
 public:
  explicit PoolScope(BufferPool* pool);
  ~PoolScope();
  PoolScope(const PoolScope&) = delete;
  PoolScope& operator=(const PoolScope&) = delete;

 private:
  BufferPool* prev_;
};

// Fluent builder (nexar PoolBuilder): defaults 1 small, 1 large, 1 huge, 0 giant.
class PoolBuilder {
 public:
  PoolBuilder& small(TierConfig c) { s_ = c; return *this; }
  PoolBuilder& large(TierConfig c) { l_ = c; return *this; }
  PoolBuilder& huge(TierConfig c) { h_ = c; return *this; }
  PoolBuilder& giant(TierConfig c) { g_ = c; return *this; }
  std::shared_ptr<BufferPool> build() const { return BufferPool::from_tiers(s_, l_, h_, g_); }

 private:
  TierConfig s_{1, BufferPool::kSmall}, l_{1, BufferPool::kLarge}, h_{1, BufferPool::kHuge}, g_{0, BufferPool::kGiant};
};

}  // namespace nexar
