// Tiered host buffer pool (nexar/src/transport/buffer_pool.rs:5-354).
//
// Four tiers (small 64 KiB, large 8 MiB, huge 64 MiB, giant 256 MiB), each a
// bounded free list filled lazily. checkout(len) returns a zeroed buffer of
// exactly `len` bytes from the smallest tier that fits (or a one-off
// allocation above the giant tier); dropping the PooledBuf returns it to its
// tier unless the tier is full or the buffer grew past 4x the tier capacity.
// Profiles: Training (256/32/16/4 buffers) and Inference (256/16/4/0).
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
  static std::shared_ptr<BufferPool> with_profile(PoolProfile p);
  static std::shared_ptr<BufferPool> with_config(size_t small_count, size_t small_cap);
  static std::shared_ptr<BufferPool> from_tiers(TierConfig s, TierConfig l, TierConfig h, TierConfig g);
  PooledBuf checkout(size_t len);
  PoolTier tier_for_size(size_t len) const;
  size_t free_count(PoolTier t) const;
  void return_buf(Bytes&& b, PoolTier t);

 private:
  TierConfig tiers_[4];
  std::vector<Bytes> free_[4];
  mutable std::mutex mu_;
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
