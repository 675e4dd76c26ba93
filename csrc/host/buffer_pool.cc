#include "buffer_pool.h"

namespace nexar {

PooledBuf::~PooledBuf() {
  if (pool_ && tier_ != PoolTier::Unpooled) pool_->return_buf(std::move(buf_), tier_);
}

std::shared_ptr<BufferPool> BufferPool::from_tiers(TierConfig s, TierConfig l, TierConfig h, TierConfig g) {
  auto p = std::shared_ptr<BufferPool>(new BufferPool());
  p->tiers_[0] = {std::max<size_t>(s.count, 1), s.capacity};
  p->tiers_[1] = {std::max<size_t>(l.count, 1), l.capacity};
  p->tiers_[2] = {std::max<size_t>(h.count, 1), h.capacity};
  p->tiers_[3] = {std::max<size_t>(g.count, 1), g.capacity};
  return p;
}

std::shared_ptr<BufferPool> BufferPool::with_profile(PoolProfile prof) {
  if (prof == PoolProfile::Training)
    return from_tiers({256, kSmall}, {32, kLarge}, {16, kHuge}, {4, kGiant});
  return from_tiers({256, kSmall}, {16, kLarge}, {4, kHuge}, {0, kGiant});
}

std::shared_ptr<BufferPool> BufferPool::with_config(size_t small_count, size_t small_cap) {
  return from_tiers({small_count, small_cap}, {4, kLarge}, {2, kHuge}, {1, kGiant});
}

PoolTier BufferPool::tier_for_size(size_t len) const {
  for (int t = 0; t < 4; ++t)
    if (len <= tiers_[t].capacity) return (PoolTier)t;
  return PoolTier::Unpooled;
}

PooledBuf BufferPool::checkout(size_t len) {
  const PoolTier t = tier_for_size(len);
  Bytes b;
  if (t != PoolTier::Unpooled) {
    std::lock_guard<std::mutex> g(mu_);
    auto& fl = free_[(int)t];
    if (!fl.empty()) {
      b = std::move(fl.back());
      fl.pop_back();
    }
  }
  if (b.capacity() < len && t != PoolTier::Unpooled) b.reserve(tiers_[(int)t].capacity);
  b.assign(len, 0);
  return PooledBuf(std::move(b), shared_from_this(), t);
}

void BufferPool::return_buf(Bytes&& b, PoolTier t) {
  if (t == PoolTier::Unpooled) return;
  const auto& tc = tiers_[(int)t];
  if (b.capacity() > tc.capacity * 4) return;  // grew too large: drop
  std::lock_guard<std::mutex> g(mu_);
  auto& fl = free_[(int)t];
  if (fl.size() >= tc.count) return;  // tier full: drop silently
  b.clear();
  fl.push_back(std::move(b));
}

size_t BufferPool::free_count(PoolTier t) const {
  if (t == PoolTier::Unpooled) return 0;
  std::lock_guard<std::mutex> g(mu_);
  return free_[(int)t].size();
}

}  // namespace nexar
