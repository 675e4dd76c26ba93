#include "buffer_pool.h"

#include <cstdlib>
#include <new>

namespace nexar {

namespace {
// Every allocation made through pool_allocate carries this header in front
// of the caller's bytes: the owning pool (nullptr for system allocations)
// and the tier, so a block can be freed on any thread.
struct alignas(64) BlockHeader {
  BufferPool* pool;
  uint32_t tier;
  uint32_t magic;
  size_t capacity;
};
constexpr uint32_t kBlockMagic = 0x4e58424cu;
thread_local BufferPool* tls_pool = nullptr;

void* system_block(size_t bytes) {
  auto* h = static_cast<BlockHeader*>(std::malloc(sizeof(BlockHeader) + bytes));
  if (!h) throw std::bad_alloc();
  h->pool = nullptr;
  h->tier = (uint32_t)PoolTier::Unpooled;
  h->magic = kBlockMagic;
  h->capacity = bytes;
  return h;
}
}  // namespace

void* pool_allocate(size_t bytes) {
  void* block = nullptr;
  if (tls_pool && bytes >= BufferPool::kPoolMinBytes) block = tls_pool->take_block(bytes);
  if (!block) block = system_block(bytes);
  return static_cast<BlockHeader*>(block) + 1;
}

void pool_deallocate(void* p) noexcept {
  if (!p) return;
  BlockHeader* h = static_cast<BlockHeader*>(p) - 1;
  if (h->pool) h->pool->give_block(h);
  else std::free(h);
}

PoolScope::PoolScope(BufferPool* pool) : prev_(tls_pool) { tls_pool = pool; }
PoolScope::~PoolScope() { tls_pool = prev_; }

struct PoolDeleter {
  void operator()(BufferPool* p) const noexcept { p->orphan(); }
};

BufferPool::~BufferPool() {
  for (auto& fl : free_blocks_)
    for (void* b : fl) std::free(b);
}

void BufferPool::orphan() noexcept {
  bool del;
  {
    std::lock_guard<std::mutex> g(mu_);
    orphaned_ = true;
    del = live_blocks_ == 0;
  }
  if (del) delete this;
}

void* BufferPool::take_block(size_t bytes) {
  const PoolTier t = tier_for_size(bytes);
  if (t == PoolTier::Unpooled) return nullptr;
  const int ti = (int)t;
  BlockHeader* h = nullptr;
  {
    std::lock_guard<std::mutex> g(mu_);
    if (!free_blocks_[ti].empty()) {
      h = static_cast<BlockHeader*>(free_blocks_[ti].back());
      free_blocks_[ti].pop_back();
      ++reused_[ti];
    } else {
      ++fresh_[ti];
    }
    ++live_blocks_;
  }
  if (!h) {
    const size_t cap = tiers_[ti].capacity;
    h = static_cast<BlockHeader*>(std::malloc(sizeof(BlockHeader) + cap));
    if (!h) {
      std::lock_guard<std::mutex> g(mu_);
      --live_blocks_;
      throw std::bad_alloc();
    }
    h->capacity = cap;
  }
  h->pool = this;
  h->tier = (uint32_t)ti;
  h->magic = kBlockMagic;
  return h;
}

void BufferPool::give_block(void* block) noexcept {
  auto* h = static_cast<BlockHeader*>(block);
  const int ti = (int)h->tier;
  bool del = false, keep = false;
  {
    std::lock_guard<std::mutex> g(mu_);
    --live_blocks_;
    if (!orphaned_ && free_blocks_[ti].size() < tiers_[ti].count) {
      free_blocks_[ti].push_back(h);
      keep = true;
    }
    del = orphaned_ && live_blocks_ == 0;
  }
  if (!keep) std::free(h);
  if (del) delete this;
}

size_t BufferPool::blocks_reused(PoolTier t) const {
  if (t == PoolTier::Unpooled) return 0;
  std::lock_guard<std::mutex> g(mu_);
  return reused_[(int)t];
}

size_t BufferPool::blocks_fresh(PoolTier t) const {
  if (t == PoolTier::Unpooled) return 0;
  std::lock_guard<std::mutex> g(mu_);
  return fresh_[(int)t];
}

PooledBuf::~PooledBuf() {
  if (pool_ && tier_ != PoolTier::Unpooled) pool_->return_buf(std::move(buf_), tier_);
}

std::shared_ptr<BufferPool> BufferPool::from_tiers(TierConfig s, TierConfig l, TierConfig h, TierConfig g) {
  auto p = std::shared_ptr<BufferPool>(new BufferPool(), PoolDeleter());
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
