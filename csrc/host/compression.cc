#include "compression.h"

#include <algorithm>
#include <cmath>
#include <numeric>

#include "reduce.h"

namespace nexar {

uint32_t CompressedTensor::k() const { return data.size() < 4 ? 0 : (uint32_t)get_le(data.data(), 4); }

CompressedTensor CompressedTensor::encode(const std::vector<uint32_t>& idx, const uint8_t* values,
                                          size_t original_count, DataType dt) {
  CompressedTensor c;
  const size_t es = dtype_size(dt);
  c.data.reserve(4 + idx.size() * (4 + es));
  put_u32(c.data, (uint32_t)idx.size());
  for (uint32_t i : idx) put_u32(c.data, i);
  put_bytes(c.data, values, idx.size() * es);
  c.original_count = original_count;
  c.dtype = dt;
  return c;
}

std::vector<uint32_t> CompressedTensor::indices() const {
  const uint32_t n = k();
  if (data.size() < 4 + (size_t)n * 4) fail(Err::DecodeFailed, "compressed tensor truncated");
  std::vector<uint32_t> v(n);
  for (uint32_t i = 0; i < n; ++i) v[i] = (uint32_t)get_le(data.data() + 4 + 4 * i, 4);
  return v;
}

const uint8_t* CompressedTensor::values() const { return data.data() + 4 + (size_t)k() * 4; }

void Compressor::decompress(const CompressedTensor& c, uint8_t* output) const {
  const size_t es = dtype_size(c.dtype);
  const auto idx = c.indices();
  if (c.data.size() != 4 + idx.size() * (4 + es)) fail(Err::DecodeFailed, "compressed tensor size mismatch");
  const uint8_t* vals = c.values();
  for (size_t i = 0; i < idx.size(); ++i) {
    if (idx[i] >= c.original_count) fail(Err::DecodeFailed, "compressed index out of range");
    std::memcpy(output + (size_t)idx[i] * es, vals + i * es, es);
  }
}

size_t topk_count(size_t count, double ratio) {
  size_t k = (size_t)std::ceil((double)count * ratio);
  if (k < 1) k = 1;
  if (k > count) k = count;
  return k;
}

// ------------------------------------------------------------------ helpers
namespace {
// residual += input, elementwise in the tensor's own type.
void accumulate(uint8_t* residual, const uint8_t* input, size_t count, DataType dt) {
  switch (dt) {
    case DataType::F32: case DataType::F64: case DataType::BF16: case DataType::F16:
    case DataType::I32: case DataType::I64: case DataType::U32: case DataType::U64:
    case DataType::I8: case DataType::U8:
      reduce_slice(residual, input, count, dt, ReduceOp::Sum);
      return;
    default:
      for (size_t i = 0; i < count * dtype_size(dt); ++i) residual[i] = (uint8_t)(residual[i] + input[i]);
  }
}

float magnitude(const uint8_t* p, DataType dt) {
  switch (dt) {
    case DataType::F32: { float v; std::memcpy(&v, p, 4); return std::fabs(v); }
    case DataType::F64: { double v; std::memcpy(&v, p, 8); return (float)std::fabs(v); }
    case DataType::BF16: { uint16_t h; std::memcpy(&h, p, 2); return std::fabs(bf16_to_f32(h)); }
    case DataType::F16: { uint16_t h; std::memcpy(&h, p, 2); return std::fabs(f16_to_f32(h)); }
    default: return 0.f;
  }
}

CompressedTensor gather_and_clear(const std::vector<uint32_t>& idx, uint8_t* residual, size_t count, DataType dt) {
  const size_t es = dtype_size(dt);
  Bytes vals(idx.size() * es);
  for (size_t i = 0; i < idx.size(); ++i) {
    std::memcpy(vals.data() + i * es, residual + (size_t)idx[i] * es, es);
    std::memset(residual + (size_t)idx[i] * es, 0, es);
  }
  return CompressedTensor::encode(idx, vals.data(), count, dt);
}
}  // namespace

// ------------------------------------------------------------------ top-k
TopKCompressor::TopKCompressor(double ratio) : ratio_(ratio) {
  if (!(ratio > 0.0 && ratio <= 1.0)) fail(Err::Elastic, "ratio must be in (0.0, 1.0]");
}

namespace {
// fp32 bit pattern of |x| (for non-negative floats the pattern orders like the
// value; a NaN sorts above infinity).
inline uint32_t mag_key(const uint8_t* p, DataType dt) {
  const float m = magnitude(p, dt);
  uint32_t b;
  std::memcpy(&b, &m, 4);
  return b & 0x7fffffffu;
}
inline uint32_t f32_key(float v) {
  uint32_t b;
  std::memcpy(&b, &v, 4);
  return b & 0x7fffffffu;
}
}  // namespace

CompressedTensor TopKCompressor::compress(const uint8_t* input, size_t count, DataType dt, uint8_t* residual) {
  const bool is_float = dt == DataType::F32 || dt == DataType::F64 || dt == DataType::BF16 || dt == DataType::F16;
  if (!is_float || count == 0) {
    accumulate(residual, input, count, dt);
    // Integer tensors are sent whole (magnitude ranking is not meaningful).
    std::vector<uint32_t> idx(count);
    std::iota(idx.begin(), idx.end(), 0u);
    return gather_and_clear(idx, residual, count, dt);
  }
  const size_t es = dtype_size(dt);
  const size_t k = topk_count(count, ratio_);
  // Radix select on the magnitude keys (mag_key). Pass 1 (fused with the
  // error-feedback accumulation for f32): a histogram of the keys' top 11
  // bits, four interleaved copies so runs of equal bins do not serialise on
  // one counter. The bin holding the k-th largest key follows from the
  // counts. Pass 2 collects, in index order, the indices of every key in a
  // higher bin and the (index, key) pairs of that bin; nth_element over the
  // bin's keys gives the threshold, and a merge of the two ascending lists
  // yields the k largest magnitudes, ties broken towards the lower index.
  uint32_t hist4[4][2048] = {};
  if (dt == DataType::F32) {
    float* r = reinterpret_cast<float*>(residual);
    const float* x = reinterpret_cast<const float*>(input);
    size_t i = 0;
    for (; i + 4 <= count; i += 4) {
      const float v0 = r[i] + x[i], v1 = r[i + 1] + x[i + 1], v2 = r[i + 2] + x[i + 2], v3 = r[i + 3] + x[i + 3];
      r[i] = v0;
      r[i + 1] = v1;
      r[i + 2] = v2;
      r[i + 3] = v3;
      ++hist4[0][f32_key(v0) >> 20];
      ++hist4[1][f32_key(v1) >> 20];
      ++hist4[2][f32_key(v2) >> 20];
      ++hist4[3][f32_key(v3) >> 20];
    }
    for (; i < count; ++i) {
      r[i] += x[i];
      ++hist4[0][f32_key(r[i]) >> 20];
    }
  } else {
    accumulate(residual, input, count, dt);
    for (size_t i = 0; i < count; ++i) ++hist4[i & 3][mag_key(residual + i * es, dt) >> 20];
  }
  if (k >= count) {
    std::vector<uint32_t> all(count);
    std::iota(all.begin(), all.end(), 0u);
    return gather_and_clear(all, residual, count, dt);
  }
  size_t above = 0;
  uint32_t bin = 2047;
  for (; bin > 0; --bin) {
    const size_t h = (size_t)hist4[0][bin] + hist4[1][bin] + hist4[2][bin] + hist4[3][bin];
    if (above + h >= k) break;
    above += h;
  }
  std::vector<uint32_t> hi_idx, c_idx, c_key;
  hi_idx.reserve(above);
  auto visit = [&](size_t i, uint32_t v) {
    const uint32_t b = v >> 20;
    if (b > bin) {
      hi_idx.push_back((uint32_t)i);
    } else if (b == bin) {
      c_idx.push_back((uint32_t)i);
      c_key.push_back(v);
    }
  };
  if (dt == DataType::F32) {
    const uint32_t* rb = reinterpret_cast<const uint32_t*>(residual);
    const uint32_t lo = bin << 20;  // keys below `lo` are skipped without a branch-heavy path
    for (size_t i = 0; i < count; ++i) {
      const uint32_t v = rb[i] & 0x7fffffffu;
      if (v >= lo) visit(i, v);
    }
  } else {
    for (size_t i = 0; i < count; ++i) visit(i, mag_key(residual + i * es, dt));
  }
  const size_t need = k - above;  // >= 1 keys from the threshold bin
  std::vector<uint32_t> sorted_keys(c_key);
  std::nth_element(sorted_keys.begin(), sorted_keys.begin() + (need - 1), sorted_keys.end(), std::greater<uint32_t>());
  const uint32_t thr = sorted_keys[need - 1];
  size_t ties = need;
  for (uint32_t v : c_key)
    if (v > thr) --ties;
  std::vector<uint32_t> idx;
  idx.reserve(k);
  size_t a = 0;
  for (size_t j = 0; j < c_idx.size(); ++j) {
    const uint32_t v = c_key[j];
    if (!(v > thr || (v == thr && ties))) continue;
    if (v == thr) --ties;
    while (a < hi_idx.size() && hi_idx[a] < c_idx[j]) idx.push_back(hi_idx[a++]);
    idx.push_back(c_idx[j]);
  }
  while (a < hi_idx.size()) idx.push_back(hi_idx[a++]);
  return gather_and_clear(idx, residual, count, dt);
}

// ------------------------------------------------------------------ random-k
RandomKCompressor::RandomKCompressor(double ratio) : ratio_(ratio) {
  if (!(ratio > 0.0 && ratio <= 1.0)) fail(Err::Elastic, "ratio must be in (0.0, 1.0]");
}

CompressedTensor RandomKCompressor::compress(const uint8_t* input, size_t count, DataType dt, uint8_t* residual) {
  accumulate(residual, input, count, dt);
  const size_t es = dtype_size(dt);
  const size_t k = count ? topk_count(count, ratio_) : 0;
  // Seed: FNV-1a over (a sample of) the residual bytes, so ranks with the
  // same residual choose the same indices.
  uint64_t h = 0xcbf29ce484222325ull;
  const size_t nb = count * es;
  const size_t step = std::max<size_t>(1, nb / 4096);
  for (size_t i = 0; i < nb; i += step) {
    h ^= residual[i];
    h *= 0x100000001b3ull;
  }
  // splitmix64 stream; partial Fisher-Yates picks k distinct indices.
  auto next = [&h]() {
    h += 0x9e3779b97f4a7c15ull;
    uint64_t z = h;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
  };
  std::vector<uint32_t> pool(count);
  std::iota(pool.begin(), pool.end(), 0u);
  for (size_t i = 0; i < k; ++i) {
    const size_t j = i + (size_t)(next() % (count - i));
    std::swap(pool[i], pool[j]);
  }
  pool.resize(k);
  std::sort(pool.begin(), pool.end());
  return gather_and_clear(pool, residual, count, dt);
}

// ------------------------------------------------------------------ none
CompressedTensor NoCompression::compress(const uint8_t* input, size_t count, DataType dt, uint8_t* residual) {
  (void)residual;
  std::vector<uint32_t> idx(count);
  std::iota(idx.begin(), idx.end(), 0u);
  return CompressedTensor::encode(idx, input, count, dt);
}

}  // namespace nexar
