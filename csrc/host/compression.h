// Gradient compressors with error feedback (nexar/src/compression/*).
//
// Wire format of a compressed tensor (nexar/src/compression/traits.rs:7-42):
//   [k u32 LE][k x u32 LE indices, ascending][k x element values]
//
// TopK keeps the k = max(1, ceil(n * ratio)) entries of largest |residual|
// (residual += input first; chosen entries are zeroed in the residual). This
// implementation selects by radix select on the magnitudes' fp32 bit
// patterns (two streaming passes plus a partial sort of one histogram bin)
// and breaks ties towards the lower index, so every run picks the same set;
// it compresses f32, f64, bf16 and f16 (the reference passes anything but
// f32/f64 through uncompressed).
// RandomK samples k distinct indices with a generator seeded from a hash of
// the residual; NoCompression sends every element.
#pragma once
#include "common.h"

namespace nexar {

struct CompressedTensor {
  Bytes data;
  size_t original_count = 0;
  DataType dtype = DataType::F32;
  uint32_t k() const;
  static CompressedTensor encode(const std::vector<uint32_t>& idx, const uint8_t* values, size_t original_count,
                                 DataType dt);
  std::vector<uint32_t> indices() const;
  const uint8_t* values() const;
};

class Compressor {
 public:
  virtual ~Compressor() = default;
  virtual std::string name() const = 0;
  // residual (count elements of dt) accumulates the untransmitted error.
  virtual CompressedTensor compress(const uint8_t* input, size_t count, DataType dt, uint8_t* residual) = 0;
  // Scatter the kept values into `output` (count elements, caller-zeroed).
  virtual void decompress(const CompressedTensor& c, uint8_t* output) const;
};

class TopKCompressor : public Compressor {
 public:
  explicit TopKCompressor(double ratio);
  std::string name() const override { return "topk"; }
  CompressedTensor compress(const uint8_t* input, size_t count, DataType dt, uint8_t* residual) override;
  double ratio() const { return ratio_; }

 private:
  double ratio_;
};

class RandomKCompressor : public Compressor {
 public:
  explicit RandomKCompressor(double ratio);
  std::string name() const override { return "randomk"; }
  CompressedTensor compress(const uint8_t* input, size_t count, DataType dt, uint8_t* residual) override;

 private:
  double ratio_;
};

class NoCompression : public Compressor {
 public:
  std::string name() const override { return "none"; }
  CompressedTensor compress(const uint8_t* input, size_t count, DataType dt, uint8_t* residual) override;
};

size_t topk_count(size_t count, double ratio);

}  // namespace nexar
