// Host-side descriptor decoding, validation and canonicalisation.
//
// The wire formats are the reference's (src/tensor0/_stride/_ffi/_descriptor.py:8-76);
// the validation rules and their error classes follow
// crates/tensor0-py/native/layout/{descriptor.cc:14-165, record.cc:260-417}.
// Errors are thrown as InvalidArgument (status 1) or std::runtime_error (status 2).
#pragma once

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

namespace t0b {

struct InvalidArgument : std::invalid_argument {
  using std::invalid_argument::invalid_argument;
};

// One semantic record: a logical box of `shape`, read at src_off + sum(i*sstr)
// and written at dst_off + sum(i*dstr).  `fiber[a]` marks summed axes
// (reduction roles, or accumulation axes whose destination stride is zero).
struct Record {
  uint64_t index = 0;
  int64_t src_off = 0;
  int64_t dst_off = 0;
  std::vector<uint64_t> shape;
  std::vector<int64_t> sstr;
  std::vector<int64_t> dstr;
  std::vector<uint8_t> fiber;
};

struct Layout {
  uint64_t source_size = 0;
  uint64_t output_size = 0;
  std::vector<Record> records;
};

enum class Validation {
  kMap,           // copy / update: injective destinations (DecodeLayout)
  kAccumulation,  // injective over nonzero destination strides (DecodeAccumulationLayout)
  kAddress,       // dot: both sides only in bounds (DecodeAddressLayout)
};

Layout DecodeLayout(const int64_t* words, std::size_t word_count, Validation validation);
Layout DecodeReductionLayout(const int64_t* words, std::size_t word_count);

uint64_t ElementCount(const Record& record);

// One side of a record against its storage: every address in [0, size)
// (an empty record's offset may equal size).  With `injective`, the side's
// strides must also prove distinct addresses.  Throws InvalidArgument with
// the layout decoder's messages.
void CheckSide(const Record& record, bool source, uint64_t size, bool injective);
bool CheckedMul(uint64_t a, uint64_t b, uint64_t* out);
bool CheckedAdd(uint64_t a, uint64_t b, uint64_t* out);
uint64_t AbsStride(int64_t stride);

// Drop extent-1 axes, order map axes by destination stride (innermost first),
// fiber axes after them by source stride, and fuse neighbouring fiber axes
// contiguous in the source.  With fuse_map, neighbouring map axes contiguous
// on both sides are fused as well.
void Canonicalize(Record& record, bool fuse_map);

}  // namespace t0b
