// Descriptor decoding and validation for the v1 wire formats.
//
// Rules (and their messages) follow the reference so callers see the same
// errors: crates/tensor0-py/native/layout/descriptor.cc:14-165 (decode),
// record.cc:260-307 (address bounds), record.cc:309-337 (injectivity proof),
// record.cc:339-417 (record construction).  The implementation is our own.
#include "layout.h"

#include <algorithm>
#include <limits>
#include <numeric>

namespace t0b {

bool CheckedMul(uint64_t a, uint64_t b, uint64_t* out) {
  unsigned __int128 product = static_cast<unsigned __int128>(a) * b;
  if (product > std::numeric_limits<uint64_t>::max()) return false;
  *out = static_cast<uint64_t>(product);
  return true;
}

bool CheckedAdd(uint64_t a, uint64_t b, uint64_t* out) {
  if (a > std::numeric_limits<uint64_t>::max() - b) return false;
  *out = a + b;
  return true;
}

uint64_t AbsStride(int64_t stride) {
  if (stride == std::numeric_limits<int64_t>::min()) return uint64_t{1} << 63;
  return stride < 0 ? static_cast<uint64_t>(-stride) : static_cast<uint64_t>(stride);
}

uint64_t ElementCount(const Record& record) {
  uint64_t count = 1;
  for (uint64_t extent : record.shape) {
    if (!CheckedMul(count, extent, &count)) throw InvalidArgument("layout element count overflows");
  }
  return count;
}

namespace {

constexpr int64_t kInt64Max = std::numeric_limits<int64_t>::max();

const char* Side(bool source) { return source ? "source" : "destination"; }

// Lowest and highest address a record touches over `axes`.
void AddressBounds(const Record& record, bool source, const std::vector<std::size_t>& axes,
                   int64_t* lowest, int64_t* highest) {
  const int64_t offset = source ? record.src_off : record.dst_off;
  const auto& strides = source ? record.sstr : record.dstr;
  if (offset < 0) throw InvalidArgument(std::string(Side(source)) + " address precedes storage");
  int64_t low = offset, high = offset;
  for (std::size_t axis : axes) {
    if (record.shape[axis] <= 1) continue;
    uint64_t span = 0;
    if (!CheckedMul(record.shape[axis] - 1, AbsStride(strides[axis]), &span) ||
        span > static_cast<uint64_t>(kInt64Max)) {
      throw InvalidArgument(std::string(Side(source)) + " address arithmetic overflow");
    }
    if (strides[axis] < 0) {
      if (span > static_cast<uint64_t>(low)) {
        throw InvalidArgument(std::string(Side(source)) + " address precedes storage");
      }
      low -= static_cast<int64_t>(span);
    } else {
      if (span > static_cast<uint64_t>(kInt64Max - high)) {
        throw InvalidArgument(std::string(Side(source)) + " address arithmetic overflow");
      }
      high += static_cast<int64_t>(span);
    }
  }
  *lowest = low;
  *highest = high;
}

// Sufficient proof of injectivity: with axes sorted by |stride|, each stride
// must exceed the span already covered by the smaller ones.
void ProveInjective(const Record& record, bool source, std::vector<std::size_t> axes) {
  const auto& strides = source ? record.sstr : record.dstr;
  std::stable_sort(axes.begin(), axes.end(), [&](std::size_t a, std::size_t b) {
    return std::make_pair(AbsStride(strides[a]), a) < std::make_pair(AbsStride(strides[b]), b);
  });
  uint64_t covered = 0;
  for (std::size_t axis : axes) {
    const uint64_t extent = record.shape[axis];
    if (extent <= 1) continue;
    const uint64_t stride = AbsStride(strides[axis]);
    if (stride <= covered) {
      throw InvalidArgument(std::string(Side(source)) + " strides do not prove an injective view");
    }
    uint64_t span = 0;
    if (!CheckedMul(extent - 1, stride, &span) || !CheckedAdd(covered, span, &covered)) {
      throw InvalidArgument("injectivity arithmetic overflow");
    }
  }
}

std::vector<std::size_t> AllAxes(std::size_t rank) {
  std::vector<std::size_t> axes(rank);
  std::iota(axes.begin(), axes.end(), 0);
  return axes;
}

// Record bounds against both storages (record.cc:339-362 semantics).
void CheckAddressRecord(const Record& record, uint64_t source_size, uint64_t output_size) {
  const uint64_t count = ElementCount(record);
  const auto axes = count == 0 ? std::vector<std::size_t>{} : AllAxes(record.shape.size());
  for (bool source : {true, false}) {
    int64_t low = 0, high = 0;
    AddressBounds(record, source, axes, &low, &high);
    const uint64_t size = source ? source_size : output_size;
    if ((count == 0 && static_cast<uint64_t>(high) > size) ||
        (count != 0 && static_cast<uint64_t>(high) >= size)) {
      throw InvalidArgument(std::string(Side(source)) + " address exceeds storage");
    }
  }
}

class WordReader {
 public:
  WordReader(const int64_t* words, std::size_t count) : words_(words), count_(count) {}
  int64_t Next(const char* truncated) {
    if (cursor_ == count_) throw InvalidArgument(truncated);
    return words_[cursor_++];
  }
  std::size_t Remaining() const { return count_ - cursor_; }
  bool Done() const { return cursor_ == count_; }

 private:
  const int64_t* words_;
  std::size_t count_;
  std::size_t cursor_ = 0;
};

}  // namespace

void CheckSide(const Record& record, bool source, uint64_t size, bool injective) {
  const uint64_t count = ElementCount(record);
  int64_t low = 0, high = 0;
  AddressBounds(record, source, count == 0 ? std::vector<std::size_t>{} : AllAxes(record.shape.size()), &low, &high);
  if ((count == 0 && static_cast<uint64_t>(high) > size) || (count != 0 && static_cast<uint64_t>(high) >= size)) {
    throw InvalidArgument(std::string(Side(source)) + " address exceeds storage");
  }
  if (injective && count != 0) ProveInjective(record, source, AllAxes(record.shape.size()));
}

Layout DecodeLayout(const int64_t* words, std::size_t word_count, Validation validation) {
  if (words == nullptr && word_count != 0) throw InvalidArgument("layout descriptor is null");
  WordReader reader(words, word_count);
  const char* truncated = "layout descriptor is truncated";
  auto size = [&]() {
    const int64_t value = reader.Next(truncated);
    if (value < 0) throw InvalidArgument("layout size or offset is negative");
    return static_cast<uint64_t>(value);
  };
  if (reader.Next(truncated) != 1) throw InvalidArgument("unsupported native layout version");
  Layout layout;
  layout.source_size = size();
  layout.output_size = size();
  const uint64_t records = size();
  if (records > reader.Remaining() / 3) {
    throw InvalidArgument("layout record count exceeds descriptor length");
  }
  layout.records.reserve(records);
  for (uint64_t index = 0; index < records; ++index) {
    Record record;
    record.index = index;
    const uint64_t rank = size();
    record.src_off = static_cast<int64_t>(size());
    record.dst_off = static_cast<int64_t>(size());
    if (rank > reader.Remaining() / 3) throw InvalidArgument("layout rank exceeds descriptor length");
    record.shape.resize(rank);
    record.sstr.resize(rank);
    record.dstr.resize(rank);
    record.fiber.assign(rank, 0);
    for (auto& extent : record.shape) extent = size();
    for (auto& stride : record.sstr) stride = reader.Next(truncated);
    for (auto& stride : record.dstr) stride = reader.Next(truncated);
    CheckAddressRecord(record, layout.source_size, layout.output_size);
    const uint64_t count = ElementCount(record);
    if (validation == Validation::kAddress) {
      // Dot reads both sides; neither needs to be injective.
    } else if (validation == Validation::kMap) {
      const bool has_zero = std::find(record.shape.begin(), record.shape.end(), 0) != record.shape.end();
      ProveInjective(record, false, has_zero ? std::vector<std::size_t>{} : AllAxes(rank));
    } else if (count != 0) {
      std::vector<std::size_t> owners;
      for (std::size_t axis = 0; axis < rank; ++axis) {
        if (record.shape[axis] > 1 && record.dstr[axis] != 0) owners.push_back(axis);
        if (record.shape[axis] > 1 && record.dstr[axis] == 0) record.fiber[axis] = 1;
      }
      try {
        ProveInjective(record, false, owners);
      } catch (const InvalidArgument&) {
        throw InvalidArgument("accumulation cannot prove injective output owners");
      }
    }
    layout.records.push_back(std::move(record));
  }
  if (!reader.Done()) throw InvalidArgument("layout descriptor has trailing words");
  return layout;
}

Layout DecodeReductionLayout(const int64_t* words, std::size_t word_count) {
  if (words == nullptr && word_count != 0) throw InvalidArgument("reduction layout descriptor is null");
  WordReader reader(words, word_count);
  const char* truncated = "reduction layout descriptor is truncated";
  auto next = [&]() { return static_cast<uint64_t>(reader.Next(truncated)); };
  auto offset = [&]() {
    const uint64_t value = next();
    if (value > static_cast<uint64_t>(kInt64Max)) {
      throw InvalidArgument("reduction layout offset exceeds address range");
    }
    return static_cast<int64_t>(value);
  };
  if (next() != 1) throw InvalidArgument("unsupported native reduction layout version");
  Layout layout;
  layout.source_size = next();
  layout.output_size = next();
  const uint64_t records = next();
  if (records > reader.Remaining() / 3) {
    throw InvalidArgument("reduction layout record count exceeds descriptor length");
  }
  layout.records.reserve(records);
  for (uint64_t index = 0; index < records; ++index) {
    Record record;
    record.index = index;
    const uint64_t rank = next();
    record.src_off = offset();
    record.dst_off = offset();
    if (rank > reader.Remaining() / 5) {
      throw InvalidArgument("reduction layout rank exceeds descriptor length");
    }
    std::vector<uint64_t> output_shape(rank);
    record.shape.resize(rank);
    record.sstr.resize(rank);
    record.dstr.resize(rank);
    record.fiber.resize(rank);
    for (auto& extent : record.shape) extent = next();
    for (auto& stride : record.sstr) stride = static_cast<int64_t>(next());
    for (auto& extent : output_shape) extent = next();
    for (auto& stride : record.dstr) stride = static_cast<int64_t>(next());
    for (auto& role : record.fiber) {
      const uint64_t flag = next();
      if (flag > 1) throw InvalidArgument("reduction layout axis flag is not boolean");
      role = static_cast<uint8_t>(flag);
    }
    // Axis roles (record.cc:380-398): reduction axes have output extent 1 and
    // a canonical zero output stride; map axes need a nonzero stride.
    uint64_t owners = 1, contributions = 1;
    std::vector<std::size_t> map_axes;
    for (std::size_t axis = 0; axis < rank; ++axis) {
      const uint64_t extent = record.shape[axis];
      const bool reduce = record.fiber[axis] != 0;
      if (output_shape[axis] != (reduce ? 1 : extent)) {
        throw InvalidArgument("reduction input/output shapes do not match axis roles");
      }
      if (reduce) record.dstr[axis] = 0;
      if (!reduce && extent > 1 && record.dstr[axis] == 0) {
        throw InvalidArgument("reduction output map has a zero nontrivial stride");
      }
      if (!CheckedMul(reduce ? contributions : owners, extent, reduce ? &contributions : &owners)) {
        throw InvalidArgument("reduction fiber element count overflow");
      }
      if (!reduce) map_axes.push_back(axis);
    }
    uint64_t logical = 0;
    if (!CheckedMul(owners, contributions, &logical)) {
      throw InvalidArgument("reduction logical element count overflow");
    }
    ProveInjective(record, false, map_axes);
    for (bool source : {true, false}) {
      const bool empty = source ? logical == 0 : owners == 0;
      const uint64_t size = source ? layout.source_size : layout.output_size;
      if (empty) {
        if (static_cast<uint64_t>(source ? record.src_off : record.dst_off) > size) {
          throw InvalidArgument("empty reduction offset exceeds storage");
        }
      } else {
        int64_t low = 0, high = 0;
        AddressBounds(record, source, source ? AllAxes(rank) : map_axes, &low, &high);
        if (static_cast<uint64_t>(high) >= size) {
          throw InvalidArgument("reduction address exceeds storage");
        }
      }
    }
    ElementCount(record);
    layout.records.push_back(std::move(record));
  }
  if (!reader.Done()) throw InvalidArgument("reduction layout descriptor has trailing words");
  return layout;
}

void Canonicalize(Record& record, bool fuse_map) {
  struct Axis { uint64_t n; int64_t s, d; uint8_t fiber; };
  std::vector<Axis> map, fiber;
  for (std::size_t a = 0; a < record.shape.size(); ++a) {
    if (record.shape[a] == 1) continue;
    (record.fiber[a] ? fiber : map).push_back({record.shape[a], record.sstr[a], record.dstr[a], record.fiber[a]});
  }
  std::stable_sort(map.begin(), map.end(),
                   [](const Axis& a, const Axis& b) { return AbsStride(a.d) < AbsStride(b.d); });
  std::stable_sort(fiber.begin(), fiber.end(),
                   [](const Axis& a, const Axis& b) { return AbsStride(a.s) < AbsStride(b.s); });
  // Fuse inner axis i into outer axis j when j's strides continue i's on both sides.
  auto fuse = [](std::vector<Axis>& axes, bool check_destination) {
    std::vector<Axis> fused;
    for (const Axis& axis : axes) {
      if (!fused.empty()) {
        Axis& inner = fused.back();
        const __int128 s_span = static_cast<__int128>(inner.s) * static_cast<__int128>(inner.n);
        const __int128 d_span = static_cast<__int128>(inner.d) * static_cast<__int128>(inner.n);
        const unsigned __int128 extent = static_cast<unsigned __int128>(inner.n) * axis.n;
        if (s_span == axis.s && (!check_destination || d_span == axis.d) &&
            extent < (static_cast<unsigned __int128>(1) << 62)) {
          inner.n = static_cast<uint64_t>(extent);
          continue;
        }
      }
      fused.push_back(axis);
    }
    axes = std::move(fused);
  };
  if (fuse_map) fuse(map, true);
  fuse(fiber, false);
  record.shape.clear();
  record.sstr.clear();
  record.dstr.clear();
  record.fiber.clear();
  for (const auto* group : {&map, &fiber}) {
    for (const Axis& axis : *group) {
      record.shape.push_back(axis.n);
      record.sstr.push_back(axis.s);
      record.dstr.push_back(axis.d);
      record.fiber.push_back(axis.fiber);
    }
  }
}

}  // namespace t0b
