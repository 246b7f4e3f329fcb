// Plan construction: validation, canonicalisation, engine selection, tiling
// and the packed device table.
#include "plan.h"

#include "layout.h"

#include <algorithm>
#include <cstring>
#include <limits>
#include <map>
#include <numeric>
#include <stdexcept>

namespace t0b {
namespace {

constexpr uint64_t kExtentLimit = uint64_t{1} << 30;   // per-axis extent kept in int32
constexpr uint64_t kProofLimit = uint64_t{1} << 28;    // largest address span checked with a bitmap

// Bytes of shared memory one map tile may stage (before row padding): 48 KB
// for copy and accumulation (four 128-thread CTAs per SM; the third box axis
// then extends short source rows to several hundred bytes), 32 KB for update,
// which stages the destination's base values beside it (three 256-thread CTAs
// per SM, 64 KB each).
#ifndef T0B_TILE_BYTES
#define T0B_TILE_BYTES 49152
#endif
#ifndef T0B_UPDATE_TILE_BYTES
#define T0B_UPDATE_TILE_BYTES 32768
#endif
constexpr int64_t kTileBytes = T0B_TILE_BYTES;
constexpr int64_t kUpdateTileBytes = T0B_UPDATE_TILE_BYTES;
// Shortest X and Y tile extents walked with the fixed rectangular thread map:
// shorter rows leave most lanes of a warp idle there, and the run walk packs
// them instead.  The map is used for update tiles, where it measured faster
// than the run walk; copy and accumulation measured faster with the run walk.
#ifndef T0B_RECT_MIN_EXTENT
#define T0B_RECT_MIN_EXTENT 32
#endif
constexpr int32_t kRectMinExtent = T0B_RECT_MIN_EXTENT;

// Split records so every axis extent fits in int32 and at most kMaxRank axes remain.
std::vector<Record> SplitForDevice(const Record& record) {
  std::vector<Record> pending{record}, done;
  while (!pending.empty()) {
    Record current = std::move(pending.back());
    pending.pop_back();
    std::size_t axis = current.shape.size();
    for (std::size_t a = 0; a < current.shape.size(); ++a) {
      if (current.shape[a] > kExtentLimit) { axis = a; break; }
    }
    if (axis != current.shape.size()) {
      for (uint64_t start = 0; start < current.shape[axis]; start += kExtentLimit) {
        Record piece = current;
        piece.shape[axis] = std::min(kExtentLimit, current.shape[axis] - start);
        piece.src_off += static_cast<int64_t>(start) * current.sstr[axis];
        piece.dst_off += static_cast<int64_t>(start) * current.dstr[axis];
        pending.push_back(std::move(piece));
      }
      continue;
    }
    if (current.shape.size() > static_cast<std::size_t>(kMaxRank)) {
      // Peel the outermost map axis (or the last fiber axis if only fibers remain).
      std::size_t peel = current.shape.size() - 1;
      for (std::size_t a = current.shape.size(); a-- > 0;) {
        if (!current.fiber[a]) { peel = a; break; }
      }
      if (current.fiber[peel]) {
        throw std::runtime_error("reduction records with more than eight fused summed axes are unsupported");
      }
      for (uint64_t i = 0; i < current.shape[peel]; ++i) {
        Record piece = current;
        piece.src_off += static_cast<int64_t>(i) * current.sstr[peel];
        piece.dst_off += static_cast<int64_t>(i) * current.dstr[peel];
        piece.shape.erase(piece.shape.begin() + peel);
        piece.sstr.erase(piece.sstr.begin() + peel);
        piece.dstr.erase(piece.dstr.begin() + peel);
        piece.fiber.erase(piece.fiber.begin() + peel);
        pending.push_back(std::move(piece));
      }
      continue;
    }
    done.push_back(std::move(current));
  }
  std::reverse(done.begin(), done.end());
  return done;
}

uint64_t OwnerCount(const Record& record) {
  uint64_t owners = 1;
  for (std::size_t a = 0; a < record.shape.size(); ++a) {
    if (!record.fiber[a]) owners *= record.shape[a];
  }
  return owners;
}

// Visit every destination address of a record's map (owner) axes.
template <typename Visit>
void ForEachOwnerAddress(const Record& record, Visit visit) {
  std::vector<std::size_t> axes;
  for (std::size_t a = 0; a < record.shape.size(); ++a) {
    if (!record.fiber[a] && record.shape[a] > 1) axes.push_back(a);
  }
  std::vector<uint64_t> index(axes.size(), 0);
  int64_t address = record.dst_off;
  for (;;) {
    if (!visit(address)) return;
    std::size_t k = 0;
    for (; k < axes.size(); ++k) {
      const std::size_t a = axes[k];
      if (++index[k] < record.shape[a]) { address += record.dstr[a]; break; }
      address -= static_cast<int64_t>(record.shape[a] - 1) * record.dstr[a];
      index[k] = 0;
    }
    if (k == axes.size()) return;
  }
}

// Address interval [lo, hi] a record's owner (map) axes reach.
void OwnerInterval(const Record& record, int64_t* lo, int64_t* hi) {
  *lo = *hi = record.dst_off;
  for (std::size_t a = 0; a < record.shape.size(); ++a) {
    if (record.fiber[a] || record.shape[a] < 2) continue;
    const int64_t span = static_cast<int64_t>(record.shape[a] - 1) * record.dstr[a];
    if (span > 0) *hi += span; else *lo += span;
  }
}

// A record's owner addresses written as origin + q * radix + m with m in
// [0, radix): axes whose stride is a multiple of the radix move q, the others
// move m.  Valid when the m span stays inside [0, radix), so q and m are
// unique; the record then lies inside the rectangle [q_lo, q_hi] x [m_lo, m_hi].
struct Rectangle {
  int64_t q_lo, q_hi, m_lo, m_hi;
};

bool Decompose(const Record& record, int64_t origin, int64_t radix, Rectangle* out) {
  const int64_t at = record.dst_off - origin;
  Rectangle r{at / radix, at / radix, at % radix, at % radix};
  for (std::size_t a = 0; a < record.shape.size(); ++a) {
    if (record.fiber[a] || record.shape[a] < 2) continue;
    const int64_t n = static_cast<int64_t>(record.shape[a] - 1), s = record.dstr[a];
    if (s % radix == 0) {
      (s > 0 ? r.q_hi : r.q_lo) += n * (s / radix);
    } else {
      (s > 0 ? r.m_hi : r.m_lo) += n * s;
    }
  }
  if (r.m_lo < 0 || r.m_hi >= radix) return false;
  *out = r;
  return true;
}

// Pairwise-disjoint rectangles, by a sweep over q; false when inconclusive
// (an overlap, or more comparisons than the budget allows).
bool RectanglesDisjoint(std::vector<Rectangle>& rects) {
  std::sort(rects.begin(), rects.end(), [](const Rectangle& a, const Rectangle& b) { return a.q_lo < b.q_lo; });
  std::vector<const Rectangle*> active;
  uint64_t budget = uint64_t{1} << 26;
  for (const Rectangle& r : rects) {
    std::size_t keep = 0;
    for (const Rectangle* other : active) {
      if (other->q_hi < r.q_lo) continue;
      if (budget-- == 0) return false;
      if (!(other->m_hi < r.m_lo || r.m_hi < other->m_lo)) return false;
      active[keep++] = other;
    }
    active.resize(keep);
    active.push_back(&r);
  }
  return true;
}

// Exact check by a bit per address over [lo, hi].
bool BitmapDisjoint(const std::vector<const Record*>& records, int64_t lo, int64_t hi) {
  const uint64_t span = static_cast<uint64_t>(hi - lo) + 1;
  uint64_t total = 0;
  for (const Record* record : records) total += OwnerCount(*record);
  if (total > span || span > kProofLimit) return false;
  std::vector<uint64_t> bits((span + 63) / 64, 0);
  bool disjoint = true;
  for (const Record* record : records) {
    ForEachOwnerAddress(*record, [&](int64_t address) {
      const uint64_t at = static_cast<uint64_t>(address - lo);
      uint64_t& word = bits[at >> 6];
      const uint64_t mask = uint64_t{1} << (at & 63);
      if (word & mask) { disjoint = false; return false; }
      word |= mask;
      return true;
    });
    if (!disjoint) return false;
  }
  return true;
}

// Pairwise disjointness of the records' owner addresses (each record's own
// injectivity is validated when the layout is decoded).  Records whose
// address intervals do not meet are disjoint; each cluster of meeting
// intervals is proven either by a radix decomposition (a packed block's
// sub-blocks are rectangles of rows x columns under the block's row stride)
// or, over spans up to 2^28 addresses, exactly with a bitmap.
bool ProveDisjoint(const std::vector<const Record*>& records, uint64_t output_size) {
  uint64_t total = 0;
  for (const Record* record : records) total += OwnerCount(*record);
  if (total > output_size) return false;
  struct Item { int64_t lo, hi; const Record* record; };
  std::vector<Item> items;
  items.reserve(records.size());
  for (const Record* record : records) {
    Item item{0, 0, record};
    OwnerInterval(*record, &item.lo, &item.hi);
    items.push_back(item);
  }
  std::sort(items.begin(), items.end(), [](const Item& a, const Item& b) { return a.lo < b.lo; });
  std::size_t begin = 0;
  while (begin < items.size()) {
    std::size_t end = begin + 1;
    int64_t reach = items[begin].hi;
    while (end < items.size() && items[end].lo <= reach) reach = std::max(reach, items[end++].hi);
    if (end - begin > 1) {
      std::vector<const Record*> cluster;
      std::map<int64_t, int> radices;
      for (std::size_t i = begin; i < end; ++i) {
        cluster.push_back(items[i].record);
        const Record& r = *items[i].record;
        for (std::size_t a = 0; a < r.shape.size(); ++a) {
          if (!r.fiber[a] && r.shape[a] > 1 && AbsStride(r.dstr[a]) > 1) ++radices[static_cast<int64_t>(AbsStride(r.dstr[a]))];
        }
      }
      std::vector<std::pair<int, int64_t>> candidates;
      for (const auto& [radix, count] : radices) candidates.emplace_back(-count, radix);
      std::sort(candidates.begin(), candidates.end());
      bool proven = false;
      for (std::size_t c = 0; c < candidates.size() && c < 8 && !proven; ++c) {
        std::vector<Rectangle> rects(cluster.size());
        bool all = true;
        for (std::size_t i = 0; i < cluster.size() && all; ++i) {
          all = Decompose(*cluster[i], items[begin].lo, candidates[c].second, &rects[i]);
        }
        proven = all && RectanglesDisjoint(rects);
      }
      if (!proven && !BitmapDisjoint(cluster, items[begin].lo, reach)) return false;
    }
    begin = end;
  }
  return true;
}

int64_t CeilDiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Division constants the device uses to decode a tile without dividing.
void SetDivisions(MapRecord& r) {
  for (int i = 0; i < kMaxRank; ++i) {
    const int32_t divisor = i < 3 ? r.c[i] : (i - 3 < r.nouter ? r.n[i] : 1);
    r.div_tiles[i] = MakeDivision(static_cast<uint32_t>(std::max(divisor, 1)));
  }
  for (int i = 0; i < 2; ++i) {
    r.edge[i] = r.n[i] - (r.c[i] - 1) * r.t[i];
    r.div_extent[2 * i] = MakeDivision(static_cast<uint32_t>(std::max(r.t[i], 1)));
    r.div_extent[2 * i + 1] = MakeDivision(static_cast<uint32_t>(std::max(r.edge[i], 1)));
  }
}

MapRecord MakeMapRecord(const Record& record, int64_t slot, int64_t budget, int64_t tile_begin, bool allow_rect) {
  MapRecord out{};
  out.src_off = record.src_off;
  out.dst_off = record.dst_off;
  out.tile_begin = tile_begin;
  out.coef_slot = static_cast<int32_t>(slot);
  const std::size_t rank = record.shape.size();
  // Canonical order: axes by |destination stride|, innermost first.
  std::size_t x = 0;
  std::size_t y = 0;
  for (std::size_t a = 1; a < rank; ++a) {
    if (AbsStride(record.sstr[a]) < AbsStride(record.sstr[y])) y = a;
  }
  std::vector<std::size_t> rest;
  for (std::size_t a = 0; a < rank; ++a) {
    if (a != x && a != y) rest.push_back(a);
  }
  auto put = [&](int slot_index, std::size_t axis) {
    out.n[slot_index] = static_cast<int32_t>(record.shape[axis]);
    out.s[slot_index] = record.sstr[axis];
    out.d[slot_index] = record.dstr[axis];
  };
  for (int i = 0; i < kMaxRank; ++i) { out.n[i] = 1; out.s[i] = 0; out.d[i] = 0; }
  if (rank == 0) {
    out.mode = kDirect;
    out.t[0] = out.t[1] = out.t[2] = 1;
    out.c[0] = out.c[1] = out.c[2] = 1;
    out.nouter = 0;
    SetDivisions(out);
    return out;
  }
  put(0, x);
  // The third box axis extends whichever contiguous run the box leaves
  // shorter: the destination run (X, possibly continued by Y) or the source
  // run (Y).  Short source runs waste DRAM bursts: the bytes that follow a run
  // belong to a later tile and are evicted before it runs.
  std::size_t z_axis = rank;
  if (!rest.empty()) {
    const uint64_t nx = record.shape[x], ny = record.shape[y];
    const bool y_continues_dst = x != y && record.dstr[y] == static_cast<int64_t>(nx) * record.dstr[x];
    const uint64_t dst_run = x == y ? nx : (y_continues_dst ? nx * ny : nx);
    const uint64_t src_run = x == y ? nx : ny;
    auto continues = [&](std::size_t axis, bool source) {
      const std::size_t from = source ? y : (y_continues_dst ? y : x);
      const auto& strides = source ? record.sstr : record.dstr;
      return strides[axis] == static_cast<int64_t>(record.shape[from]) * strides[from];
    };
    std::size_t pick = rest.front();
    bool found = false;
    const bool extend_source = src_run <= dst_run;
    for (std::size_t axis : rest) {
      if (continues(axis, extend_source)) { pick = axis; found = true; break; }
    }
    if (!found) {
      for (std::size_t axis : rest) {
        if (continues(axis, !extend_source)) { pick = axis; break; }
      }
    }
    z_axis = pick;
    rest.erase(std::find(rest.begin(), rest.end(), pick));
  }
  if (x == y) {
    out.mode = kDirect;
    out.t[0] = static_cast<int32_t>(std::min<int64_t>(out.n[0], budget));   // one run per (y, z)
    out.t[1] = 1;
  } else {
    out.mode = kTranspose;
    put(1, y);
    out.t[0] = static_cast<int32_t>(std::min<int64_t>(out.n[0], 64));
    out.t[1] = static_cast<int32_t>(std::min<int64_t>(out.n[1], std::max<int64_t>(1, std::min<int64_t>(64, budget / out.t[0]))));
  }
  if (z_axis != rank) put(2, z_axis);
  out.t[2] = static_cast<int32_t>(std::min<int64_t>(out.n[2], std::max<int64_t>(1, budget / (int64_t{out.t[0]} * out.t[1]))));
  // The rectangular thread map covers X and Y extents up to 64 (two lanes' worth).
  if (allow_rect && out.mode == kTranspose && out.s[1] == 1 && out.d[0] == 1 && out.t[0] >= kRectMinExtent &&
      out.t[1] >= kRectMinExtent && out.t[0] <= 64 && out.t[1] <= 64) {
    out.mode = kRect;
  }
  for (int i = 0; i < 3; ++i) out.c[i] = static_cast<int32_t>(CeilDiv(out.n[i], out.t[i]));
  out.nouter = static_cast<int32_t>(rest.size());
  for (std::size_t i = 0; i < rest.size(); ++i) put(3 + static_cast<int>(i), rest[i]);
  SetDivisions(out);
  return out;
}

int64_t MapTiles(const MapRecord& record) {
  int64_t tiles = int64_t{record.c[0]} * record.c[1] * record.c[2];
  for (int i = 0; i < record.nouter; ++i) tiles *= record.n[3 + i];
  if (tiles >= (int64_t{1} << 31)) {
    throw std::runtime_error("a record spans more than 2^31 tiles; split it into smaller records");
  }
  return tiles;
}

// In-tile offsets fit in int32 when every box-axis stride and span does.
bool NeedsWideOffsets(const MapRecord& record) {
  constexpr int64_t kLimit = (int64_t{1} << 31) - 1;
  int64_t src_span = 0, dst_span = 0;
  for (int i = 0; i < 3; ++i) {
    const int64_t s = record.s[i] < 0 ? -record.s[i] : record.s[i];
    const int64_t d = record.d[i] < 0 ? -record.d[i] : record.d[i];
    if (s > kLimit || d > kLimit) return true;
    src_span += (record.t[i] - 1) * s;
    dst_span += (record.t[i] - 1) * d;
    if (src_span > kLimit || dst_span > kLimit) return true;
  }
  return false;
}

template <typename T>
void Append(std::vector<int64_t>& table, const std::vector<T>& items) {
  static_assert(sizeof(T) % 16 == 0, "device records are 16-byte multiples");
  const std::size_t words = items.size() * sizeof(T) / sizeof(int64_t);
  const std::size_t at = table.size();
  table.resize(at + words);
  if (words) std::memcpy(table.data() + at, items.data(), words * sizeof(int64_t));
}

// Dot: out[b] = sum over records and elements of conj?(left[src]) * right[dst]
// (the reference's dot_p; execute/dot.h).  Records are canonicalised with
// both sides' contiguous axes fused; the row (axis 0) is cut into units of at
// most kDotChunk elements.
constexpr int64_t kDotChunk = 1024;

Plan BuildDotPlan(const int64_t* words, std::size_t word_count, int32_t element_bytes, uint32_t flags) {
  Layout layout = DecodeLayout(words, word_count, Validation::kAddress);
  Plan plan;
  plan.operation = 2;
  plan.element_bytes = element_bytes;
  plan.flags = flags;
  plan.source_size = layout.source_size;
  plan.output_size = layout.output_size;
  plan.records = layout.records.size();
  std::vector<DotRecord> dots;
  int64_t units = 0;
  uint64_t elements = 0;
  for (const Record& original : layout.records) {
    if (ElementCount(original) == 0) continue;
    Record record = original;
    Canonicalize(record, true);
    for (Record& piece : SplitForDevice(record)) {
      DotRecord d{};
      d.left_off = piece.src_off;
      d.right_off = piece.dst_off;
      d.unit_begin = units;
      const int rank = static_cast<int>(piece.shape.size());
      d.rank = std::max(rank, 1);
      for (int a = 0; a < kMaxRank; ++a) { d.n[a] = 1; d.sl[a] = 0; d.sr[a] = 0; }
      for (int a = 0; a < rank; ++a) {
        d.n[a] = static_cast<int32_t>(piece.shape[a]);
        d.sl[a] = piece.sstr[a];
        d.sr[a] = piece.dstr[a];
      }
      d.chunk = static_cast<int32_t>(std::min<int64_t>(d.n[0], kDotChunk));
      d.chunks = static_cast<int32_t>(CeilDiv(d.n[0], d.chunk));
      int64_t record_units = d.chunks;
      for (int a = 1; a < d.rank; ++a) record_units *= d.n[a];
      if (units + record_units >= (int64_t{1} << 31)) {
        throw std::runtime_error("a dot layout spans more than 2^31 work units per batch");
      }
      d.div[0] = MakeDivision(static_cast<uint32_t>(d.chunks));
      for (int a = 1; a < kMaxRank; ++a) d.div[a] = MakeDivision(static_cast<uint32_t>(std::max(d.n[a], 1)));
      units += record_units;
      elements += ElementCount(piece);
      dots.push_back(d);
    }
  }
  plan.dot_units = static_cast<uint64_t>(units);
  plan.scratch = kDotPartials;
  plan.bytes_moved = 2 * elements * static_cast<uint64_t>(element_bytes);
  TableHeader header{};
  header.version = kTableVersion;
  header.scratch = kDotPartials;
  plan.table.assign(sizeof(TableHeader) / sizeof(int64_t), 0);
  header.dot_offset = static_cast<int64_t>(plan.table.size());
  header.dot_records = static_cast<int64_t>(dots.size());
  header.dot_units = units;
  Append(plan.table, dots);
  header.map_offset = header.group_offset = header.reduce_offset = static_cast<int64_t>(plan.table.size());
  std::memcpy(plan.table.data(), &header, sizeof(header));
  return plan;
}

// Grouped transform words (this engine's format; the reference builds pack
// and unpack records instead, _stride/_tensor_ops.py:119-203):
//   [1, source_size, output_size, groups,
//    per group: rank, n_src, n_dst, shape[rank],
//               n_src x (offset, strides[rank]),   source strides in the shape's axis order
//               n_dst x (offset, strides[rank])]
// Every address is bounds-checked; each destination must be injective and
// all destinations pairwise disjoint (the producer's "complete disjoint
// output selections").
Plan BuildGroupedPlan(const int64_t* words, std::size_t word_count, int32_t element_bytes, uint32_t flags) {
  if (words == nullptr && word_count != 0) throw InvalidArgument("grouped descriptor is null");
  std::size_t cursor = 0;
  auto next = [&]() {
    if (cursor == word_count) throw InvalidArgument("grouped descriptor is truncated");
    return words[cursor++];
  };
  auto size = [&]() {
    const int64_t value = next();
    if (value < 0) throw InvalidArgument("grouped size, count or offset is negative");
    return value;
  };
  if (next() != 1) throw InvalidArgument("unsupported grouped descriptor version");
  Plan plan;
  plan.operation = 5;
  plan.element_bytes = element_bytes;
  plan.flags = flags;
  plan.source_size = static_cast<uint64_t>(size());
  plan.output_size = static_cast<uint64_t>(size());
  const int64_t group_count = size();
  if (static_cast<uint64_t>(group_count) > (word_count - cursor) / 3) {
    throw InvalidArgument("grouped group count exceeds descriptor length");
  }
  std::vector<GroupedGroup> groups;
  std::vector<GroupedOperand> operands;
  std::vector<Record> destinations;
  int64_t units = 0, matrix = 0;
  uint64_t covered = 0, read = 0;
  auto pow2 = [](uint64_t n) { int32_t t = 1; while (t < 32 && static_cast<uint64_t>(t) < n) t <<= 1; return t; };
  for (int64_t index = 0; index < group_count; ++index) {
    const int64_t rank = size();
    const int64_t n_src = size();
    const int64_t n_dst = size();
    if (n_src < 1 || n_dst < 1) throw InvalidArgument("a group needs at least one source and one destination");
    if (n_src > 4096 || n_dst > 4096) throw InvalidArgument("groups are limited to 4096 sources and destinations");
    // The group needs rank shape words and (1 + rank) words per operand.
    const uint64_t operand_count = static_cast<uint64_t>(n_src + n_dst);
    const uint64_t remaining = word_count - cursor;
    if (remaining < operand_count || static_cast<uint64_t>(rank) > (remaining - operand_count) / (1 + operand_count)) {
      throw InvalidArgument("grouped rank exceeds descriptor length");
    }
    Record shape_record;
    shape_record.shape.resize(rank);
    for (auto& extent : shape_record.shape) extent = static_cast<uint64_t>(size());
    shape_record.fiber.assign(rank, 0);
    const uint64_t elements = ElementCount(shape_record);
    std::vector<Record> sides;   // sources (src_* fields), then destinations (dst_* fields)
    for (int64_t k = 0; k < n_src + n_dst; ++k) {
      Record side = shape_record;
      const bool source = k < n_src;
      const int64_t offset = size();
      std::vector<int64_t> strides(rank);
      for (auto& stride : strides) stride = next();
      if (source) { side.src_off = offset; side.sstr = strides; side.dstr.assign(rank, 0); }
      else { side.dst_off = offset; side.dstr = strides; side.sstr.assign(rank, 0); }
      CheckSide(side, source, source ? plan.source_size : plan.output_size, !source);
      sides.push_back(std::move(side));
    }
    matrix += n_src * n_dst;
    if (elements == 0) continue;
    for (int64_t k = n_src; k < n_src + n_dst; ++k) destinations.push_back(sides[k]);
    // Device axis order: extent-1 axes dropped, the first destination's
    // smallest stride innermost; neighbouring axes contiguous in every
    // operand fused.
    const Record& first = sides[n_src];
    std::vector<std::size_t> axes;
    for (std::size_t a = 0; a < shape_record.shape.size(); ++a) if (shape_record.shape[a] > 1) axes.push_back(a);
    std::stable_sort(axes.begin(), axes.end(), [&](std::size_t a, std::size_t b) {
      return AbsStride(first.dstr[a]) < AbsStride(first.dstr[b]);
    });
    auto stride_of = [&](const Record& side, bool source, std::size_t a) { return source ? side.sstr[a] : side.dstr[a]; };
    std::vector<uint64_t> extents;
    std::vector<std::vector<int64_t>> strides(n_src + n_dst);
    for (std::size_t a : axes) {
      bool fuse = !extents.empty();
      for (int64_t k = 0; k < n_src + n_dst && fuse; ++k) {
        fuse = stride_of(sides[k], k < n_src, a) == strides[k].back() * static_cast<int64_t>(extents.back());
      }
      if (fuse && extents.back() * shape_record.shape[a] <= kExtentLimit) {
        extents.back() *= shape_record.shape[a];
        continue;
      }
      extents.push_back(shape_record.shape[a]);
      for (int64_t k = 0; k < n_src + n_dst; ++k) strides[k].push_back(stride_of(sides[k], k < n_src, a));
    }
    if (extents.empty()) {
      extents.push_back(1);
      for (auto& list : strides) list.push_back(0);
    }
    if (extents.size() > static_cast<std::size_t>(kMaxRank)) {
      throw InvalidArgument("grouped blocks with more than eight non-unit axes are unsupported");
    }
    for (uint64_t extent : extents) {
      if (extent > kExtentLimit) throw InvalidArgument("grouped block extent exceeds 2^30");
    }
    // Tiled when the first source's smallest stride is not along X: Y, its
    // innermost axis, becomes axis 1.
    int y_axis = -1;
    if (extents.size() >= 2) {
      std::size_t best = 0;
      for (std::size_t a = 1; a < extents.size(); ++a) {
        if (AbsStride(strides[0][a]) < AbsStride(strides[0][best])) best = a;
      }
      if (best != 0) y_axis = static_cast<int>(best);
    }
    GroupedGroup g{};
    if (y_axis > 0) {
      const int32_t tx = pow2(extents[0]), ty = pow2(extents[y_axis]);
      // The third tile axis (the next axis in device order, if any) grows the
      // tile to at most 2048 elements while the stage stays small enough for
      // several CTAs per SM.
      int32_t tz = 1;
      const uint64_t z_extent = extents.size() >= 3 ? extents[y_axis == 1 ? 2 : 1] : 1;
      while (tz < 8 && static_cast<uint64_t>(tz) < z_extent && tx * ty * tz * 2 <= 2048 &&
             n_src * 2 * tz * ty * (tx + 1) * element_bytes <= kGroupedGrowBytes) {
        tz <<= 1;
      }
      const int64_t stage = n_src * tz * ty * (tx + 1);
      if (stage * element_bytes <= kGroupedStageBytes && n_src + n_dst <= kTiledOperands) {
        g.tiled = 1;
        g.tx = tx;
        g.ty = ty;
        g.tz = tz;
        plan.grouped_stage = std::max<uint64_t>(plan.grouped_stage, static_cast<uint64_t>(stage));
        auto move = [&](auto& list) {
          auto value = list[y_axis];
          list.erase(list.begin() + y_axis);
          list.insert(list.begin() + 1, value);
        };
        move(extents);
        for (auto& list : strides) move(list);
      }
    }
    g.unit_begin = units;
    g.elements = static_cast<int64_t>(elements);
    g.operand_begin = static_cast<int64_t>(operands.size());
    g.matrix_offset = matrix - n_src * n_dst;
    g.rank = static_cast<int32_t>(extents.size());
    g.n_src = static_cast<int32_t>(n_src);
    g.n_dst = static_cast<int32_t>(n_dst);
    for (int a = 0; a < kMaxRank; ++a) {
      g.n[a] = a < g.rank ? static_cast<int32_t>(extents[a]) : 1;
      g.div_n[a] = MakeDivision(static_cast<uint32_t>(g.n[a]));
    }
    int64_t group_units = CeilDiv(static_cast<int64_t>(elements), kGroupedTile);
    if (g.tiled) {
      g.tiles_x = static_cast<int32_t>(CeilDiv(g.n[0], g.tx));
      g.tiles_y = static_cast<int32_t>(CeilDiv(g.n[1], g.ty));
      g.tiles_z = static_cast<int32_t>(CeilDiv(g.n[2], g.tz));
      g.div_tiles_x = MakeDivision(static_cast<uint32_t>(g.tiles_x));
      g.div_tiles_y = MakeDivision(static_cast<uint32_t>(g.tiles_y));
      g.div_tiles_z = MakeDivision(static_cast<uint32_t>(g.tiles_z));
      group_units = static_cast<int64_t>(g.tiles_x) * g.tiles_y * g.tiles_z;
      for (int a = 3; a < g.rank; ++a) group_units *= g.n[a];
    }
    for (int64_t k = 0; k < n_src + n_dst; ++k) {
      GroupedOperand op{};
      op.offset = k < n_src ? sides[k].src_off : sides[k].dst_off;
      for (int a = 0; a < kMaxRank; ++a) op.s[a] = a < g.rank ? strides[k][a] : 0;
      operands.push_back(op);
    }
    units += group_units;
    if (units >= (int64_t{1} << 31)) throw std::runtime_error("a grouped transform spans more than 2^31 tiles per batch");
    covered += elements * static_cast<uint64_t>(n_dst);
    read += elements * static_cast<uint64_t>(n_src);
    groups.push_back(g);
  }
  if (cursor != word_count) throw InvalidArgument("grouped descriptor has trailing words");
  std::vector<const Record*> pointers;
  for (const Record& record : destinations) pointers.push_back(&record);
  if (!ProveDisjoint(pointers, plan.output_size)) {
    throw InvalidArgument("grouped destinations are not pairwise disjoint");
  }
  plan.records = static_cast<uint64_t>(group_count);
  plan.coefficient_rows = static_cast<uint64_t>(matrix);
  plan.grouped_units = static_cast<uint64_t>(units);
  plan.full_coverage = covered == plan.output_size;
  plan.bytes_moved = (read + plan.output_size) * static_cast<uint64_t>(element_bytes);
  TableHeader header{};
  header.version = kTableVersion;
  plan.table.assign(sizeof(TableHeader) / sizeof(int64_t), 0);
  header.grouped = static_cast<int64_t>(groups.size());
  header.grouped_offset = static_cast<int64_t>(plan.table.size());
  Append(plan.table, groups);
  header.operand_offset = static_cast<int64_t>(plan.table.size());
  Append(plan.table, operands);
  header.grouped_units = units;
  header.map_offset = header.group_offset = header.reduce_offset = header.dot_offset =
      static_cast<int64_t>(plan.table.size());
  std::memcpy(plan.table.data(), &header, sizeof(header));
  return plan;
}

}  // namespace

Plan BuildPlan(int32_t operation, const int64_t* words, std::size_t word_count,
               const int64_t* coefficient_records, std::size_t coefficient_count,
               int32_t element_bytes, uint32_t flags) {
  if (element_bytes != 4 && element_bytes != 8 && element_bytes != 16) {
    throw InvalidArgument("element size must be 4, 8 or 16 bytes");
  }
  if (operation == 2) {
    if (coefficient_count != 0) throw InvalidArgument("dot plans take no coefficient records");
    if ((flags & 4u) != 0) throw InvalidArgument("source conjugation is supported for accumulation and reduction plans");
    return BuildDotPlan(words, word_count, element_bytes, flags);
  }
  if (operation == 5) {
    if (coefficient_count != 0) throw InvalidArgument("grouped plans take their matrices at execution, not coefficient records");
    if (flags != 0) throw InvalidArgument("grouped plans take no flags");
    return BuildGroupedPlan(words, word_count, element_bytes, flags);
  }
  Layout layout;
  switch (operation) {
    case 0: case 1: layout = DecodeLayout(words, word_count, Validation::kMap); break;
    case 3: layout = DecodeLayout(words, word_count, Validation::kAccumulation); break;
    case 4: layout = DecodeReductionLayout(words, word_count); break;
    default: throw InvalidArgument("unsupported stride layout operation");
  }
  const bool summing = operation == 3 || operation == 4;
  if (!summing && coefficient_count != 0) {
    throw InvalidArgument("copy and update plans take no coefficient records");
  }
  if (!summing && (flags & 4u) != 0) {
    throw InvalidArgument("source conjugation is supported for accumulation and reduction plans");
  }
  std::vector<int64_t> slot(layout.records.size(), -1);
  int64_t previous = -1;
  for (std::size_t i = 0; i < coefficient_count; ++i) {
    const int64_t record = coefficient_records[i];
    if (record <= previous || record < 0 || static_cast<uint64_t>(record) >= layout.records.size()) {
      // The reference handlers' wording (accumulation.cu:64, reduction.cu:75).
      throw InvalidArgument(std::string("CUDA ") + (operation == 4 ? "reduction" : "accumulation") +
                            " coefficient records must be increasing valid record indices");
    }
    previous = record;
    slot[record] = static_cast<int64_t>(i);
  }

  Plan plan;
  plan.operation = operation;
  plan.element_bytes = element_bytes;
  plan.flags = flags;
  plan.source_size = layout.source_size;
  plan.output_size = layout.output_size;
  plan.records = layout.records.size();
  plan.coefficient_rows = coefficient_count;

  // Nonempty records in the reduce engine's canonical form (map axes ordered,
  // not fused), split to the device limits.  Records with the same owner map
  // share a key.
  struct Key {
    int64_t dst_off;
    std::vector<std::pair<uint64_t, int64_t>> axes;
    bool operator<(const Key& other) const {
      return std::tie(dst_off, axes) < std::tie(other.dst_off, other.axes);
    }
  };
  std::vector<Record> records;
  std::vector<int64_t> record_slot;
  for (const Record& original : layout.records) {
    if (ElementCount(original) == 0) continue;
    Record record = original;
    Canonicalize(record, false);
    for (Record& piece : SplitForDevice(record)) {
      records.push_back(std::move(piece));
      record_slot.push_back(slot[original.index]);
    }
  }
  std::map<Key, std::size_t> group_of;
  std::vector<std::vector<std::size_t>> group_members;
  std::vector<Key> group_keys;
  for (std::size_t i = 0; i < records.size(); ++i) {
    const Record& record = records[i];
    Key key{record.dst_off, {}};
    for (std::size_t a = 0; a < record.shape.size(); ++a) {
      if (!record.fiber[a]) key.axes.emplace_back(record.shape[a], record.dstr[a]);
    }
    auto found = group_of.find(key);
    if (found == group_of.end()) {
      found = group_of.emplace(key, group_members.size()).first;
      group_members.emplace_back();
      group_keys.push_back(key);
    }
    group_members[found->second].push_back(i);
  }

  // Distinct owner maps must be disjoint for concurrent execution: asserted
  // by the producer, or proven here.  Copy and update rely on the reference's
  // producer precondition of disjoint records.
  const bool asserted = (flags & 1u) != 0;
  bool disjoint = !summing || asserted;
  if (!disjoint) {
    std::vector<const Record*> maps;
    for (const auto& members : group_members) maps.push_back(&records[members.front()]);
    disjoint = ProveDisjoint(maps, plan.output_size);
  }

  // Engine selection: a record runs in the map engine when it has no summed
  // axes, is the only record of its owner map, and maps are disjoint.
  std::vector<std::size_t> map_ids;
  std::vector<std::size_t> reduce_groups;
  for (std::size_t g = 0; g < group_members.size(); ++g) {
    const auto& members = group_members[g];
    bool has_fiber = false;
    for (std::size_t i : members) {
      for (uint8_t f : records[i].fiber) has_fiber |= f != 0;
    }
    if (operation != 4 && disjoint && (!summing || (members.size() == 1 && !has_fiber))) {
      map_ids.insert(map_ids.end(), members.begin(), members.end());
    } else {
      reduce_groups.push_back(g);
    }
  }
  std::sort(map_ids.begin(), map_ids.end());

  // Map engine.
  std::vector<MapRecord> map_records;
  int64_t tiles = 0;
  uint64_t covered = 0;
  uint64_t read_elements = 0;
  for (std::size_t i : map_ids) {
    Record fused = records[i];
    Canonicalize(fused, true);
    MapRecord record = MakeMapRecord(fused, record_slot[i],
                                     (operation == 1 ? kUpdateTileBytes : kTileBytes) / element_bytes, tiles,
                                     operation == 1);
    tiles += MapTiles(record);
    plan.map_wide = plan.map_wide || NeedsWideOffsets(record);
    covered += ElementCount(records[i]);
    read_elements += ElementCount(records[i]);
    map_records.push_back(record);
  }

  // Reduce engine: groups in order of their first record; records keep their
  // semantic order within a group.
  std::vector<ReduceGroup> groups;
  std::vector<ReduceRecord> reduce_records;
  int64_t tasks = 0, owners = 0, scratch = 0;
  std::vector<const Record*> group_maps;
  for (std::size_t g : reduce_groups) {
    const Key& key = group_keys[g];
    ReduceGroup group{};
    group.dst_off = key.dst_off;
    group.rank = static_cast<int32_t>(key.axes.size());
    int64_t group_owners = 1;
    for (int a = 0; a < kMaxRank; ++a) { group.n[a] = 1; group.d[a] = 0; }
    for (std::size_t a = 0; a < key.axes.size(); ++a) {
      group.n[a] = static_cast<int32_t>(key.axes[a].first);
      group.d[a] = key.axes[a].second;
      group_owners *= static_cast<int64_t>(key.axes[a].first);
    }
    group.owners = group_owners;
    group.rec_begin = static_cast<int64_t>(reduce_records.size());
    uint64_t fiber_total = 0;
    for (std::size_t i : group_members[g]) {
      const Record& record = records[i];
      ReduceRecord rr{};
      rr.src_off = record.src_off;
      rr.coef_slot = static_cast<int32_t>(record_slot[i]);
      for (int a = 0; a < kMaxRank; ++a) { rr.n[a] = 1; rr.s[a] = 0; }
      int k = 0;
      uint64_t fiber_count = 1;
      for (std::size_t a = 0; a < record.shape.size(); ++a) {
        if (!record.fiber[a]) { rr.n[k] = static_cast<int32_t>(record.shape[a]); rr.s[k] = record.sstr[a]; ++k; }
      }
      rr.map_rank = k;
      for (std::size_t a = 0; a < record.shape.size(); ++a) {
        if (record.fiber[a]) {
          rr.n[k] = static_cast<int32_t>(record.shape[a]);
          rr.s[k] = record.sstr[a];
          fiber_count *= record.shape[a];
          ++k;
        }
      }
      if (fiber_count > static_cast<uint64_t>(std::numeric_limits<int32_t>::max())) {
        throw std::runtime_error("summed fibers longer than 2^31 elements are unsupported");
      }
      rr.fiber_rank = k - rr.map_rank;
      rr.fiber_count = static_cast<int32_t>(fiber_count);
      for (int a = 0; a < kMaxRank; ++a) rr.div_n[a] = MakeDivision(static_cast<uint32_t>(std::max(rr.n[a], 1)));
      fiber_total += fiber_count;
      read_elements += fiber_count * static_cast<uint64_t>(group_owners);
      reduce_records.push_back(rr);
    }
    group.rec_end = static_cast<int64_t>(reduce_records.size());
    const int64_t members = group.rec_end - group.rec_begin;
    const int64_t average = std::max<int64_t>(1, static_cast<int64_t>(fiber_total) / std::max<int64_t>(1, members));
    // Chunks of records sized for about 512 summed elements per warp task.
    // Short fibers (a trace's diagonals) are summed one record per lane, so a
    // warp's records are fetched in parallel rather than one after another.
    group.lanes_per_record = average < 32 ? 1 : 32;
    group.chunk_records = static_cast<int32_t>(std::clamp<int64_t>(
        group.lanes_per_record == 1 ? 32 : CeilDiv(512, average), 1, members));
    group.chunks = static_cast<int32_t>(CeilDiv(members, group.chunk_records));
    if (group.owners * group.chunks >= (int64_t{1} << 31)) {
      throw std::runtime_error("a reduction group has more than 2^31 (output, chunk) tasks");
    }
    group.div_owners = MakeDivision(static_cast<uint32_t>(group.owners));
    for (int a = 0; a < kMaxRank; ++a) group.div_n[a] = MakeDivision(static_cast<uint32_t>(std::max(group.n[a], 1)));
    group.task_begin = tasks;
    group.owner_begin = owners;
    group.scratch_off = scratch;
    tasks += group.owners * group.chunks;
    owners += group.owners;
    scratch += group.owners * group.chunks;
    covered += static_cast<uint64_t>(group.owners);
    groups.push_back(group);
    group_maps.push_back(&records[group_members[g].front()]);
  }

  // Waves of groups whose outputs are pairwise disjoint.
  if (!groups.empty()) {
    auto wave_for = [&](std::size_t begin, std::size_t end) {
      Wave wave{};
      wave.group_begin = static_cast<int64_t>(begin);
      wave.group_end = static_cast<int64_t>(end);
      wave.task_begin = groups[begin].task_begin;
      wave.owner_begin = groups[begin].owner_begin;
      wave.task_end = end < groups.size() ? groups[end].task_begin : tasks;
      wave.owner_end = end < groups.size() ? groups[end].owner_begin : owners;
      return wave;
    };
    if (disjoint) {
      plan.waves.push_back(wave_for(0, groups.size()));
    } else {
      for (std::size_t g = 0; g < groups.size(); ++g) plan.waves.push_back(wave_for(g, g + 1));
    }
  }

  if ((flags & 2u) != 0) plan.map_wide = true;
  plan.conjugate = (flags & 4u) != 0;
  plan.has_map = !map_records.empty();
  plan.has_reduce = !groups.empty();
  plan.map_tiles = static_cast<uint64_t>(tiles);
  plan.tasks = static_cast<uint64_t>(tasks);
  plan.owners = static_cast<uint64_t>(owners);
  plan.scratch = static_cast<uint64_t>(scratch);
  // Every output element is written by the map engine exactly once, or (a
  // trace's usual case) the reduce engine's owners cover the output exactly
  // once in one wave, so pass 2 assigns 0 + sum and no zeroing is needed.
  plan.reduce_assign = disjoint && plan.has_reduce && !plan.has_map && covered == plan.output_size;
  plan.full_coverage = (disjoint && !plan.has_reduce && covered == plan.output_size) || plan.reduce_assign;
  const uint64_t out_bytes = plan.output_size * element_bytes;
  plan.bytes_moved = read_elements * element_bytes + out_bytes + (operation == 1 ? out_bytes : 0);

  TableHeader header{};
  header.version = kTableVersion;
  header.map_records = static_cast<int64_t>(map_records.size());
  header.map_tiles = tiles;
  header.groups = static_cast<int64_t>(groups.size());
  header.reduce_records = static_cast<int64_t>(reduce_records.size());
  header.tasks = tasks;
  header.owners = owners;
  header.scratch = scratch;
  plan.table.assign(sizeof(TableHeader) / sizeof(int64_t), 0);
  header.map_offset = static_cast<int64_t>(plan.table.size());
  Append(plan.table, map_records);
  header.group_offset = static_cast<int64_t>(plan.table.size());
  Append(plan.table, groups);
  header.reduce_offset = static_cast<int64_t>(plan.table.size());
  Append(plan.table, reduce_records);
  std::memcpy(plan.table.data(), &header, sizeof(header));
  return plan;
}

}  // namespace t0b
