// The packed per-call descriptor table and the plan that owns its host copy.
//
// One table replaces the reference's per-record owner/fiber words
// (crates/tensor0-py/native/layout/descriptor.cc:237-290) and its one launch
// per record (crates/tensor0-cuda12/native/cuda/execute/sum.cuh:15-57):
//
//   map engine    — injective, mutually disjoint records without summed axes
//                   (copy, permute-accumulate, update).  Each record is cut
//                   into tiles: a box over its destination-innermost axis X,
//                   its source-innermost axis Y and one more destination axis
//                   Z; the remaining axes are enumerated per tile.  A tile is
//                   staged through shared memory so both the reads and the
//                   writes are coalesced.  All tiles of all records form one
//                   grid.
//   reduce engine — records with summed (fiber) axes or shared outputs
//                   (partial trace, general accumulation).  Records with the
//                   same output map form a group; pass 1 reduces chunks of a
//                   group's records per output owner with warp shuffles into
//                   scratch, pass 2 combines the chunks in record order.
#pragma once

#include <cstdint>
#include <vector>

namespace t0b {

constexpr int kMaxRank = 8;

// Constants for dividing 32-bit values below 2^31 by a fixed divisor d >= 1:
// n / d = (umulhi(n, magic) + n) >> shift with shift = ceil(log2 d) and
// magic = floor(2^32 (2^shift - d) / d) + 1 (the round-up multiplier method).
struct DivisionConstants {
  uint32_t magic;
  uint32_t shift;
};

inline DivisionConstants MakeDivision(uint32_t divisor) {
  uint32_t shift = 0;
  while ((uint64_t{1} << shift) < divisor) ++shift;
  const uint64_t magic = ((uint64_t{1} << 32) * ((uint64_t{1} << shift) - divisor)) / divisor + 1;
  return DivisionConstants{static_cast<uint32_t>(magic), shift};
}

// Map-engine record (device layout; shared by host and device code).
struct alignas(16) MapRecord {
  int64_t src_off;
  int64_t dst_off;
  int64_t tile_begin;   // first tile of this record within one batch
  int64_t s[kMaxRank];  // source strides:      X, Y, Z, outer...
  int64_t d[kMaxRank];  // destination strides: X, Y, Z, outer...
  int32_t n[kMaxRank];  // extents:             X, Y, Z, outer...
  int32_t t[3];         // tile extents of X, Y, Z
  int32_t c[3];         // chunks along X, Y, Z
  int32_t nouter;       // outer axes after the three box axes
  int32_t mode;         // kTranspose or kDirect
  int32_t coef_slot;    // coefficient row, or -1 for factor one
  int32_t pad_;
  // Splitting a tile index: division by c[0], c[1], c[2], then by n[3], n[4], ...
  DivisionConstants div_tiles[kMaxRank];
  // Extents of the last tile along X and Y, and division by t[0], edge[0], t[1], edge[1].
  int32_t edge[2];
  DivisionConstants div_extent[4];
  int32_t pad2_[2];
};

// kTranspose: the general run walk of a transposing tile.  kDirect: X is
// innermost on both sides.  kRect: a transposing tile whose X has unit
// destination stride and Y unit source stride, both at least kRectMinExtent
// long: walked with a fixed thread map (lanes along Y to load, along X to
// store) and no run lists.
enum MapMode : int32_t { kTranspose = 0, kDirect = 1, kRect = 2 };


// Reduce-engine group of records that write the same output map.
struct alignas(16) ReduceGroup {
  int64_t dst_off;
  int64_t d[kMaxRank];  // destination strides of the map (owner) axes
  int32_t n[kMaxRank];  // extents of the map axes
  int32_t rank;         // map axes
  int32_t chunks;       // record chunks (pass-1 partials per owner)
  int64_t owners;
  int64_t rec_begin;    // [rec_begin, rec_end) in the ReduceRecord array
  int64_t rec_end;
  int64_t task_begin;   // first pass-1 task (one task = one owner x one chunk)
  int64_t owner_begin;  // prefix of owners over groups (pass-2 threads)
  int64_t scratch_off;  // partial of (chunk, owner) at scratch_off + chunk * owners + owner
  int32_t chunk_records;
  int32_t lanes_per_record;              // 32: lanes stride one record's fiber; 1: each lane sums whole records
  DivisionConstants div_owners;          // task -> (chunk, owner)
  DivisionConstants div_n[kMaxRank];     // owner -> map indices
};

struct alignas(16) ReduceRecord {
  int64_t src_off;
  int64_t s[kMaxRank];  // source strides: map axes (group order) then fiber axes
  int32_t n[kMaxRank];  // extents: map axes then fiber axes
  int32_t map_rank;
  int32_t fiber_rank;
  int32_t coef_slot;
  int32_t fiber_count;
  DivisionConstants div_n[kMaxRank];     // fiber index -> fiber axis indices (fiber axes only)
};

// Dot record: axis 0 (the smallest right stride after canonicalisation) is
// the row walked by a warp in chunks of `chunk` elements; a unit is one chunk
// of one row.
struct alignas(16) DotRecord {
  int64_t left_off;
  int64_t right_off;
  int64_t unit_begin;       // first unit of this record within one batch
  int64_t sl[kMaxRank];     // left strides, axis 0 first
  int64_t sr[kMaxRank];     // right strides
  int32_t n[kMaxRank];      // extents
  int32_t rank;
  int32_t chunk;            // elements of a row per unit
  int32_t chunks;           // units per row
  int32_t pad_;
  DivisionConstants div[kMaxRank];   // unit -> (chunk, row index): by chunks, then n[1], n[2], ...
};

// Partial sums per batch of the dot engine's first pass.
constexpr int64_t kDotPartials = 1184;

// Grouped transform: a group maps n_src source blocks of one logical shape
// through an [n_dst][n_src] matrix to n_dst destination blocks.  Axes are in
// the device order: axis 0 (X) has the smallest destination stride.  An
// element group's unit is kGroupedTile consecutive block elements, one per
// thread.  A tiled group (one whose first source is not innermost along X)
// puts the source's innermost axis second (Y); its unit is a tx x ty x tz
// tile of (X, Y, axis 2) at one index of the remaining axes, read along Y
// into shared memory and written along X out of it.
constexpr int32_t kGroupedTile = 256;
constexpr int64_t kGroupedStageBytes = 96 * 1024;   // shared memory of one tiled unit, at most
constexpr int64_t kGroupedGrowBytes = 40 * 1024;    // the third tile axis grows while the stage fits this
constexpr int32_t kTiledOperands = 64;              // sources + destinations of a tiled group, at most

struct alignas(16) GroupedGroup {
  int64_t unit_begin;       // first unit of this group within one batch
  int64_t elements;         // block elements
  int64_t operand_begin;    // first GroupedOperand: n_src sources, then n_dst destinations
  int64_t matrix_offset;    // element offset of the group's row-major [n_dst][n_src] matrix
  int32_t n[kMaxRank];      // extents
  int32_t rank;
  int32_t n_src;
  int32_t n_dst;
  int32_t tiled;            // 1: staged (X, Y, Z) tiles
  int32_t tx, ty, tz;       // tile extents (powers of two; tx, ty at most 32, tz at most 8)
  int32_t tiles_x, tiles_y, tiles_z;
  DivisionConstants div_n[kMaxRank];   // element (or, tiled, remaining-axes index) -> axis indices
  DivisionConstants div_tiles_x;
  DivisionConstants div_tiles_y;
  DivisionConstants div_tiles_z;
  int32_t pad_[2];
};

struct alignas(16) GroupedOperand {
  int64_t offset;
  int64_t s[kMaxRank];      // strides in the group's axis order
};

struct TableHeader {
  int64_t version;          // kTableVersion
  int64_t map_records;
  int64_t map_tiles;        // tiles per batch
  int64_t map_offset;       // word offset of the MapRecord array
  int64_t groups;
  int64_t group_offset;
  int64_t reduce_records;
  int64_t reduce_offset;
  int64_t tasks;            // pass-1 tasks per batch
  int64_t owners;           // pass-2 threads per batch
  int64_t scratch;          // scratch elements per batch
  int64_t dot_records;
  int64_t dot_offset;
  int64_t dot_units;        // units per batch
  int64_t grouped;          // grouped-transform groups
  int64_t grouped_offset;   // word offset of the GroupedGroup array
  int64_t operand_offset;   // word offset of the GroupedOperand array
  int64_t grouped_units;    // units per batch
};

constexpr int64_t kTableVersion = 0x7430620003;

struct Wave {               // consecutive groups that may run concurrently
  int64_t group_begin, group_end;
  int64_t task_begin, task_end;
  int64_t owner_begin, owner_end;
};

struct Plan {
  int32_t operation = 0;
  int32_t element_bytes = 0;
  uint32_t flags = 0;
  uint64_t source_size = 0;
  uint64_t output_size = 0;
  uint64_t records = 0;
  uint64_t coefficient_rows = 0;
  bool full_coverage = false;    // every output element is written exactly once (no zeroing first)
  bool reduce_assign = false;    // the reduce engine's owners alone cover the output once: pass 2 assigns
  bool has_map = false;
  bool has_reduce = false;
  bool map_wide = false;         // some tile needs 64-bit in-tile offsets
  bool conjugate = false;        // read the complex conjugate of the source
  uint64_t map_tiles = 0;
  uint64_t tasks = 0;
  uint64_t owners = 0;
  uint64_t scratch = 0;
  uint64_t bytes_moved = 0;      // algorithmic bytes of one batch
  uint64_t dot_units = 0;        // dot plans: work units per batch
  uint64_t grouped_units = 0;    // grouped plans: work units per batch
  uint64_t grouped_stage = 0;    // grouped plans: shared-memory elements of a tiled unit
  std::vector<Wave> waves;       // reduce-engine waves, in order
  std::vector<int64_t> table;    // packed device table (host words)
};

// Build a plan; throws InvalidArgument / std::runtime_error.
Plan BuildPlan(int32_t operation, const int64_t* words, std::size_t word_count,
               const int64_t* coefficient_records, std::size_t coefficient_count,
               int32_t element_bytes, uint32_t flags);

}  // namespace t0b
