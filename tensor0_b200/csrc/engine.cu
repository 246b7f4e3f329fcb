// Map and reduce engines: the grouped strided permute / accumulate / update
// kernel and the two-pass segmented reduction for partial traces.
//
// The map kernel is one persistent grid over every tile of every record of
// every batch; each CTA walks a contiguous range of tiles.  A tile is a box
// over the record's destination-innermost axis X, its source-innermost axis Y
// and one further axis Z.  One thread decodes the tile with host-computed
// division constants into two run lists: the source runs (along Y, continued
// by Z when Z follows Y in the source), copied asynchronously into a
// destination-ordered shared-memory tile, and the destination runs (rows
// along X, or whole (x, y) planes when they are contiguous on both sides),
// written out of it.  Warps take runs with constant address increments and
// lanes stride each run, so reads and writes are coalesced and an element
// costs its memory instruction and an addition or two.
#include "engine.h"

#include "arith.cuh"
#include "copy_async.cuh"

#include <algorithm>
#include <atomic>

namespace t0b {

std::atomic<uint64_t> g_kernel_launches{0};

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
// Map CTA shape per operation (threads, CTAs per SM the register budget is
// sized for).  Copy and accumulation do best with small CTAs, whose barriers
// span few warps; update, which stages two operands, with larger ones and more
// registers.
#ifndef T0B_PERMUTE_THREADS
#define T0B_PERMUTE_THREADS 128
#endif
#ifndef T0B_PERMUTE_MIN_BLOCKS
#define T0B_PERMUTE_MIN_BLOCKS 8
#endif
#ifndef T0B_UPDATE_THREADS
#define T0B_UPDATE_THREADS 256
#endif
#ifndef T0B_UPDATE_MIN_BLOCKS
#define T0B_UPDATE_MIN_BLOCKS 3
#endif


// "Division" by 2^31: every run index of a single-plane run list is in plane 0.
constexpr FastDiv kSinglePlane{0, 31};

// The runs one phase of a tile copies: run (a, b), a in [0, na), b in
// [0, nb), starts at global offset a * ga + b * gb and shared-memory index
// a * sa + b * sb; its element j in [0, len) sits at + j * gj and + j * sj.
template <typename Off>
struct Runs {
  Off ga, gb, gj;
  int sa, sb, sj;
  int na, nb, len;
  FastDiv by_na;           // run index -> b
  FastDiv by_len;          // element index -> run (packed short runs only)
};

// A decoded tile, shared by the CTA.  In-tile offsets use Off (int32 unless
// the plan marked a record wide).  Shared memory holds the tile in
// destination order: element (x, y, z) at x + px * y + pz * z, px = ex | 1
// (odd, so source runs, which step px, hit distinct banks) and pz = px * ey.
// A rectangular tile (MapMode kRect): box ex x ey x ez, source element
// (x, y, z) at x * sx + y + z * sz, destination at x + y * dy + z * dz.
template <typename Off>
struct RectBox {
  int ex, ey, ez, px, pz;
  Off sx, sz, dy, dz;
};

template <typename Off>
struct TileState {
  int64_t so, dof;        // element offsets of the tile origin, batch included
  Runs<Off> load;         // source runs into shared memory
  Runs<Off> store;        // destination runs out of shared memory (also the update's base loads)
  RectBox<Off> box;       // rectangular tiles: the fixed thread map's box (runs unused)
  int64_t batch;
  int slot;
  int rect;
  alignas(16) unsigned char coef[32];   // the tile's coefficients, fetched by the decoding thread
};

// Thread 0 only: decode tile `local` of record `r` in `batch`.
template <typename Off, int kThreadsPerCta>
__device__ __forceinline__ void DecodeTile(const MapArgs& a, const MapRecord& r, int64_t batch, int64_t local,
                                           TileState<Off>& s) {
  uint32_t q = static_cast<uint32_t>(local - r.tile_begin);
  uint32_t chunk[3];
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    const uint32_t next = Division(r.div_tiles[i]).Div(q);
    chunk[i] = q - next * static_cast<uint32_t>(r.c[i]);
    q = next;
  }
  int64_t so = r.src_off + batch * a.src_size;
  int64_t dof = r.dst_off + batch * a.out_size;
  for (int i = 0; i < r.nouter; ++i) {
    const uint32_t next = Division(r.div_tiles[3 + i]).Div(q);
    const int64_t idx = q - next * static_cast<uint32_t>(r.n[3 + i]);
    q = next;
    so += idx * r.s[3 + i];
    dof += idx * r.d[3 + i];
  }
  const bool last_x = static_cast<int>(chunk[0]) == r.c[0] - 1;
  const bool last_y = static_cast<int>(chunk[1]) == r.c[1] - 1;
  const int ex = last_x ? r.edge[0] : r.t[0];
  const int ey = last_y ? r.edge[1] : r.t[1];
  const int z0 = static_cast<int>(chunk[2]) * r.t[2];
  const int ez = min(r.t[2], r.n[2] - z0);
  const int64_t x0 = static_cast<int64_t>(chunk[0]) * r.t[0], y0 = static_cast<int64_t>(chunk[1]) * r.t[1];
  s.so = so + x0 * r.s[0] + y0 * r.s[1] + z0 * r.s[2];
  s.dof = dof + x0 * r.d[0] + y0 * r.d[1] + z0 * r.d[2];
  const Off sx = static_cast<Off>(r.s[0]), sy = static_cast<Off>(r.s[1]), sz = static_cast<Off>(r.s[2]);
  const Off dx = static_cast<Off>(r.d[0]), dy = static_cast<Off>(r.d[1]), dz = static_cast<Off>(r.d[2]);
  const int px = ex | 1, pz = px * ey;
  s.batch = batch;
  s.slot = r.coef_slot;
  s.rect = r.mode == kRect;
  if (s.rect) {
    s.box = RectBox<Off>{ex, ey, ez, px, pz, sx, sz, dy, dz};
    return;
  }
  const FastDiv by_x = Division(r.div_extent[last_x ? 1 : 0]);
  const FastDiv by_y = Division(r.div_extent[last_y ? 3 : 2]);
  // Destination: when (x, y) is contiguous on both sides (an odd ex needs no
  // padding) each z plane is one run, else (y, z) rows of ex.
  Runs<Off>& w = s.store;
  if (ey > 1 && px == ex && r.d[1] == static_cast<int64_t>(ex) * r.d[0] && ex * ey >= kThreadsPerCta) {
    w = Runs<Off>{dz, 0, dx, pz, 0, 1, ez, 1, ex * ey, kSinglePlane, FastDiv{0, 0}};
  } else {
    w = Runs<Off>{dy, dz, dx, px, pz, 1, ey, ez, ex, by_y, by_x};
  }
  // Source.
  Runs<Off>& l = s.load;
  if (r.mode == kDirect) {
    // X is innermost on both sides: the source runs are the destination rows.
    l = Runs<Off>{sy, sz, sx, px, pz, 1, ey, ez, ex, by_y, by_x};
  } else if (ez > 1 && r.s[2] == static_cast<int64_t>(ey) * r.s[1] && ex >= kThreadsPerCta / 32 && ey * ez >= 32) {
    // Z continues Y in the source (and, as pz = px * ey, in shared memory).
    l = Runs<Off>{sx, 0, sy, 1, 0, px, ex, 1, ey * ez, kSinglePlane, FastDiv{0, 0}};
  } else {
    l = Runs<Off>{sx, sz, sy, 1, pz, px, ex, ez, ey, by_x, by_y};
  }
}

// Per-operation element rule applied when a value reaches the destination.
// Fetch (decoding thread) stages the tile's coefficients in shared memory;
// the constructor reads them back.  Kind() selects a specialised store loop:
// 1 and 2 are the common unit cases, 0 the general rule.
template <int Op, typename T, typename CA, typename CB>
struct Emit;

// Copy: bit-preserving move (T is an unsigned storage type).
template <typename T, typename CA, typename CB>
struct Emit<kOpCopy, T, CA, CB> {
  static constexpr bool kReadsBase = false;
  __device__ static void Fetch(const MapArgs&, int, int64_t, unsigned char*) {}
  __device__ __forceinline__ explicit Emit(const unsigned char*) {}
  __device__ __forceinline__ bool SkipSource() const { return false; }
  __device__ __forceinline__ bool NeedsBase() const { return false; }
  __device__ __forceinline__ int Kind() const { return 1; }
  template <int K> __device__ __forceinline__ T Apply(T v, T) const { return v; }
};

// Accumulation into a zeroed output: 0 + c * v, with the zero / one rules.
template <typename T, typename CA, typename CB>
struct Emit<kOpAccumulation, T, CA, CB> {
  static constexpr bool kReadsBase = false;
  using Real = typename Elem<T>::Real;
  using C = typename BoundOf<Real, CA>::type;
  struct Staged { C c; int present; };
  C c;
  bool zero, one;
  __device__ static void Fetch(const MapArgs& a, int slot, int64_t batch, unsigned char* out) {
    Staged s{C{}, slot >= 0};
    if (slot >= 0) s.c = ReadCoefficient<Real>(static_cast<const CA*>(a.ca), slot, a.ca_count, batch);
    *reinterpret_cast<Staged*>(out) = s;
  }
  __device__ __forceinline__ explicit Emit(const unsigned char* staged) {
    const Staged s = *reinterpret_cast<const Staged*>(staged);
    c = s.c;
    zero = s.present && IsZero(c);
    one = !s.present || IsOne(c);
  }
  __device__ __forceinline__ bool SkipSource() const { return zero; }
  __device__ __forceinline__ bool NeedsBase() const { return false; }
  __device__ __forceinline__ int Kind() const { return zero ? 2 : (one ? 1 : 0); }
  template <int K> __device__ __forceinline__ T Apply(T v, T) const {
    if constexpr (K == 2) return Zero<T>();
    else if constexpr (K == 1) return PlusZero(v);
    else return PlusZero(Scale(c, v));
  }
};

// Update: alpha * src + beta * base with the reference's short-circuits.
template <typename T, typename CA, typename CB>
struct Emit<kOpUpdate, T, CA, CB> {
  static constexpr bool kReadsBase = true;
  using Real = typename Elem<T>::Real;
  using A = typename BoundOf<Real, CA>::type;
  using B = typename BoundOf<Real, CB>::type;
  A a; B b;
  bool a0, a1, b0, b1;
  __device__ static void Fetch(const MapArgs& args, int, int64_t batch, unsigned char* out) {
    *reinterpret_cast<A*>(out) = ReadCoefficient<Real>(static_cast<const CA*>(args.ca), 0, args.ca_count, batch);
    *reinterpret_cast<B*>(out + 16) = ReadCoefficient<Real>(static_cast<const CB*>(args.cb), 0, args.cb_count, batch);
  }
  __device__ __forceinline__ explicit Emit(const unsigned char* staged) {
    a = *reinterpret_cast<const A*>(staged);
    b = *reinterpret_cast<const B*>(staged + 16);
    a0 = IsZero(a); a1 = IsOne(a); b0 = IsZero(b); b1 = IsOne(b);
  }
  __device__ __forceinline__ bool SkipSource() const { return a0; }
  __device__ __forceinline__ bool NeedsBase() const { return !b0; }
  __device__ __forceinline__ int Kind() const { return (a1 && b1) ? 1 : ((a1 && b0) ? 2 : 0); }
  template <int K> __device__ __forceinline__ T Apply(T v, T old) const {
    if constexpr (K == 1) {
      return Add(v, old);
    } else if constexpr (K == 2) {
      return v;
    } else {
      if (a0) {
        if (b0) return Zero<T>();
        return b1 ? old : Scale(b, old);
      }
      const T s = a1 ? v : Scale(a, v);
      if (b0) return s;
      return Add(s, b1 ? old : Scale(b, old));
    }
  }
};

// This thread's elements j = first_j, first_j + kStep, ... of one run
// (first_j < kStep): element j's global address is p + (j - first_j) * gj and
// its shared-memory byte address s + (j - first_j) / kStep * ss.  The number
// of unrolled blocks is the same for every thread of the warp, and the last
// up-to-four elements are predicated, so lanes never split between the two
// paths.  kG is the global step when known at compile time (1: unit stride,
// the usual case) and kSs the shared-memory step of kStep elements (or 0 for
// ss); known steps become immediate address offsets.
template <typename P, typename Off, int kG, int kSs, int kStep, typename ElemF>
__device__ __forceinline__ void RunElements(P p, uint32_t s, int j, int len, Off gj, uint32_t ss_runtime,
                                            ElemF& elem) {
  const Off gs = kStep * (kG != 0 ? static_cast<Off>(kG) : gj);
  const uint32_t ss = kSs != 0 ? static_cast<uint32_t>(kSs) : ss_runtime;
  for (int block = len / (4 * kStep); block > 0; --block, j += 4 * kStep, p += 4 * gs, s += 4 * ss) {
    elem(p, s);
    elem(p + gs, s + ss);
    elem(p + 2 * gs, s + 2 * ss);
    elem(p + 3 * gs, s + 3 * ss);
  }
  if (j < len) elem(p, s);
  if (j + kStep < len) elem(p + gs, s + ss);
  if (j + 2 * kStep < len) elem(p + 2 * gs, s + 2 * ss);
  if (j + 3 * kStep < len) elem(p + 3 * gs, s + 3 * ss);
}

// Runs taken kLanes lanes at a time: each warp step covers 32 / kLanes runs
// of the flattened (a, b) order, and each lane group strides its run.  Short
// runs get few lanes, so every lane handles several elements and the per-run
// set-up is amortised; a warp access still covers whole 32-byte sectors.
// kSUnit: the run's shared-memory step is one element.
template <typename P, typename Off, int kG, bool kSUnit, int kLanes, int kThreadsPerCta, typename ElemF>
__device__ __forceinline__ void GroupRuns(const Runs<Off>& w, P base, uint32_t sbase, ElemF& elem) {
  constexpr int kGroups = 32 / kLanes;
  constexpr uint32_t kBytes = sizeof(*base);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = lane % kLanes, group = lane / kLanes;
  const Off g1 = kG != 0 ? static_cast<Off>(kG) : w.gj;
  const int runs = w.na * w.nb;
  const uint32_t ss = static_cast<uint32_t>(kLanes * w.sj) * kBytes;
  for (int r0 = warp * kGroups; r0 < runs; r0 += (kThreadsPerCta / 32) * kGroups) {
    const int r = r0 + group;
    if (r < runs) {
      const int b = static_cast<int>(w.by_na.Div(static_cast<uint32_t>(r)));
      const int a = r - b * w.na;
      RunElements<P, Off, kG, kSUnit ? kLanes * kBytes : 0, kLanes>(
          base + (a * w.ga + b * w.gb + sub * g1), sbase + static_cast<uint32_t>(a * w.sa + b * w.sb + sub * w.sj) * kBytes,
          sub, w.len, w.gj, ss, elem);
    }
  }
}

// Walk every element of a phase's runs; elem(p, s) moves the element at
// global address p and shared-memory byte address s.  The CTA's threads are
// spread so every warp has work:
//   * few runs of at least a CTA's length: the whole CTA strides each run;
//   * runs of 8 or more: 8, 16 or 32 lanes per run (by length), see GroupRuns;
//   * shorter runs:      packed end to end, the threads stride the sequence.
template <typename P, typename Off, int kG, bool kSUnit, int kThreadsPerCta, typename ElemF>
__device__ __forceinline__ void WalkRuns(const Runs<Off>& w, P base, uint32_t sbase, ElemF& elem) {
  constexpr uint32_t kBytes = sizeof(*base);
  const int tid = threadIdx.x;
  const int len = w.len;
  if (len >= kThreadsPerCta && w.na * w.nb < kThreadsPerCta / 32) {
    const Off g1 = kG != 0 ? static_cast<Off>(kG) : w.gj;
    const uint32_t ss = static_cast<uint32_t>(kThreadsPerCta * w.sj) * kBytes;
    for (int b = 0; b < w.nb; ++b) {
      for (int a = 0; a < w.na; ++a) {
        RunElements<P, Off, kG, kSUnit ? kThreadsPerCta * kBytes : 0, kThreadsPerCta>(
            base + (a * w.ga + b * w.gb + tid * g1), sbase + static_cast<uint32_t>(a * w.sa + b * w.sb + tid * w.sj) * kBytes,
            tid, len, w.gj, ss, elem);
      }
    }
  } else if (len > 128) {
    GroupRuns<P, Off, kG, kSUnit, 32, kThreadsPerCta>(w, base, sbase, elem);
  } else if (len > 64) {
    GroupRuns<P, Off, kG, kSUnit, 16, kThreadsPerCta>(w, base, sbase, elem);
  } else if (len >= 8) {
    GroupRuns<P, Off, kG, kSUnit, 8, kThreadsPerCta>(w, base, sbase, elem);
  } else {
    const int total = w.na * w.nb * len;
    for (int f = tid; f < total; f += kThreadsPerCta) {
      const int r = static_cast<int>(w.by_len.Div(static_cast<uint32_t>(f)));
      const int j = f - r * len;
      const int b = static_cast<int>(w.by_na.Div(static_cast<uint32_t>(r)));
      const int a = r - b * w.na;
      elem(base + (a * w.ga + b * w.gb + j * w.gj), sbase + static_cast<uint32_t>(a * w.sa + b * w.sb + j * w.sj) * kBytes);
    }
  }
}

// `runs` lives in shared memory; the walk uses a register copy, which stores
// through generic pointers cannot alias.
template <typename Off, int kThreadsPerCta, bool kSUnit, typename P, typename ElemF>
__device__ __forceinline__ void Walk(const Runs<Off>& runs, P base, uint32_t sbase, ElemF&& elem) {
  const Runs<Off> w = runs;
  if (w.gj == 1) WalkRuns<P, Off, 1, kSUnit, kThreadsPerCta>(w, base, sbase, elem);
  else WalkRuns<P, Off, 0, kSUnit, kThreadsPerCta>(w, base, sbase, elem);
}

// Shared-memory load of one element at a byte address.  Volatile, so it stays
// after the CTA barrier that publishes the tile.
template <typename T>
__device__ __forceinline__ T LoadShared(uint32_t addr) {
  T v;
  if constexpr (sizeof(T) == 4) {
    uint32_t x;
    asm volatile("ld.shared.b32 %0, [%1];\n" : "=r"(x) : "r"(addr));
    __builtin_memcpy(&v, &x, 4);
  } else if constexpr (sizeof(T) == 8) {
    uint2 x;
    asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];\n" : "=r"(x.x), "=r"(x.y) : "r"(addr));
    __builtin_memcpy(&v, &x, 8);
  } else {
    uint4 x;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];\n" : "=r"(x.x), "=r"(x.y), "=r"(x.z), "=r"(x.w) : "r"(addr));
    __builtin_memcpy(&v, &x, 16);
  }
  return v;
}



// Rectangular tiles.  Every element of the box goes through shared memory at
// x + px * y + pz * z.  Loads: lane l takes y = l and l + 32 (consecutive
// source addresses, and shared-memory words px apart: distinct banks as px is
// odd), warps take rows x.  Stores: lane l takes x = l and l + 32, warps take
// rows y.  Both halves of a row are issued back to back, and each thread walks
// its rows with constant pointer steps.
template <int kCta, typename T, typename Off, typename Move>
__device__ __forceinline__ void RectRows(int lanes_extent, int rows_extent, int ez, Off row_step, Off z_step,
                                         int s_lane, int s_row, int s_z, T* base, uint32_t sbase, Move&& move) {
  constexpr int kW = kCta / 32;
  constexpr uint32_t B = sizeof(T);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane >= lanes_extent) return;
  const bool second = lane + 32 < lanes_extent;
  const Off row_w = row_step * kW;
  const uint32_t srow_w = static_cast<uint32_t>(s_row * kW) * B;
  const uint32_t s_half = static_cast<uint32_t>(32 * s_lane) * B;
  for (int z = 0; z < ez; ++z) {
    T* g = base + (z * z_step + warp * row_step + lane);
    uint32_t sm = sbase + static_cast<uint32_t>(s_z * z + s_row * warp + s_lane * lane) * B;
    int row = warp;
    if (lanes_extent > 32) {
      for (; row + kW < rows_extent; row += 2 * kW) {
        move(g, sm);
        if (second) move(g + 32, sm + s_half);
        move(g + row_w, sm + srow_w);
        if (second) move(g + row_w + 32, sm + srow_w + s_half);
        g += 2 * row_w;
        sm += 2 * srow_w;
      }
      if (row < rows_extent) {
        move(g, sm);
        if (second) move(g + 32, sm + s_half);
      }
    } else {
      for (; row + 3 * kW < rows_extent; row += 4 * kW) {
        move(g, sm);
        move(g + row_w, sm + srow_w);
        move(g + 2 * row_w, sm + 2 * srow_w);
        move(g + 3 * row_w, sm + 3 * srow_w);
        g += 4 * row_w;
        sm += 4 * srow_w;
      }
      for (; row < rows_extent; row += kW) {
        move(g, sm);
        g += row_w;
        sm += srow_w;
      }
    }
  }
}

// Source rows (lanes along Y, rows along X) into the tile.
template <int kCta, typename T, typename Off, typename Move>
__device__ __forceinline__ void RectSourceRows(const RectBox<Off>& b, T* src, uint32_t tile_s, Move&& move) {
  RectRows<kCta, T, Off>(b.ey, b.ex, b.ez, b.sx, b.sz, b.px, 1, b.pz, src, tile_s, move);
}

// Destination rows (lanes along X, rows along Y) of the tile.
template <int kCta, typename T, typename Off, typename Move>
__device__ __forceinline__ void RectDestinationRows(const RectBox<Off>& b, T* dst, uint32_t tile_s, Move&& move) {
  RectRows<kCta, T, Off>(b.ex, b.ey, b.ez, b.dy, b.dz, 1, b.px, b.pz, dst, tile_s, move);
}

// Issue the asynchronous loads of one tile: the source runs into the tile
// and, for update, the destination's base values into the same positions of
// the base buffer.
template <typename E, typename T, typename Off, int kThreadsPerCta>
__device__ __forceinline__ void LoadTile(const MapArgs& args, const TileState<Off>& st, uint32_t tile_s,
                                         uint32_t base_s) {
  const E emit(st.coef);
  auto copy = [](const T* p, uint32_t s) { CopyAsync<sizeof(T)>(s, p); };
  if (st.rect) {
    const RectBox<Off> box = st.box;
    if (!emit.SkipSource()) {
      RectSourceRows<kThreadsPerCta>(box, static_cast<const T*>(args.src) + st.so, tile_s, copy);
    }
    if constexpr (E::kReadsBase) {
      if (emit.NeedsBase()) {
        RectDestinationRows<kThreadsPerCta>(box, static_cast<const T*>(args.base) + st.dof, base_s, copy);
      }
    }
    return;
  }
  if (!emit.SkipSource()) {
    Walk<Off, kThreadsPerCta, false>(st.load, static_cast<const T*>(args.src) + st.so, tile_s, copy);
  }
  if constexpr (E::kReadsBase) {
    if (emit.NeedsBase()) Walk<Off, kThreadsPerCta, true>(st.store, static_cast<const T*>(args.base) + st.dof, base_s, copy);
  }
}

// The decoding thread's position: the current record, copied into shared
// memory once per record (a CTA walks a contiguous tile range, so records
// change rarely), the next record's first tile, and the coefficients of the
// current (record, batch).  Decoding a tile then reads no global memory.
struct alignas(16) MapCursor {
  MapRecord rec;
  int64_t rec_index;
  int64_t next_begin;     // first tile of record rec_index + 1 (or past the end)
  int64_t batch;
  int64_t local;          // tile within the batch
  int64_t coef_batch;     // batch the staged coefficients belong to (-1: none)
  int64_t pad_;
  alignas(16) unsigned char coef[32];
};

__device__ __forceinline__ void LoadRecord(const MapArgs& args, int64_t index, MapCursor& c) {
  static_assert(sizeof(MapRecord) % 16 == 0, "records are copied in 16-byte words");
  const int4* from = reinterpret_cast<const int4*>(args.recs + index);
  int4* to = reinterpret_cast<int4*>(&c.rec);
#pragma unroll
  for (int k = 0; k < static_cast<int>(sizeof(MapRecord) / 16); ++k) to[k] = from[k];
  c.rec_index = index;
  c.next_begin = index + 1 < args.nrec ? args.recs[index + 1].tile_begin : (int64_t{1} << 62);
  c.coef_batch = -1;
}

// Thread 0 only: decode the cursor's tile into `next`, staging its coefficients.
template <typename E, typename Off, int kThreadsPerCta>
__device__ __forceinline__ void DecodeAt(const MapArgs& args, MapCursor& c, TileState<Off>& next) {
  DecodeTile<Off, kThreadsPerCta>(args, c.rec, c.batch, c.local, next);
  if (c.coef_batch != c.batch) {
    E::Fetch(args, c.rec.coef_slot, c.batch, c.coef);
    c.coef_batch = c.batch;
  }
  const int4* from = reinterpret_cast<const int4*>(c.coef);
  int4* to = reinterpret_cast<int4*>(next.coef);
  to[0] = from[0];
  to[1] = from[1];
}

// Thread 0 only: advance the cursor to the next tile and decode it.
template <typename E, typename Off, int kThreadsPerCta>
__device__ __forceinline__ void DecodeNext(const MapArgs& args, MapCursor& c, TileState<Off>& next) {
  ++c.local;
  if (c.local == args.tiles_per_batch) {
    c.local = 0;
    ++c.batch;
    if (c.rec_index != 0) LoadRecord(args, 0, c);
  }
  while (c.local >= c.next_begin) LoadRecord(args, c.rec_index + 1, c);
  DecodeAt<E, Off, kThreadsPerCta>(args, c, next);
}

// One persistent CTA walks a contiguous range of tiles through kMapStages
// shared-memory stages: while tile i is written out of its stage, the loads
// of tiles i + 1 .. i + kMapStages - 1 are in flight (one cp.async group per
// tile), and thread 0 decodes tile i + kMapStages.  Tile states live in
// kMapStages + 1 slots: the tile being stored, the tiles in flight and the one
// being decoded.
#ifndef T0B_MAP_STAGES
#define T0B_MAP_STAGES 1
#endif
constexpr int kMapStages = T0B_MAP_STAGES;

template <int Op>
struct MapShape {
  static constexpr int kThreads = Op == kOpUpdate ? T0B_UPDATE_THREADS : T0B_PERMUTE_THREADS;
  static constexpr int kMinBlocks = Op == kOpUpdate ? T0B_UPDATE_MIN_BLOCKS : T0B_PERMUTE_MIN_BLOCKS;
};

__device__ __forceinline__ void CommitGroup() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }

// Wait until at most kMapStages - 1 of this thread's cp.async groups are pending.
__device__ __forceinline__ void WaitOldestGroup() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(kMapStages - 1) : "memory");
}

template <int Op, typename T, typename CA, typename CB, typename Off>
__global__ void __launch_bounds__(MapShape<Op>::kThreads, MapShape<Op>::kMinBlocks) MapKernel(MapArgs args) {
  using E = Emit<Op, T, CA, CB>;
  constexpr int kCta = MapShape<Op>::kThreads;
  constexpr int kSlots = kMapStages + 1;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ TileState<Off> states[kSlots];
  __shared__ MapCursor cursor;                 // the decoding thread's position
  const uint32_t smem_s = static_cast<uint32_t>(__cvta_generic_to_shared(smem_raw));
  // A stage holds the source tile and, for update, the base values after it.
  const uint32_t tile_bytes = static_cast<uint32_t>(args.tile_elems * sizeof(T));
  const uint32_t stage_bytes = E::kReadsBase ? 2 * tile_bytes : tile_bytes;
  const int64_t total = args.tiles_per_batch * args.batches;
  const int64_t per_cta = (total + gridDim.x - 1) / gridDim.x;
  const int64_t first = static_cast<int64_t>(blockIdx.x) * per_cta;
  const int64_t count = first < total ? min(total, first + per_cta) - first : 0;
  if (count == 0) return;
  if (threadIdx.x == 0) {
    const int64_t batch = first / args.tiles_per_batch;
    const int64_t local = first - batch * args.tiles_per_batch;
    int64_t lo = 0, hi = args.nrec - 1;
    while (lo < hi) {
      const int64_t mid = (lo + hi + 1) >> 1;
      if (args.recs[mid].tile_begin <= local) lo = mid; else hi = mid - 1;
    }
    LoadRecord(args, lo, cursor);
    cursor.batch = batch;
    cursor.local = local;
    DecodeAt<E, Off, kCta>(args, cursor, states[0]);
    for (int64_t k = 1; k < kMapStages && k < count; ++k) DecodeNext<E, Off, kCta>(args, cursor, states[k]);
  }
  __syncthreads();
  // Prologue: the loads of tiles 0 .. kMapStages - 2.
  for (int64_t k = 0; k + 1 < kMapStages; ++k) {
    if (k < count) {
      const uint32_t stage = smem_s + static_cast<uint32_t>(k) * stage_bytes;
      LoadTile<E, T, Off, kCta>(args, states[k], stage, stage + tile_bytes);
    }
    CommitGroup();
  }
  for (int64_t i = 0; i < count; ++i) {
    // Loads of tile i + kMapStages - 1 into the stage tile i - 1 released.
    const int64_t ahead = i + kMapStages - 1;
    if (ahead < count) {
      const uint32_t stage = smem_s + static_cast<uint32_t>(ahead % kMapStages) * stage_bytes;
      LoadTile<E, T, Off, kCta>(args, states[ahead % kSlots], stage, stage + tile_bytes);
    }
    CommitGroup();
    // While the copies fly, the decoding thread prepares tile i + kMapStages
    // in the slot tile i - 1 released.
    if (threadIdx.x == 0 && i + kMapStages < count) {
      DecodeNext<E, Off, kCta>(args, cursor, states[(i + kMapStages) % kSlots]);
    }
    WaitOldestGroup();
    __syncthreads();
    // Store: destination runs out of the tile, with the rule specialised per kind.
    {
      const TileState<Off>& st = states[i % kSlots];
      const uint32_t tile_s = smem_s + static_cast<uint32_t>(i % kMapStages) * stage_bytes;
      const E emit(st.coef);
      const bool skip = emit.SkipSource();
      const bool conjugate = args.conjugate != 0;
      T* __restrict__ out = static_cast<T*>(args.out) + st.dof;
      const uint32_t base_offset = tile_bytes;
      auto store = [&](auto kind) {
        constexpr int K = decltype(kind)::value;
        auto element = [&](T* p, uint32_t s) {
          T v{}, old{};
          if constexpr (E::kReadsBase) {
            // Update reads both stages without a branch (measured faster); a
            // stage the tile did not load (zero alpha or beta) holds stale
            // values the element rule ignores.
            v = LoadShared<T>(s);
            old = LoadShared<T>(s + base_offset);
          } else {
            if (!skip) v = LoadShared<T>(s);
            if constexpr (Op == kOpAccumulation) {
              if constexpr (Elem<T>::kComplex) {
                if (conjugate) v.y = -v.y;
              }
            }
          }
          *p = emit.template Apply<K>(v, old);
        };
        if (st.rect) {
          RectDestinationRows<kCta>(st.box, out, tile_s, element);
        } else {
          Walk<Off, kCta, true>(st.store, out, tile_s, element);
        }
      };
      switch (emit.Kind()) {
        case 1: store(std::integral_constant<int, 1>{}); break;
        case 2: store(std::integral_constant<int, 2>{}); break;
        default: store(std::integral_constant<int, 0>{}); break;
      }
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Reduce engine.

__device__ __forceinline__ int64_t FindGroup(const ReduceGroup* groups, int64_t lo, int64_t hi,
                                             int64_t value, bool by_task) {
  hi -= 1;
  while (lo < hi) {
    const int64_t mid = (lo + hi + 1) >> 1;
    const int64_t key = by_task ? groups[mid].task_begin : groups[mid].owner_begin;
    if (key <= value) lo = mid; else hi = mid - 1;
  }
  return lo;
}

template <typename T>
__device__ __forceinline__ T WarpSum(T v) {
#pragma unroll
  for (int offset = 16; offset > 0; offset >>= 1) {
    if constexpr (Elem<T>::kComplex) {
      T other;
      other.x = __shfl_xor_sync(0xffffffffu, v.x, offset);
      other.y = __shfl_xor_sync(0xffffffffu, v.y, offset);
      v = Add(v, other);
    } else {
      v = Add(v, __shfl_xor_sync(0xffffffffu, v, offset));
    }
  }
  return v;
}

// Pass 1: one warp per (owner, chunk of records); lanes stride the fibers.
constexpr int kFiberLoads = 4;
template <typename T, typename CA>
__global__ void __launch_bounds__(kThreads) ReducePartials(ReduceArgs args) {
  using Real = typename Elem<T>::Real;
  using C = typename BoundOf<Real, CA>::type;
  const T* __restrict__ src = static_cast<const T*>(args.src);
  T* scratch = static_cast<T*>(args.scratch);
  const int lane = threadIdx.x & 31;
  const int64_t wave_tasks = args.task_end - args.task_begin;
  const int64_t total = wave_tasks * args.batches;
  for (int64_t w = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) >> 5; w < total;
       w += (static_cast<int64_t>(gridDim.x) * kThreads) >> 5) {
    const int64_t batch = w / wave_tasks;
    const int64_t task = args.task_begin + (w - batch * wave_tasks);
    const ReduceGroup& g = args.groups[FindGroup(args.groups, args.group_begin, args.group_end, task, true)];
    const uint32_t local = static_cast<uint32_t>(task - g.task_begin);
    const uint32_t chunk = Division(g.div_owners).Div(local);
    const uint32_t owner = local - chunk * static_cast<uint32_t>(g.owners);
    int idx[kMaxRank];
    uint32_t rem = owner;
    for (int a = 0; a < g.rank; ++a) {
      const uint32_t next = Division(g.div_n[a]).Div(rem);
      idx[a] = static_cast<int>(rem - next * static_cast<uint32_t>(g.n[a]));
      rem = next;
    }
    const int64_t first = g.rec_begin + static_cast<int64_t>(chunk) * g.chunk_records;
    const int64_t last = min(g.rec_end, first + g.chunk_records);
    // Lanes take (record, fiber element) pairs: lanes stride one record's
    // fiber (lanes_per_record 32), or each lane sums whole records.
    const int per = g.lanes_per_record;
    const int sub = lane % per;
    T acc{};
    for (int64_t r = first + lane / per; r < last; r += 32 / per) {
      const ReduceRecord& rec = args.records[r];
      C c{};
      bool one = true, zero = false;
      if (rec.coef_slot >= 0) {
        c = ReadCoefficient<Real>(static_cast<const CA*>(args.ca), rec.coef_slot, args.ca_count, batch);
      }
      int64_t at = rec.src_off + batch * args.src_size;
      for (int a = 0; a < rec.map_rank; ++a) at += idx[a] * rec.s[a];
      const int fr = rec.fiber_rank, mr = rec.map_rank;
      // kFiberLoads elements' loads are issued before their sums, which are
      // added in fiber order; the coefficient is read alongside the first
      // loads (a zero coefficient skips the record's terms, as the reference
      // does, without a round trip ahead of the loads).
      for (int f0 = sub; f0 < rec.fiber_count; f0 += per * kFiberLoads) {
        T value[kFiberLoads];
#pragma unroll
        for (int u = 0; u < kFiberLoads; ++u) {
          const int f = f0 + u * per;
          value[u] = T{};
          if (f < rec.fiber_count) {
            int64_t off = 0;
            uint32_t rest = static_cast<uint32_t>(f);
            for (int a = 0; a < fr; ++a) {
              const uint32_t next = Division(rec.div_n[mr + a]).Div(rest);
              off += static_cast<int64_t>(rest - next * static_cast<uint32_t>(rec.n[mr + a])) * rec.s[mr + a];
              rest = next;
            }
            value[u] = src[at + off];
          }
        }
        if (f0 == sub && rec.coef_slot >= 0) {
          zero = IsZero(c);
          one = IsOne(c);
        }
        if (zero) break;
#pragma unroll
        for (int u = 0; u < kFiberLoads; ++u) {
          if (f0 + u * per < rec.fiber_count) {
            T v = value[u];
            if constexpr (Elem<T>::kComplex) {
              if (args.conjugate) v.y = -v.y;
            }
            acc = Add(acc, one ? v : Scale(c, v));
          }
        }
      }
    }
    acc = WarpSum(acc);
    if (lane == 0) scratch[batch * args.scratch_stride + g.scratch_off + chunk * g.owners + owner] = acc;
  }
}

// Pass 2: one thread per owner; chunks combined in record order.
template <typename T>
__global__ void __launch_bounds__(kThreads) ReduceFinish(ReduceArgs args) {
  const T* scratch = static_cast<const T*>(args.scratch);
  T* out = static_cast<T*>(args.out);
  const int64_t wave_owners = args.owner_end - args.owner_begin;
  const int64_t total = wave_owners * args.batches;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int64_t batch = i / wave_owners;
    const int64_t owner_id = args.owner_begin + (i - batch * wave_owners);
    const ReduceGroup& g = args.groups[FindGroup(args.groups, args.group_begin, args.group_end, owner_id, false)];
    const int64_t owner = owner_id - g.owner_begin;
    const T* partial = scratch + batch * args.scratch_stride + g.scratch_off + owner;
    // Loads of four partials are issued before their (in-order) sums.
    T sum = partial[0];
    int k = 1;
    for (; k + 3 < g.chunks; k += 4) {
      const T a = partial[static_cast<int64_t>(k) * g.owners];
      const T b = partial[static_cast<int64_t>(k + 1) * g.owners];
      const T c = partial[static_cast<int64_t>(k + 2) * g.owners];
      const T d = partial[static_cast<int64_t>(k + 3) * g.owners];
      sum = Add(Add(Add(Add(sum, a), b), c), d);
    }
    for (; k < g.chunks; ++k) sum = Add(sum, partial[static_cast<int64_t>(k) * g.owners]);
    int64_t at = g.dst_off + batch * args.out_size;
    uint32_t rem = static_cast<uint32_t>(owner);
    for (int a = 0; a < g.rank; ++a) {
      const uint32_t next = Division(g.div_n[a]).Div(rem);
      at += static_cast<int64_t>(rem - next * static_cast<uint32_t>(g.n[a])) * g.d[a];
      rem = next;
    }
    out[at] = args.assign ? PlusZero(sum) : Add(out[at], sum);
  }
}

// ---------------------------------------------------------------------------
// Dot engine: out[b] = sum of conj?(left[src]) * right[dst] over every element
// of every record.  Pass 1: CTA (x, b) walks a contiguous range of units of
// batch b, one unit (a chunk of one row) per warp at a time with lanes
// striding the chunk, and writes its sum to partials[b][x]; pass 2 sums the
// partials of each batch in index order.  Deterministic for a given grid.
// Products are rounded in the storage precision (as the reference's
// arithmetic::Product); single-precision sums accumulate in double precision
// and round once at the end, so long sums stay within the stated tolerance.
// The partials live in the caller's scratch (kDotPartials storage elements
// per batch), as DotSum values.

template <typename T> struct DotSumOf { using type = T; };
template <> struct DotSumOf<float> { using type = double; };
template <> struct DotSumOf<float2> { using type = double2; };

__device__ __forceinline__ double Widen(float v) { return v; }
__device__ __forceinline__ double2 Widen(float2 v) { return {v.x, v.y}; }
__device__ __forceinline__ double Widen(double v) { return v; }
__device__ __forceinline__ double2 Widen(double2 v) { return v; }
__device__ __forceinline__ float Narrow(double v, float*) { return __double2float_rn(v); }
__device__ __forceinline__ float2 Narrow(double2 v, float2*) { return {__double2float_rn(v.x), __double2float_rn(v.y)}; }
__device__ __forceinline__ double Narrow(double v, double*) { return v; }
__device__ __forceinline__ double2 Narrow(double2 v, double2*) { return v; }

template <typename T>
__device__ __forceinline__ T DotProduct(T a, T b, bool conjugate) {
  if constexpr (Elem<T>::kComplex) {
    if (conjugate) a.y = -a.y;
    return Scale(a, b);
  } else {
    return Mul(a, b);
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) DotPartials(DotArgs a) {
  using S = typename DotSumOf<T>::type;
  const int64_t batch = blockIdx.y;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * kWarps;
  const int64_t w = static_cast<int64_t>(blockIdx.x) * kWarps + warp;
  const int64_t per = (a.units + warps - 1) / warps;
  const int64_t first = w * per, last = min(a.units, first + per);
  const T* __restrict__ left = static_cast<const T*>(a.left) + batch * a.left_size;
  const T* __restrict__ right = static_cast<const T*>(a.right) + batch * a.right_size;
  const bool conjugate = a.conjugate_left != 0;
  S acc{};
  int64_t rec = 0;
  if (first < last) {
    int64_t lo = 0, hi = a.nrec - 1;
    while (lo < hi) {
      const int64_t mid = (lo + hi + 1) >> 1;
      if (a.recs[mid].unit_begin <= first) lo = mid; else hi = mid - 1;
    }
    rec = lo;
  }
  for (int64_t u = first; u < last; ++u) {
    while (rec + 1 < a.nrec && a.recs[rec + 1].unit_begin <= u) ++rec;
    const DotRecord& r = a.recs[rec];
    uint32_t q = static_cast<uint32_t>(u - r.unit_begin);
    const uint32_t row = Division(r.div[0]).Div(q);
    const int chunk = static_cast<int>(q - row * static_cast<uint32_t>(r.chunks));
    q = row;
    int64_t lo_off = r.left_off, ro_off = r.right_off;
    for (int ax = 1; ax < r.rank; ++ax) {
      const uint32_t next = Division(r.div[ax]).Div(q);
      const int64_t idx = q - next * static_cast<uint32_t>(r.n[ax]);
      q = next;
      lo_off += idx * r.sl[ax];
      ro_off += idx * r.sr[ax];
    }
    const int begin = chunk * r.chunk;
    const int end = min(r.n[0], begin + r.chunk);
    const int64_t sl = r.sl[0], sr = r.sr[0];
    for (int j = begin + lane; j < end; j += 32) {
      acc = Add(acc, Widen(DotProduct(left[lo_off + j * sl], right[ro_off + j * sr], conjugate)));
    }
  }
  acc = WarpSum(acc);
  __shared__ S sums[kWarps];
  if (lane == 0) sums[warp] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    S total = sums[0];
    for (int k = 1; k < kWarps; ++k) total = Add(total, sums[k]);
    S* partials = reinterpret_cast<S*>(static_cast<T*>(a.partials) + batch * kDotPartials);
    partials[blockIdx.x] = total;
  }
}

template <typename T>
__global__ void __launch_bounds__(32) DotFinish(DotArgs a, int parts) {
  using S = typename DotSumOf<T>::type;
  const int64_t batch = blockIdx.x;
  const S* partials = reinterpret_cast<const S*>(static_cast<const T*>(a.partials) + batch * kDotPartials);
  S acc{};
  for (int k = threadIdx.x; k < parts; k += 32) acc = Add(acc, partials[k]);
  acc = WarpSum(acc);
  if (threadIdx.x == 0) static_cast<T*>(a.out)[batch] = Narrow(acc, static_cast<T*>(nullptr));
}

// ---------------------------------------------------------------------------
// TensorMap.add.

template <typename T, typename S>
__global__ void __launch_bounds__(kThreads) AxpbyKernel(int64_t n, S alpha, const T* __restrict__ x,
                                                      S beta, const T* __restrict__ y, T* out) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    out[i] = Add(Scale(alpha, x[i]), Scale(beta, y[i]));
  }
}

template <int Op, typename T, typename CA, typename CB, typename Off>
void LaunchMapKernel(const MapArgs& args, int smem, cudaStream_t stream) {
  auto kernel = MapKernel<Op, T, CA, CB, Off>;
  // Allow as much dynamic shared memory as the device gives one block beyond
  // the kernel's static shared memory.
  static const bool configured = [&] {
    int device = 0, limit = 48 * 1024;
    cudaFuncAttributes attributes{};
    Check(cudaGetDevice(&device), "map device");
    Check(cudaDeviceGetAttribute(&limit, cudaDevAttrMaxSharedMemoryPerBlockOptin, device), "map shared limit");
    Check(cudaFuncGetAttributes(&attributes, kernel), "map attributes");
    Check(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               limit - static_cast<int>(attributes.sharedSizeBytes)), "map attribute");
    return true;
  }();
  (void)configured;
  int blocks = 0;
  Check(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kernel, MapShape<Op>::kThreads, smem), "map occupancy");
  const int per_sm = std::max(blocks, 1);
  const int64_t total = args.tiles_per_batch * args.batches;
  const int64_t grid = std::min<int64_t>(total, static_cast<int64_t>(per_sm) * SmCount());
  kernel<<<static_cast<unsigned>(grid), MapShape<Op>::kThreads, smem, stream>>>(args);
  Check(cudaGetLastError(), "map launch");
  g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
}

template <int Op, typename T, typename CA, typename CB>
void LaunchMapTyped(const MapArgs& args, int smem, bool wide, cudaStream_t stream) {
  if (wide) LaunchMapKernel<Op, T, CA, CB, int64_t>(args, smem, stream);
  else LaunchMapKernel<Op, T, CA, CB, int32_t>(args, smem, stream);
}

template <typename Real, typename Complex, typename F>
void VisitCoefficient(int32_t dtype, bool complex_storage, F&& f) {
  if (dtype == 4) { f(static_cast<const int32_t*>(nullptr)); return; }
  if ((dtype == 11 && sizeof(Real) == 4) || (dtype == 12 && sizeof(Real) == 8)) {
    f(static_cast<const Real*>(nullptr)); return;
  }
  if (complex_storage && ((dtype == 15 && sizeof(Real) == 4) || (dtype == 18 && sizeof(Real) == 8))) {
    f(static_cast<const Complex*>(nullptr)); return;
  }
  throw InvalidArgumentError("unsupported CUDA coefficient dtype; expected S32 or matching real/complex precision");
}

template <typename F>
void WithStorage(int32_t dtype, F&& f) {
  switch (dtype) {
    case 11: f(static_cast<float*>(nullptr)); return;
    case 12: f(static_cast<double*>(nullptr)); return;
    case 15: f(static_cast<float2*>(nullptr)); return;
    case 18: f(static_cast<double2*>(nullptr)); return;
    default: throw InvalidArgumentError("CUDA stride storage supports only F32/F64/C64/C128");
  }
}

}  // namespace

int SmCount() {
  static int count = [] {
    int device = 0, sms = 148;
    if (cudaGetDevice(&device) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    return sms;
  }();
  return count;
}

void Check(cudaError_t status, const char* what) {
  if (status != cudaSuccess) {
    // Clear the runtime's last-error slot so the next launch check does not
    // report this (non-sticky) failure again.
    (void)cudaGetLastError();
    throw std::runtime_error(std::string("CUDA ") + what + ": " + cudaGetErrorString(status));
  }
}

int64_t MapSharedBytes(int op, int64_t tile_elems, int element_bytes) {
  const int64_t tile = tile_elems * element_bytes;
  return (op == kOpUpdate ? 2 * tile : tile) * kMapStages;
}

void MapTileElements(const MapRecord* recs, int64_t count, int element_bytes, int64_t* tile, int64_t* box) {
  *tile = 0;
  *box = 0;
  for (int64_t i = 0; i < count; ++i) {
    const int64_t t0 = recs[i].t[0], t1 = recs[i].t[1], t2 = recs[i].t[2];
    *tile = std::max<int64_t>(*tile, (t0 | 1) * t1 * t2);
    *box = std::max<int64_t>(*box, t0 * t1 * t2);
  }
}

void LaunchMap(int op, int32_t dtype, int32_t ca_dtype, int32_t cb_dtype, const MapArgs& args,
               int smem, bool wide, cudaStream_t stream) {
  WithStorage(dtype, [&](auto* tag) {
    using T = std::remove_pointer_t<decltype(tag)>;
    using Real = typename Elem<T>::Real;
    using Complex = std::conditional_t<sizeof(Real) == 4, float2, double2>;
    constexpr bool kComplex = Elem<T>::kComplex;
    if (op == kOpCopy) {
      using Bits = std::conditional_t<sizeof(T) == 4, uint32_t, std::conditional_t<sizeof(T) == 8, uint2, uint4>>;
      LaunchMapTyped<kOpCopy, Bits, int32_t, int32_t>(args, smem, wide, stream);
    } else if (op == kOpAccumulation) {
      VisitCoefficient<Real, Complex>(ca_dtype, kComplex, [&](auto* ca) {
        using CA = std::remove_cv_t<std::remove_pointer_t<decltype(ca)>>;
        if constexpr (!kComplex && sizeof(CA) == 2 * sizeof(Real)) {
        } else {
          LaunchMapTyped<kOpAccumulation, T, CA, int32_t>(args, smem, wide, stream);
        }
      });
    } else {
      VisitCoefficient<Real, Complex>(ca_dtype, kComplex, [&](auto* ca) {
        using CA = std::remove_cv_t<std::remove_pointer_t<decltype(ca)>>;
        VisitCoefficient<Real, Complex>(cb_dtype, kComplex, [&](auto* cb) {
          using CB = std::remove_cv_t<std::remove_pointer_t<decltype(cb)>>;
          if constexpr (!kComplex && (sizeof(CA) == 2 * sizeof(Real) || sizeof(CB) == 2 * sizeof(Real))) {
          } else {
            LaunchMapTyped<kOpUpdate, T, CA, CB>(args, smem, wide, stream);
          }
        });
      });
    }
  });
}

void LaunchReduce(int32_t dtype, int32_t ca_dtype, const ReduceArgs& args, cudaStream_t stream) {
  WithStorage(dtype, [&](auto* tag) {
    using T = std::remove_pointer_t<decltype(tag)>;
    using Real = typename Elem<T>::Real;
    using Complex = std::conditional_t<sizeof(Real) == 4, float2, double2>;
    constexpr bool kComplex = Elem<T>::kComplex;
    VisitCoefficient<Real, Complex>(ca_dtype, kComplex, [&](auto* ca) {
      using CA = std::remove_cv_t<std::remove_pointer_t<decltype(ca)>>;
      if constexpr (!kComplex && sizeof(CA) == 2 * sizeof(Real)) {
      } else {
        const int64_t warps = (args.task_end - args.task_begin) * args.batches;
        if (warps > 0) {
          const int64_t grid = std::min<int64_t>((warps + kWarps - 1) / kWarps, int64_t{SmCount()} * 16);
          ReducePartials<T, CA><<<static_cast<unsigned>(grid), kThreads, 0, stream>>>(args);
          Check(cudaGetLastError(), "reduce launch");
          g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
        }
        const int64_t threads = (args.owner_end - args.owner_begin) * args.batches;
        if (threads > 0) {
          const int64_t grid = std::min<int64_t>((threads + kThreads - 1) / kThreads, int64_t{SmCount()} * 16);
          ReduceFinish<T><<<static_cast<unsigned>(grid), kThreads, 0, stream>>>(args);
          Check(cudaGetLastError(), "reduce finish launch");
          g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
        }
      }
    });
  });
}

void LaunchDot(int32_t dtype, const DotArgs& args, cudaStream_t stream) {
  if (args.batches == 0) return;
  if (args.batches > 65535) throw InvalidArgumentError("dot supports at most 65535 batches per call");
  const int64_t warps_wanted = std::max<int64_t>(1, args.units / 4);
  WithStorage(dtype, [&](auto* tag) {
    using T = std::remove_pointer_t<decltype(tag)>;
    // Partials are double precision for single-precision storage: half as many fit.
    const int64_t fit = sizeof(typename DotSumOf<T>::type) > sizeof(T) ? kDotPartials / 2 : kDotPartials;
    const int parts = static_cast<int>(std::min<int64_t>(
        fit, std::min<int64_t>((warps_wanted + kWarps - 1) / kWarps,
                               std::max<int64_t>(1, int64_t{SmCount()} * 8 / args.batches))));
    DotPartials<T><<<dim3(static_cast<unsigned>(parts), static_cast<unsigned>(args.batches)), kThreads, 0, stream>>>(args);
    Check(cudaGetLastError(), "dot launch");
    g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
    DotFinish<T><<<static_cast<unsigned>(args.batches), 32, 0, stream>>>(args, parts);
    Check(cudaGetLastError(), "dot finish launch");
    g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
  });
}

void LaunchAxpby(int32_t dtype, int64_t n, double ar, double ai, const void* x, double br, double bi,
                 const void* y, void* out, cudaStream_t stream) {
  if (n == 0) return;
  const int64_t grid = std::min<int64_t>((n + kThreads - 1) / kThreads, int64_t{SmCount()} * 8);
  switch (dtype) {
    case 11:
      AxpbyKernel<float, float><<<static_cast<unsigned>(grid), kThreads, 0, stream>>>(
          n, static_cast<float>(ar), static_cast<const float*>(x), static_cast<float>(br),
          static_cast<const float*>(y), static_cast<float*>(out));
      break;
    case 12:
      AxpbyKernel<double, double><<<static_cast<unsigned>(grid), kThreads, 0, stream>>>(
          n, ar, static_cast<const double*>(x), br, static_cast<const double*>(y), static_cast<double*>(out));
      break;
    case 15:
      AxpbyKernel<float2, float2><<<static_cast<unsigned>(grid), kThreads, 0, stream>>>(
          n, float2{static_cast<float>(ar), static_cast<float>(ai)}, static_cast<const float2*>(x),
          float2{static_cast<float>(br), static_cast<float>(bi)}, static_cast<const float2*>(y),
          static_cast<float2*>(out));
      break;
    case 18:
      AxpbyKernel<double2, double2><<<static_cast<unsigned>(grid), kThreads, 0, stream>>>(
          n, double2{ar, ai}, static_cast<const double2*>(x), double2{br, bi},
          static_cast<const double2*>(y), static_cast<double2*>(out));
      break;
    default:
      throw InvalidArgumentError("axpby supports only F32/F64/C64/C128");
  }
  Check(cudaGetLastError(), "axpby launch");
  g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
}

}  // namespace t0b
