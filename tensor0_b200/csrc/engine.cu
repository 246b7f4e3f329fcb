// Map and reduce engines: the grouped strided permute / accumulate / update
// kernel and the two-pass segmented reduction for partial traces.
//
// The map kernel is one persistent grid over every tile of every record of
// every batch; each CTA walks a contiguous range of tiles.  A tile is a box
// over the record's destination-innermost axis X, its source-innermost axis Y
// and one further axis Z.  One thread decodes the tile with host-computed
// division constants.  The CTA copies the tile's source runs into shared
// memory in source order, as the 16-byte units that cover each run (one
// cp.async per four f32 elements), then writes the destination rows along X,
// each lane group reading its column of the staged rows.  Reads and writes
// are coalesced and no element costs more than its shared-memory read, its
// store and an addition or two.
#include "engine.h"

#include "arith.cuh"

#include <algorithm>
#include <atomic>

namespace t0b {

std::atomic<uint64_t> g_kernel_launches{0};

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
#ifndef T0B_MAP_MIN_BLOCKS
#define T0B_MAP_MIN_BLOCKS 4   // map CTAs per SM the register budget is sized for
#endif

// Division by a constant computed on the host (MakeDivision).
struct FastDiv {
  uint32_t m, l;
  __device__ __forceinline__ uint32_t Div(uint32_t n) const { return (__umulhi(n, m) + n) >> l; }
};

__device__ __forceinline__ FastDiv Division(const DivisionConstants& c) { return FastDiv{c.magic, c.shift}; }

// "Division" by 2^31: every row index of a single-plane row list is in plane 0.
constexpr FastDiv kSinglePlane{0, 31};

// A decoded tile, shared by the CTA.  In-tile offsets use Off (int32 unless
// the plan marked a record wide).
//
// Shared memory holds the tile in source order: one row per source run (a
// transpose tile's (x, z) runs along Y, or its x runs along (Y, Z) when Z
// continues Y; a direct tile's (y, z) runs along X), `py` elements apart.  A
// unit-stride run is copied as the 16-byte units that cover it, so its first
// element sits delta elements into its row, delta being the run's global
// offset modulo 16 bytes.  The update's base values are staged the same way
// in destination order: one row per destination (y, z) row, `qx` apart.
template <typename Off>
struct TileState {
  int64_t so, dof;        // element offsets of the tile origin, batch included
  Off sx, sy, sz, dx, dy, dz;
  int ex, ey, ez;         // tile extents (edge tiles are smaller)
  int mode;               // kTranspose or kDirect
  int linear;             // transpose: Z continues Y in the source (one run per x)
  int py, qx;             // row pitches of the source and base stages
  FastDiv by_x, by_y;     // by ex, by ey
  int64_t batch;
  int slot;
  alignas(16) unsigned char coef[32];   // the tile's coefficients, fetched by the decoding thread
};

// Thread 0 only: decode tile `local` of record `rec` in `batch`.
template <typename T, typename Off>
__device__ __forceinline__ void DecodeTile(const MapArgs& a, int64_t rec, int64_t batch, int64_t local,
                                           TileState<Off>& s) {
  constexpr int kVec = 16 / sizeof(T);
  const MapRecord& r = a.recs[rec];
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
  s.sx = static_cast<Off>(r.s[0]); s.sy = static_cast<Off>(r.s[1]); s.sz = static_cast<Off>(r.s[2]);
  s.dx = static_cast<Off>(r.d[0]); s.dy = static_cast<Off>(r.d[1]); s.dz = static_cast<Off>(r.d[2]);
  s.ex = ex; s.ey = ey; s.ez = ez;
  s.mode = r.mode;
  s.linear = r.mode == kTranspose && ez > 1 && r.s[2] == static_cast<int64_t>(ey) * r.s[1];
  const int run = r.mode == kDirect ? ex : (s.linear ? ey * ez : ey);
  s.py = static_cast<int>(RowPitch(run, kVec));
  s.qx = static_cast<int>(RowPitch(ex, kVec));
  s.by_x = Division(r.div_extent[last_x ? 1 : 0]);
  s.by_y = Division(r.div_extent[last_y ? 3 : 2]);
  s.batch = batch;
  s.slot = r.coef_slot;
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

// Asynchronous global -> shared copy of Bytes (no register round trip).  The
// copies are ordered against shared-memory reads by WaitAsync and the CTA
// barrier that follows it.
template <int Bytes>
__device__ __forceinline__ void CopyAsync(uint32_t smem, const void* gmem) {
  if constexpr (Bytes == 16) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem), "l"(gmem));
  } else {
    asm volatile("cp.async.ca.shared.global [%0], [%1], %2;\n" ::"r"(smem), "l"(gmem), "n"(Bytes));
  }
}

__device__ __forceinline__ void WaitAsync() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }

// Rows r = 0 .. rows - 1 handed out kLanes lanes at a time: each warp step
// covers 32 / kLanes rows; f(r, sub) runs in the row's lane group, sub being
// the lane's index in it.
template <int kLanes, typename F>
__device__ __forceinline__ void ForRowGroups(int rows, F&& f) {
  constexpr int kGroups = 32 / kLanes;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = lane % kLanes, group = lane / kLanes;
  for (int r0 = warp * kGroups; r0 < rows; r0 += kWarps * kGroups) {
    if (r0 + group < rows) f(r0 + group, sub);
  }
}

// Element offset of a pointer modulo the 16-byte unit.
template <typename T>
__device__ __forceinline__ int UnitOffset(const T* p) {
  return static_cast<int>((reinterpret_cast<uintptr_t>(p) / sizeof(T)) & (16 / sizeof(T) - 1));
}

// Stage `rows` runs of `len` elements into shared-memory rows `pitch` apart:
// run r = a + na * b starts at from + a * ga + b * gb and steps gj.  A
// unit-step run is copied as the 16-byte units covering it (its first element
// lands UnitOffset(run) into the row; the units reach at most 15 bytes beyond
// the run on either side, never past the 16-byte units holding its ends);
// other runs element by element, from the row start.  Few long runs are
// spread over the whole CTA, the rest over 4- to 32-lane groups.
template <typename T, typename Off>
__device__ __forceinline__ void StageRows(const T* from, int rows, int na, FastDiv by_na, Off ga, Off gb, Off gj,
                                          int len, int pitch, uint32_t smem) {
  constexpr int kVec = 16 / sizeof(T);
  auto run_of = [&](int r) {
    const int b = static_cast<int>(by_na.Div(static_cast<uint32_t>(r)));
    const int a = r - b * na;
    return from + (a * ga + b * gb);
  };
  if (gj == 1) {
    const int most = (len + 2 * kVec - 2) / kVec;   // 16-byte units a run may span
    auto units = [&](auto lanes) {
      constexpr int kLanes = decltype(lanes)::value;
      ForRowGroups<kLanes>(rows, [&](int r, int sub) {
        const T* run = run_of(r);
        const int delta = UnitOffset(run);
        const T* aligned = run - delta;
        const int n = (delta + len + kVec - 1) / kVec;
        const uint32_t row = smem + static_cast<uint32_t>(r * pitch) * static_cast<uint32_t>(sizeof(T));
        for (int u = sub; u < n; u += kLanes) CopyAsync<16>(row + 16 * u, aligned + kVec * u);
      });
    };
    if (rows < kWarps && most >= kThreads) {
      for (int r = 0; r < rows; ++r) {
        const T* run = run_of(r);
        const int delta = UnitOffset(run);
        const T* aligned = run - delta;
        const int n = (delta + len + kVec - 1) / kVec;
        const uint32_t row = smem + static_cast<uint32_t>(r * pitch) * static_cast<uint32_t>(sizeof(T));
        for (int u = threadIdx.x; u < n; u += kThreads) CopyAsync<16>(row + 16 * u, aligned + kVec * u);
      }
    } else if (most <= 4) {
      units(std::integral_constant<int, 4>{});
    } else if (most <= 8) {
      units(std::integral_constant<int, 8>{});
    } else if (most <= 16) {
      units(std::integral_constant<int, 16>{});
    } else {
      units(std::integral_constant<int, 32>{});
    }
  } else {
    auto elements = [&](auto lanes) {
      constexpr int kLanes = decltype(lanes)::value;
      ForRowGroups<kLanes>(rows, [&](int r, int sub) {
        const T* run = run_of(r);
        const uint32_t row = smem + static_cast<uint32_t>(r * pitch) * static_cast<uint32_t>(sizeof(T));
        for (int j = sub; j < len; j += kLanes) {
          CopyAsync<sizeof(T)>(row + static_cast<uint32_t>(j) * static_cast<uint32_t>(sizeof(T)), run + j * gj);
        }
      });
    };
    if (len <= 8) elements(std::integral_constant<int, 8>{});
    else if (len <= 64) elements(std::integral_constant<int, 16>{});
    else elements(std::integral_constant<int, 32>{});
  }
}

// Issue the asynchronous loads of one tile: the source runs into the source
// stage and, for update, the destination rows' base values into the base
// stage.
template <typename E, typename T, typename Off>
__device__ __forceinline__ void LoadTile(const MapArgs& args, const TileState<Off>& st, uint32_t tile_s,
                                         uint32_t base_s) {
  const E emit(st.coef);
  const int ex = st.ex, ey = st.ey, ez = st.ez;
  if (!emit.SkipSource()) {
    const T* src = static_cast<const T*>(args.src) + st.so;
    if (st.mode == kDirect) {
      StageRows<T, Off>(src, ey * ez, ey, st.by_y, st.sy, st.sz, st.sx, ex, st.py, tile_s);
    } else if (st.linear) {
      StageRows<T, Off>(src, ex, ex, kSinglePlane, st.sx, Off{0}, st.sy, ey * ez, st.py, tile_s);
    } else {
      StageRows<T, Off>(src, ex * ez, ex, st.by_x, st.sx, st.sz, st.sy, ey, st.py, tile_s);
    }
  }
  if constexpr (E::kReadsBase) {
    if (emit.NeedsBase()) {
      const T* base = static_cast<const T*>(args.base) + st.dof;
      StageRows<T, Off>(base, ey * ez, ey, st.by_y, st.dy, st.dz, st.dx, ex, st.qx, base_s);
    }
  }
}

// Write one tile: destination rows (y, z) along X, lane groups sized to ex
// (or the whole CTA for few long rows).  Element (x, y, z) is read from its
// source row -- row x (+ ex * z), column y (+ ey * z) for a transpose tile;
// row y + ey * z, column x for a direct one -- plus that run's delta.  A
// lane's columns step by its group size, a multiple of the 16-byte unit, so
// its delta is fixed along the row.  A lane handles its columns in blocks of
// eight slots without branches: a slot past the row end reads the lane's
// first column again and skips only its store.  Values of a stage the tile
// did not load (zero alpha or beta) are read but ignored by the element rule.
template <int K, bool kUnitDx, typename E, typename T, typename Off>
__device__ __forceinline__ void StoreTile(const MapArgs& args, const TileState<Off>& st, const E& emit,
                                          const T* tile, const T* base_tile) {
  constexpr int kVec = 16 / sizeof(T);
  constexpr uint32_t kMask = kVec - 1;
  const int ex = st.ex, ey = st.ey, rows = ey * st.ez;
  const bool direct = st.mode == kDirect, linear = st.linear;
  const int py = st.py, qx = st.qx;
  const Off dx = kUnitDx ? Off{1} : st.dx, dy = st.dy, dz = st.dz;
  const FastDiv by_y = st.by_y;
  // Deltas of the source runs (zero for runs staged element by element).
  const bool src_units = (direct ? st.sx : st.sy) == 1;
  const uint32_t s0 = static_cast<uint32_t>(UnitOffset(static_cast<const T*>(args.src) + st.so));
  const uint32_t sx = static_cast<uint32_t>(st.sx), sy = static_cast<uint32_t>(st.sy), sz = static_cast<uint32_t>(st.sz);
  const uint32_t b0 = E::kReadsBase ? static_cast<uint32_t>(UnitOffset(static_cast<const T*>(args.base) + st.dof)) : 0u;
  const uint32_t udy = static_cast<uint32_t>(dy), udz = static_cast<uint32_t>(dz);
  T* __restrict__ out = static_cast<T*>(args.out) + st.dof;
  // Row r = y + ey * z as seen by the lane whose first column is x0 < ex.
  auto row = [&](int r, int x0, auto lanes) {
    constexpr int kLanes = decltype(lanes)::value;
    const int z = static_cast<int>(by_y.Div(static_cast<uint32_t>(r)));
    const int y = r - z * ey;
    int t, t_step;
    if (direct) {
      const int delta = src_units ? static_cast<int>((s0 + y * sy + z * sz) & kMask) : 0;
      t = r * py + delta + x0;
      t_step = 1;
    } else if (linear) {
      const int delta = src_units ? static_cast<int>((s0 + x0 * sx) & kMask) : 0;
      t = x0 * py + delta + r;
      t_step = py;
    } else {
      const int delta = src_units ? static_cast<int>((s0 + x0 * sx + z * sz) & kMask) : 0;
      t = (x0 + ex * z) * py + delta + y;
      t_step = py;
    }
    const T* tp = tile + t;
    const T* bp = base_tile;
    if constexpr (E::kReadsBase) {
      bp += r * qx + (kUnitDx ? static_cast<int>((b0 + y * udy + z * udz) & kMask) : 0) + x0;
    }
    T* p = out + (y * dy + z * dz + x0 * dx);
    for (int k0 = 0; x0 + k0 < ex; k0 += 8 * kLanes) {
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        const int k = k0 + m * kLanes;
        const bool ok = x0 + k < ex;
        const int kk = ok ? k : 0;
        const T v = tp[kk * t_step];
        T old{};
        if constexpr (E::kReadsBase) old = bp[kk];
        const T w = emit.template Apply<K>(v, old);
        if (ok) p[kUnitDx ? k : k * dx] = w;
      }
    }
  };
  auto groups = [&](auto lanes) {
    ForRowGroups<decltype(lanes)::value>(rows, [&](int r, int sub) {
      if (sub < ex) row(r, sub, lanes);
    });
  };
  if (rows < kWarps && ex >= kThreads) {
    for (int r = 0; r < rows; ++r) row(r, threadIdx.x, std::integral_constant<int, kThreads>{});
  } else if (ex <= 64) {
    groups(std::integral_constant<int, 8>{});
  } else if (ex <= 128) {
    groups(std::integral_constant<int, 16>{});
  } else {
    groups(std::integral_constant<int, 32>{});
  }
}

// Thread 0 only: advance the tile cursor (record, batch, tile within the
// batch) to the next tile and decode it.
template <typename E, typename T, typename Off>
__device__ __forceinline__ void DecodeNext(const MapArgs& args, int64_t* cursor, TileState<Off>& next) {
  int64_t rec = cursor[0], batch = cursor[1], local = cursor[2] + 1;
  if (local == args.tiles_per_batch) { local = 0; ++batch; rec = 0; }
  while (rec + 1 < args.nrec && args.recs[rec + 1].tile_begin <= local) ++rec;
  cursor[0] = rec; cursor[1] = batch; cursor[2] = local;
  DecodeTile<T, Off>(args, rec, batch, local, next);
  E::Fetch(args, next.slot, next.batch, next.coef);
}

// One persistent CTA walks a contiguous range of tiles.  Per tile: issue the
// asynchronous loads, let thread 0 decode the next tile while they fly, wait,
// then write the destination rows out of shared memory.
template <int Op, typename T, typename CA, typename CB, typename Off>
__global__ void __launch_bounds__(kThreads, T0B_MAP_MIN_BLOCKS) MapKernel(MapArgs args) {
  using E = Emit<Op, T, CA, CB>;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ TileState<Off> states[2];        // the current tile and the next one
  __shared__ int64_t cursor[3];               // decoding thread: record, batch, tile within the batch
  const T* tile = reinterpret_cast<const T*>(smem_raw);
  const T* base_tile = tile + args.tile_elems;   // update: destination base values
  const uint32_t tile_s = static_cast<uint32_t>(__cvta_generic_to_shared(smem_raw));
  const uint32_t base_s = tile_s + static_cast<uint32_t>(args.tile_elems * sizeof(T));
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
    cursor[0] = lo; cursor[1] = batch; cursor[2] = local;
    DecodeTile<T, Off>(args, lo, batch, local, states[0]);
    E::Fetch(args, states[0].slot, states[0].batch, states[0].coef);
  }
  __syncthreads();
  for (int64_t i = 0; i < count; ++i) {
    const TileState<Off>& st = states[i & 1];
    LoadTile<E, T, Off>(args, st, tile_s, base_s);
    // While the copies fly, the decoding thread prepares the next tile.
    if (threadIdx.x == 0 && i + 1 < count) DecodeNext<E, T, Off>(args, cursor, states[(i + 1) & 1]);
    WaitAsync();
    __syncthreads();
    {
      const E emit(st.coef);
      auto store = [&](auto unit_dx) {
        constexpr bool kUnitDx = decltype(unit_dx)::value;
        switch (emit.Kind()) {
          case 1: StoreTile<1, kUnitDx, E, T, Off>(args, st, emit, tile, base_tile); break;
          case 2: StoreTile<2, kUnitDx, E, T, Off>(args, st, emit, tile, base_tile); break;
          default: StoreTile<0, kUnitDx, E, T, Off>(args, st, emit, tile, base_tile); break;
        }
      };
      if (st.dx == 1) store(std::true_type{});
      else store(std::false_type{});
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
    const int64_t local = task - g.task_begin;
    const int64_t chunk = local / g.owners;
    const int64_t owner = local - chunk * g.owners;
    int idx[kMaxRank];
    int64_t rem = owner;
    for (int a = 0; a < g.rank; ++a) { idx[a] = static_cast<int>(rem % g.n[a]); rem /= g.n[a]; }
    const int64_t first = g.rec_begin + chunk * g.chunk_records;
    const int64_t last = min(g.rec_end, first + g.chunk_records);
    T acc{};
    for (int64_t r = first; r < last; ++r) {
      const ReduceRecord& rec = args.records[r];
      C c{};
      bool one = true;
      if (rec.coef_slot >= 0) {
        c = ReadCoefficient<Real>(static_cast<const CA*>(args.ca), rec.coef_slot, args.ca_count, batch);
        if (IsZero(c)) continue;
        one = IsOne(c);
      }
      int64_t at = rec.src_off + batch * args.src_size;
      for (int a = 0; a < rec.map_rank; ++a) at += idx[a] * rec.s[a];
      const int fr = rec.fiber_rank, mr = rec.map_rank;
      for (int f = lane; f < rec.fiber_count; f += 32) {
        int64_t off = 0;
        int rest = f;
        for (int a = 0; a < fr; ++a) {
          const int n = rec.n[mr + a];
          const int i = rest % n;
          rest /= n;
          off += i * rec.s[mr + a];
        }
        const T value = src[at + off];
        acc = Add(acc, one ? value : Scale(c, value));
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
    T sum = partial[0];
    for (int k = 1; k < g.chunks; ++k) sum = Add(sum, partial[static_cast<int64_t>(k) * g.owners]);
    int64_t at = g.dst_off + batch * args.out_size;
    int64_t rem = owner;
    for (int a = 0; a < g.rank; ++a) { at += (rem % g.n[a]) * g.d[a]; rem /= g.n[a]; }
    out[at] = Add(out[at], sum);
  }
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

int SmCount() {
  static int count = [] {
    int device = 0, sms = 148;
    if (cudaGetDevice(&device) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    return sms;
  }();
  return count;
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
  Check(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kernel, kThreads, smem), "map occupancy");
  const int per_sm = std::max(blocks, 1);
  const int64_t total = args.tiles_per_batch * args.batches;
  const int64_t grid = std::min<int64_t>(total, static_cast<int64_t>(per_sm) * SmCount());
  kernel<<<static_cast<unsigned>(grid), kThreads, smem, stream>>>(args);
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

void Check(cudaError_t status, const char* what) {
  if (status != cudaSuccess) {
    // Clear the runtime's last-error slot so the next launch check does not
    // report this (non-sticky) failure again.
    (void)cudaGetLastError();
    throw std::runtime_error(std::string("CUDA ") + what + ": " + cudaGetErrorString(status));
  }
}

void MapStageElements(const MapRecord* recs, int64_t count, int32_t element_bytes, int64_t* tile, int64_t* base) {
  const int64_t vec = 16 / element_bytes;
  *tile = 0;
  *base = 0;
  for (int64_t i = 0; i < count; ++i) {
    const int64_t t0 = recs[i].t[0], t1 = recs[i].t[1], t2 = recs[i].t[2];
    const int64_t rows_of_x = t1 * t2 * RowPitch(t0, vec);
    const int64_t need = recs[i].mode == kDirect
                             ? rows_of_x
                             : std::max(t0 * t2 * RowPitch(t1, vec), t0 * RowPitch(t1 * t2, vec));
    *tile = std::max(*tile, need);
    *base = std::max(*base, rows_of_x);
  }
  *tile = (*tile + vec - 1) / vec * vec;   // the base stage starts on a 16-byte boundary
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
