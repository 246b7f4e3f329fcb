// Map and reduce engines: the grouped strided permute / accumulate / update
// kernel and the two-pass segmented reduction for partial traces.
//
// The map kernel is one persistent grid over every tile of every record of
// every batch; each CTA walks a contiguous range of tiles.  A tile is a box
// over the record's destination-innermost axis X, its source-innermost axis Y
// and one further axis Z.  One thread decodes the tile (record cursor, chunk
// coordinates, outer axes) into shared memory.  The CTA then copies the tile
// in contiguous runs: source runs (Y, continued by Z when Z follows Y in the
// source) into shared memory, and destination runs (X, continued by Y when Y
// follows X in the destination) out of it.  Lanes stride each run, so reads
// and writes are coalesced and each element costs a few integer operations.
// When X and Y coincide the tile is copied run by run without staging.
#include "engine.h"

#include "arith.cuh"

#include <algorithm>
#include <atomic>

namespace t0b {

std::atomic<uint64_t> g_kernel_launches{0};

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

// Division by a runtime divisor in [1, 2^24) for dividends below 2^24:
// n / d = (umulhi(n, m) + n) >> l with l = ceil(log2 d) and
// m = floor(2^32 (2^l - d) / d) + 1 (round-up multiplier method).
struct FastDiv {
  uint32_t m, l;
  __device__ __forceinline__ FastDiv() = default;
  __device__ __forceinline__ FastDiv(uint32_t magic, uint32_t shift) : m(magic), l(shift) {}
  __device__ __forceinline__ static FastDiv Of(uint32_t divisor) {
    const uint32_t shift = 32 - __clz(divisor - 1);
    const uint64_t one = 1;
    return FastDiv(static_cast<uint32_t>(((one << 32) * ((one << shift) - divisor)) / divisor + 1), shift);
  }
  __device__ __forceinline__ uint32_t Div(uint32_t n) const { return (__umulhi(n, m) + n) >> l; }
};

// A decoded tile, shared by the CTA.  In-tile offsets use Off (int32 unless
// the plan marked a record wide).
template <typename Off>
struct TileState {
  int64_t so, dof;        // element offsets of the tile origin, batch included
  Off sx, sy, sz, dx, dy, dz;
  int ex, ey, ez;         // tile extents (edge tiles are smaller)
  int px, pz;             // shared-memory pitches along Y (odd, >= ex) and Z
  int mode, slot;
  int src_runs, src_len;  // source runs: ex runs of ey*ez (Z follows Y) or ex*ez runs of ey
  int dst_runs, dst_len;  // destination runs: ez runs of ex*ey (Y follows X) or ey*ez runs of ex
  int src_linear, dst_linear;
  FastDiv div_x, div_y, div_src, div_dst;   // by ex, by ey, by src_len, by dst_len
  int64_t batch;
  alignas(16) unsigned char coef[32];       // the tile's coefficients, fetched by the decoding thread
};

// Thread 0 only: advance the record cursor to the tile and decode it.
template <typename Off>
__device__ __forceinline__ void DecodeTile(const MapArgs& a, int64_t tile, int64_t& cursor, TileState<Off>& s) {
  const int64_t batch = tile / a.tiles_per_batch;
  const int64_t local = tile - batch * a.tiles_per_batch;
  if (cursor < 0 || a.recs[cursor].tile_begin > local) {
    int64_t lo = 0, hi = a.nrec - 1;
    while (lo < hi) {
      const int64_t mid = (lo + hi + 1) >> 1;
      if (a.recs[mid].tile_begin <= local) lo = mid; else hi = mid - 1;
    }
    cursor = lo;
  }
  while (cursor + 1 < a.nrec && a.recs[cursor + 1].tile_begin <= local) ++cursor;
  const MapRecord& r = a.recs[cursor];
  uint32_t q = static_cast<uint32_t>(local - r.tile_begin);
  const uint32_t c0 = r.c[0], c1 = r.c[1], c2 = r.c[2];
  const uint32_t cx = q % c0; q /= c0;
  const uint32_t cy = q % c1; q /= c1;
  const uint32_t cz = q % c2; q /= c2;
  int64_t so = r.src_off + batch * a.src_size;
  int64_t dof = r.dst_off + batch * a.out_size;
  for (int i = 0; i < r.nouter; ++i) {
    const uint32_t n = static_cast<uint32_t>(r.n[3 + i]);
    const uint32_t idx = q % n;
    q /= n;
    so += static_cast<int64_t>(idx) * r.s[3 + i];
    dof += static_cast<int64_t>(idx) * r.d[3 + i];
  }
  const int x0 = cx * r.t[0], y0 = cy * r.t[1], z0 = cz * r.t[2];
  const int ex = min(r.t[0], r.n[0] - x0);
  const int ey = min(r.t[1], r.n[1] - y0);
  const int ez = min(r.t[2], r.n[2] - z0);
  s.ex = ex; s.ey = ey; s.ez = ez;
  s.so = so + x0 * r.s[0] + y0 * r.s[1] + z0 * r.s[2];
  s.dof = dof + x0 * r.d[0] + y0 * r.d[1] + z0 * r.d[2];
  s.sx = static_cast<Off>(r.s[0]); s.sy = static_cast<Off>(r.s[1]); s.sz = static_cast<Off>(r.s[2]);
  s.dx = static_cast<Off>(r.d[0]); s.dy = static_cast<Off>(r.d[1]); s.dz = static_cast<Off>(r.d[2]);
  s.px = r.t[0] | 1;
  s.pz = s.px * r.t[1];
  s.mode = r.mode;
  s.slot = r.coef_slot;
  // Z continues the source run of Y when sz = ey * sy and the shared-memory
  // Z pitch equals px * ey (a full-height tile); Y continues the destination
  // run of X when dy = ex * dx.
  s.src_linear = ez > 1 && r.s[2] == static_cast<int64_t>(ey) * r.s[1] && ey == r.t[1];
  s.dst_linear = ey > 1 && r.d[1] == static_cast<int64_t>(ex) * r.d[0];
  if (r.mode == kDirect) {
    // Runs along X on both sides, one per (y, z).
    s.src_linear = 0;
    s.dst_linear = 0;
    s.src_runs = ey * ez;
    s.src_len = ex;
  } else {
    s.src_runs = s.src_linear ? ex : ex * ez;
    s.src_len = s.src_linear ? ey * ez : ey;
  }
  s.dst_runs = s.dst_linear ? ez : ey * ez;
  s.dst_len = s.dst_linear ? ex * ey : ex;
  s.div_x = FastDiv::Of(static_cast<uint32_t>(ex));
  s.div_y = FastDiv::Of(static_cast<uint32_t>(ey));
  s.div_src = FastDiv::Of(static_cast<uint32_t>(s.src_len));
  s.div_dst = FastDiv::Of(static_cast<uint32_t>(s.dst_len));
  s.batch = batch;
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

// Walk `runs` runs of `len` elements.  Runs of 32 elements or more take a
// whole warp and lanes stride them (unrolled, so several loads are in flight);
// shorter runs are packed several to a warp, one element per lane.
// start(run) -> per-run state; f(state, j) handles element j of the run.
template <typename StartF, typename F>
__device__ __forceinline__ void WalkRuns(int runs, int len, FastDiv by_len, StartF&& start, F&& f) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (len >= 32) {
    for (int r = warp; r < runs; r += kWarps) {
      const auto state = start(r);
#pragma unroll 4
      for (int j = lane; j < len; j += 32) f(state, j);
    }
  } else {
    // Element e of the packed sequence: run e / len, element e % len.
    const int total = runs * len;
    for (int e0 = warp * 32; e0 < total; e0 += kThreads * 4) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int e = e0 + u * kThreads + lane;
        if (e < total) {
          const int r = static_cast<int>(by_len.Div(static_cast<uint32_t>(e)));
          f(start(r), e - r * len);
        }
      }
    }
  }
}

template <typename Off>
struct Run { Off a, b; };

template <typename Off>
struct Run3 { Off a, b; int c; };

// Asynchronous global -> shared copy of one element (no register round trip).
template <int Bytes>
__device__ __forceinline__ void CopyAsync(void* smem, const void* gmem) {
  const unsigned dst = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  if constexpr (Bytes == 16) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(gmem) : "memory");
  } else {
    asm volatile("cp.async.ca.shared.global [%0], [%1], %2;\n" ::"r"(dst), "l"(gmem), "n"(Bytes) : "memory");
  }
}

__device__ __forceinline__ void WaitAsync() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }

template <int Op, typename T, typename CA, typename CB, typename Off>
__global__ void __launch_bounds__(kThreads, 4) MapKernel(MapArgs args) {
  using E = Emit<Op, T, CA, CB>;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ TileState<Off> states[2];        // the current tile and the next one
  T* tile = reinterpret_cast<T*>(smem_raw);
  T* base_tile = tile + args.tile_elems;     // update: destination base values, in run order
  const int64_t total = args.tiles_per_batch * args.batches;
  const int64_t per_cta = (total + gridDim.x - 1) / gridDim.x;
  const int64_t first = static_cast<int64_t>(blockIdx.x) * per_cta;
  const int64_t last = min(total, first + per_cta);
  int64_t cursor = -1;   // record cursor, meaningful in thread 0 only
  if (threadIdx.x == 0 && first < last) {
    DecodeTile<Off>(args, first, cursor, states[0]);
    E::Fetch(args, states[0].slot, states[0].batch, states[0].coef);
  }
  __syncthreads();
  int buffer = 0;
  for (int64_t t = first; t < last; ++t, buffer ^= 1) {
    const TileState<Off>& st = states[buffer];
    const E emit(st.coef);
    const T* __restrict__ src = static_cast<const T*>(args.src) + st.so;
    const T* __restrict__ base = static_cast<const T*>(args.base) + st.dof;
    T* __restrict__ out = static_cast<T*>(args.out) + st.dof;
    const bool skip = emit.SkipSource();
    const bool needs_base = E::kReadsBase && emit.NeedsBase();
    const int ex = st.ex, ey = st.ey;
    const bool direct = st.mode == kDirect;
    const int px = st.px, pz = st.pz;
    const Off dx = st.dx, dy = st.dy, dz = st.dz;
    const bool dst_linear = st.dst_linear;
    const FastDiv by_x = st.div_x, by_y = st.div_y;
    const int dst_runs = st.dst_runs, dst_len = st.dst_len;
    const FastDiv div_dst = st.div_dst;
    // Destination run r: its tile offset and its destination offset.
    auto dst_run = [&](int r) {
      if (dst_linear) return Run<Off>{static_cast<Off>(pz * r), static_cast<Off>(r * dz)};
      const int z = static_cast<int>(by_y.Div(static_cast<uint32_t>(r)));
      const int y = r - z * ey;
      return Run<Off>{static_cast<Off>(px * y + pz * z), static_cast<Off>(y * dy + z * dz)};
    };
    // Load: source runs into tile[x + px * y + pz * z]; base values (update) into base_tile.
    if (!skip) {
      const Off sx = st.sx, sy = st.sy, sz = st.sz;
      const bool linear = st.src_linear;
      const Off step = direct ? sx : sy;        // source stride along a run
      const int pitch = direct ? 1 : px;        // tile stride along a run
      WalkRuns(st.src_runs, st.src_len, st.div_src,
          [&](int r) {
            if (direct) return Run<Off>{static_cast<Off>(r * sz), static_cast<Off>(pz * r)};
            if (linear) return Run<Off>{static_cast<Off>(r * sx), static_cast<Off>(r)};
            const int z = static_cast<int>(by_x.Div(static_cast<uint32_t>(r)));
            const int x = r - z * ex;
            return Run<Off>{static_cast<Off>(x * sx + z * sz), static_cast<Off>(x + pz * z)};
          },
          [&](const Run<Off>& run, int j) { CopyAsync<sizeof(T)>(tile + run.b + j * pitch, src + run.a + j * step); });
    }
    if constexpr (E::kReadsBase) {
      if (needs_base) {
        WalkRuns(dst_runs, dst_len, div_dst,
            [&](int r) { return Run<Off>{static_cast<Off>(r * dst_len), dst_run(r).b}; },
            [&](const Run<Off>& run, int k) { CopyAsync<sizeof(T)>(base_tile + run.a + k, base + run.b + k * dx); });
      }
    }
    // While the copies fly, the decoding thread prepares the next tile.
    if (threadIdx.x == 0 && t + 1 < last) {
      TileState<Off>& next = states[buffer ^ 1];
      DecodeTile<Off>(args, t + 1, cursor, next);
      E::Fetch(args, next.slot, next.batch, next.coef);
    }
    WaitAsync();
    __syncthreads();
    // Store: destination runs out of the tile, with the rule specialised per kind.
    auto store = [&](auto kind) {
      constexpr int K = decltype(kind)::value;
      WalkRuns(dst_runs, dst_len, div_dst,
          [&](int r) {
            const Run<Off> run = dst_run(r);
            return Run3<Off>{run.a, run.b, r * dst_len};
          },
          [&](const Run3<Off>& run, int k) {
            // Linear runs cover (x, y) with x fastest: k = x + ex * y.
            int at_tile = run.a + k;
            if (dst_linear) at_tile += (px - ex) * static_cast<int>(by_x.Div(static_cast<uint32_t>(k)));
            T v{}, old{};
            if (!skip) v = tile[at_tile];
            if constexpr (E::kReadsBase) {
              if (needs_base) old = base_tile[run.c + k];
            }
            out[run.b + k * dx] = emit.template Apply<K>(v, old);
          });
    };
    switch (emit.Kind()) {
      case 1: store(std::integral_constant<int, 1>{}); break;
      case 2: store(std::integral_constant<int, 2>{}); break;
      default: store(std::integral_constant<int, 0>{}); break;
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
  static int per_sm = [&] {
    Check(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024), "map attribute");
    return 0;
  }();
  int blocks = 0;
  Check(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kernel, kThreads, smem), "map occupancy");
  per_sm = std::max(blocks, 1);
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
  if (status != cudaSuccess) throw std::runtime_error(std::string("CUDA ") + what + ": " + cudaGetErrorString(status));
}

void MapTileElements(const MapRecord* recs, int64_t count, int64_t* tile, int64_t* box) {
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
