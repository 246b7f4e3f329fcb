// Grouped transform: the non-abelian (SU2) permute's multi-tree groups in one
// pass.  The reference packs each group's source blocks into rows
// (copy_p), multiplies by the group's small dense basis matrix (an XLA dot),
// and unpacks the rows into the destination blocks (update_p / copy_p),
// _stride/_tensor_ops.py:119-203, with the matrices from
// crates/tensor0-core/src/transform/tree_transformers.rs:244-271.  Here each
// element position of a group's block is read once from every source block;
// every destination row's sum sum_i M[j][i] * v_i is formed in source order
// and written once.  The HBM traffic is one read per distinct source element
// and one write per destination element; no packed intermediate exists.
//
// Element groups (the first source innermost along X, the destination's
// innermost axis) give a thread one element.  Tiled groups stage a
// tx x ty x tz tile of every source in shared memory with asynchronous
// copies, lanes along Y (the source's innermost axis), and write every
// destination with lanes along X.  A CTA walks a contiguous range of units, so the group is looked
// up once and then advanced.
//
// Single-tree groups (1 x 1 matrices) follow the reference's direct path,
// the accumulation of one record into zeros (_tensor_ops.py:168-176):
// coefficient 0 writes +0, coefficient 1 copies (0 + x), others scale.
#include "engine.h"

#include "arith.cuh"
#include "copy_async.cuh"

#include <algorithm>

namespace t0b {
namespace {

constexpr int kGroupedThreads = kGroupedTile;
constexpr int kSourceRegisters = 4;   // element groups with up to this many sources keep them in registers

template <typename T, typename M>
__device__ __forceinline__ T Term(M m, T v) { return Scale(m, v); }

__device__ __forceinline__ int64_t FindGrouped(const GroupedGroup* groups, int64_t n, int64_t unit) {
  int64_t lo = 0, hi = n - 1;
  while (lo < hi) {
    const int64_t mid = (lo + hi + 1) >> 1;
    if (groups[mid].unit_begin <= unit) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ int64_t Address(const GroupedOperand& op, const int (&idx)[kMaxRank], int rank) {
  int64_t at = op.offset;
#pragma unroll
  for (int a = 0; a < kMaxRank; ++a) {
    if (a < rank) at += static_cast<int64_t>(idx[a]) * op.s[a];
  }
  return at;
}

// Destination j's value from the sources' values at one element position.
template <typename T, typename M, typename Value>
__device__ __forceinline__ T Combine(const M* row, int n_src, Value value) {
  T acc = Term(row[0], value(0));
  if (n_src <= kSourceRegisters) {
#pragma unroll
    for (int i = 1; i < kSourceRegisters; ++i) {
      if (i < n_src) acc = Add(acc, Term(row[i], value(i)));
    }
    return acc;
  }
  for (int i = 1; i < n_src; ++i) acc = Add(acc, Term(row[i], value(i)));
  return acc;
}

// Every destination of one element position; single-tree groups use the
// direct accumulation rule.
template <typename T, typename M, typename Value, typename Store>
__device__ __forceinline__ void EmitAll(const M* matrix, int n_src, int n_dst, Value value, Store store) {
  if (n_src == 1 && n_dst == 1) {
    const M c = matrix[0];
    const T v = value(0);
    store(0, IsZero(c) ? T{} : PlusZero(IsOne(c) ? v : Scale(c, v)));
    return;
  }
  for (int j = 0; j < n_dst; ++j) store(j, Combine<T>(matrix + static_cast<int64_t>(j) * n_src, n_src, value));
}

template <typename T, typename M>
__global__ void __launch_bounds__(kGroupedThreads) GroupedKernel(GroupedArgs args) {
  extern __shared__ __align__(16) unsigned char grouped_stage[];
  T* stage = reinterpret_cast<T*>(grouped_stage);
  __shared__ int64_t tile_base[kTiledOperands];
  __shared__ int64_t tile_sx[kTiledOperands];
  __shared__ int64_t tile_sy[kTiledOperands];
  __shared__ int64_t tile_sz[kTiledOperands];
  __shared__ int tile_w[3];
  const int64_t total = args.units * args.batches;
  const M* __restrict__ matrices = static_cast<const M*>(args.matrices);
  const int64_t per_cta = (total + gridDim.x - 1) / gridDim.x;
  const int64_t first = static_cast<int64_t>(blockIdx.x) * per_cta;
  const int64_t last = min(total, first + per_cta);
  if (first >= last) return;
  int64_t batch = first / args.units;
  int64_t unit = first - batch * args.units;
  int64_t group = FindGrouped(args.groups, args.ngroups, unit);
  for (int64_t u = first; u < last; ++u, ++unit) {
    if (unit == args.units) {
      unit = 0;
      ++batch;
      group = 0;
    }
    while (group + 1 < args.ngroups && args.groups[group + 1].unit_begin <= unit) ++group;
    const GroupedGroup& g = args.groups[group];
    const T* __restrict__ src = static_cast<const T*>(args.src) + batch * args.src_size;
    T* __restrict__ out = static_cast<T*>(args.out) + batch * args.out_size;
    const GroupedOperand* ops = args.operands + g.operand_begin;
    const M* matrix = matrices + g.matrix_offset;
    const int n_src = g.n_src, n_dst = g.n_dst, rank = g.rank;
    if (g.tiled) {
      // Unit -> (tile along X, Y and axis 2, index of the remaining axes);
      // one thread per operand puts that operand's tile origin and tile-axis
      // strides in shared memory.
      const int n_ops = n_src + n_dst;
      for (int t = threadIdx.x; t < n_ops; t += kGroupedThreads) {
        const uint32_t local = static_cast<uint32_t>(unit - g.unit_begin);
        const uint32_t q = Division(g.div_tiles_x).Div(local);
        const uint32_t tile_x = local - q * static_cast<uint32_t>(g.tiles_x);
        const uint32_t q2 = Division(g.div_tiles_y).Div(q);
        const uint32_t tile_y = q - q2 * static_cast<uint32_t>(g.tiles_y);
        const uint32_t rest = Division(g.div_tiles_z).Div(q2);
        const uint32_t tile_z = q2 - rest * static_cast<uint32_t>(g.tiles_z);
        const GroupedOperand& op = ops[t];
        int64_t at = op.offset + static_cast<int64_t>(tile_x) * g.tx * op.s[0] +
                     static_cast<int64_t>(tile_y) * g.ty * op.s[1] + static_cast<int64_t>(tile_z) * g.tz * op.s[2];
        uint32_t r = rest;
        for (int a = 3; a < rank; ++a) {
          const uint32_t next = Division(g.div_n[a]).Div(r);
          at += static_cast<int64_t>(r - next * static_cast<uint32_t>(g.n[a])) * op.s[a];
          r = next;
        }
        tile_base[t] = at;
        tile_sx[t] = op.s[0];
        tile_sy[t] = op.s[1];
        tile_sz[t] = op.s[2];
        if (t == 0) {
          tile_w[0] = min(g.tx, g.n[0] - static_cast<int>(tile_x) * g.tx);
          tile_w[1] = min(g.ty, g.n[1] - static_cast<int>(tile_y) * g.ty);
          tile_w[2] = min(g.tz, g.n[2] - static_cast<int>(tile_z) * g.tz);
        }
      }
      __syncthreads();
      const int tx = g.tx, ty = g.ty, pitch = g.tx + 1;
      const int wx = tile_w[0], wy = tile_w[1], wz = tile_w[2];
      const int tx_shift = __ffs(tx) - 1, ty_shift = __ffs(ty) - 1;
      const int plane_shift = tx_shift + ty_shift;
      const int tile_shift = plane_shift + __ffs(g.tz) - 1;
      const int rows = 1 << (tile_shift - tx_shift);   // (axis 2, Y) rows of one source's stage
      // Load: lanes along Y, then X, then axis 2, as asynchronous copies into
      // shared memory: a thread's whole share of the tile is in flight at once.
      const int items = n_src << tile_shift;
      const uint32_t stage_s = static_cast<uint32_t>(__cvta_generic_to_shared(stage));
      for (int k = threadIdx.x; k < items; k += kGroupedThreads) {
        const int i = k >> tile_shift;
        const int within = k & ((1 << tile_shift) - 1);
        const int lz = within >> plane_shift;
        const int lx = (within >> ty_shift) & (tx - 1), ly = within & (ty - 1);
        if (lx < wx && ly < wy && lz < wz) {
          const int slot = (i * rows + (lz << ty_shift) + ly) * pitch + lx;
          CopyAsync<sizeof(T)>(stage_s + static_cast<uint32_t>(slot * sizeof(T)),
                               src + tile_base[i] + lx * tile_sx[i] + ly * tile_sy[i] + lz * tile_sz[i]);
        }
      }
      asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;\n" ::: "memory");
      __syncthreads();
      // Combine and store: lanes along X, then Y, then axis 2.
      for (int k = threadIdx.x; k < (1 << tile_shift); k += kGroupedThreads) {
        const int lx = k & (tx - 1), ly = (k >> tx_shift) & (ty - 1), lz = k >> plane_shift;
        if (lx < wx && ly < wy && lz < wz) {
          const int row = (lz << ty_shift) + ly;
          EmitAll<T>(matrix, n_src, n_dst, [&](int i) { return stage[(i * rows + row) * pitch + lx]; },
                     [&](int j, T value) {
                       const int o = n_src + j;
                       out[tile_base[o] + lx * tile_sx[o] + ly * tile_sy[o] + lz * tile_sz[o]] = value;
                     });
        }
      }
      __syncthreads();
      continue;
    }
    const int64_t e = (unit - g.unit_begin) * kGroupedTile + threadIdx.x;
    if (e >= g.elements) continue;
    int idx[kMaxRank];
    uint32_t rest = static_cast<uint32_t>(e);
#pragma unroll
    for (int a = 0; a < kMaxRank; ++a) {
      if (a < rank) {
        const uint32_t next = Division(g.div_n[a]).Div(rest);
        idx[a] = static_cast<int>(rest - next * static_cast<uint32_t>(g.n[a]));
        rest = next;
      } else {
        idx[a] = 0;
      }
    }
    if (n_src <= kSourceRegisters) {
      T v[kSourceRegisters];
#pragma unroll
      for (int i = 0; i < kSourceRegisters; ++i) {
        if (i < n_src) v[i] = src[Address(ops[i], idx, rank)];
      }
      EmitAll<T>(matrix, n_src, n_dst, [&](int i) { return v[i]; },
                 [&](int j, T value) { out[Address(ops[n_src + j], idx, rank)] = value; });
    } else {
      // Wide groups: sources are re-read per destination row (from L1/L2).
      EmitAll<T>(matrix, n_src, n_dst, [&](int i) { return src[Address(ops[i], idx, rank)]; },
                 [&](int j, T value) { out[Address(ops[n_src + j], idx, rank)] = value; });
    }
  }
}

template <typename F>
void WithGroupedTypes(int32_t dtype, int32_t matrix_dtype, F&& f) {
  switch (dtype) {
    case 11:
      if (matrix_dtype == 11) return f(static_cast<float*>(nullptr), static_cast<float*>(nullptr));
      break;
    case 12:
      if (matrix_dtype == 12) return f(static_cast<double*>(nullptr), static_cast<double*>(nullptr));
      break;
    case 15:
      if (matrix_dtype == 11) return f(static_cast<float2*>(nullptr), static_cast<float*>(nullptr));
      if (matrix_dtype == 15) return f(static_cast<float2*>(nullptr), static_cast<float2*>(nullptr));
      break;
    case 18:
      if (matrix_dtype == 12) return f(static_cast<double2*>(nullptr), static_cast<double*>(nullptr));
      if (matrix_dtype == 18) return f(static_cast<double2*>(nullptr), static_cast<double2*>(nullptr));
      break;
    default:
      throw InvalidArgumentError("CUDA stride storage supports only F32/F64/C64/C128");
  }
  throw InvalidArgumentError("grouped matrices must be the storage's real type or, for complex storage, its complex type");
}

}  // namespace

void LaunchGrouped(int32_t dtype, int32_t matrix_dtype, const GroupedArgs& args, int64_t stage_bytes,
                   cudaStream_t stream) {
  WithGroupedTypes(dtype, matrix_dtype, [&](auto* t, auto* m) {
    using T = std::remove_pointer_t<decltype(t)>;
    using M = std::remove_pointer_t<decltype(m)>;
    const int64_t total = args.units * args.batches;
    if (total == 0) return;
    const int64_t grid = std::min<int64_t>(total, int64_t{SmCount()} * 8);
    auto kernel = GroupedKernel<T, M>;
    if (stage_bytes > 48 * 1024) {
      Check(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(stage_bytes)),
            "grouped shared memory");
    }
    kernel<<<static_cast<unsigned>(grid), kGroupedThreads, static_cast<size_t>(stage_bytes), stream>>>(args);
    Check(cudaGetLastError(), "grouped launch");
    g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
  });
}

}  // namespace t0b
