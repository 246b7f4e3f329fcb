// C ABI (include/tensor0_b200.h): argument validation before any write, then
// stream-ordered launches.  No entry point synchronizes, allocates or reads
// device memory on the host.
#include "../../include/tensor0_b200.h"

#include "engine.h"
#include "gemm.h"
#include "layout.h"
#include "plan.h"

#include <atomic>
#include <cstdio>
#include <cstring>
#include <memory>
#include <new>

struct t0b_plan {
  t0b::Plan plan;
  int map_smem = 0;        // dynamic shared memory of one map CTA (bytes)
  int64_t tile_elems = 0;  // staged-tile elements; update plans place the base buffer after them
};

namespace {

std::atomic<uint64_t> g_created{0};
std::atomic<uint64_t> g_destroyed{0};

void Message(char* error, size_t size, const char* text) {
  if (error != nullptr && size != 0) std::snprintf(error, size, "%s", text);
}

// Run `body`, mapping invalid arguments to 1 and everything else to 2.
template <typename Body>
int Guard(char* error, size_t size, Body&& body) {
  try {
    body();
    return 0;
  } catch (const t0b::InvalidArgument& e) {
    Message(error, size, (std::string("tensor0-b200: ") + e.what()).c_str());
    return 1;
  } catch (const std::bad_alloc&) {
    Message(error, size, "tensor0-b200: out of host memory");
    return 2;
  } catch (const std::exception& e) {
    Message(error, size, (std::string("tensor0-b200: ") + e.what()).c_str());
    return 2;
  } catch (...) {
    Message(error, size, "tensor0-b200: unknown exception");
    return 2;
  }
}

int ElementBytes(int32_t dtype) {
  switch (dtype) {
    case T0B_F32: return 4;
    case T0B_F64: case T0B_C64: return 8;
    case T0B_C128: return 16;
    default: throw t0b::InvalidArgument("CUDA stride storage supports only F32/F64/C64/C128");
  }
}

int CoefficientBytes(int32_t coefficient, int32_t storage) {
  const bool complex = storage == T0B_C64 || storage == T0B_C128;
  const bool single = storage == T0B_F32 || storage == T0B_C64;
  if (coefficient == T0B_S32) return 4;
  if (coefficient == (single ? T0B_F32 : T0B_F64)) return single ? 4 : 8;
  if (complex && coefficient == (single ? T0B_C64 : T0B_C128)) return single ? 8 : 16;
  throw t0b::InvalidArgument("unsupported CUDA coefficient dtype; expected S32 or matching real/complex precision");
}

uint64_t Bytes(uint64_t elements, uint64_t item) {
  uint64_t out = 0;
  if (!t0b::CheckedMul(elements, item, &out) || out > static_cast<uint64_t>(PTRDIFF_MAX)) {
    throw t0b::InvalidArgument("buffer size exceeds addressable storage");
  }
  return out;
}

// The reference's overlap rule (ffi/buffers.h:43-52).
void Disjoint(const void* a, uint64_t a_bytes, const void* b, uint64_t b_bytes) {
  if (a_bytes == 0 || b_bytes == 0) return;
  const auto x = reinterpret_cast<uintptr_t>(a), y = reinterpret_cast<uintptr_t>(b);
  const bool overlap = x <= y ? y - x < a_bytes : x - y < b_bytes;
  if (overlap) throw t0b::InvalidArgument("input and output buffers overlap");
}

// Storage buffers are aligned to their element size: the map engine copies
// whole elements asynchronously (16 bytes at a time for C128).
void RequireAligned(const void* buffer, int element_bytes, const char* what) {
  if (buffer != nullptr && reinterpret_cast<uintptr_t>(buffer) % static_cast<uintptr_t>(element_bytes) != 0) {
    throw t0b::InvalidArgument(std::string(what) + " buffer is not aligned to its element size");
  }
}

// The device table holds 16-byte records read with vector loads.
void RequireTableAligned(const int64_t* table) {
  if (reinterpret_cast<uintptr_t>(table) % 16 != 0) {
    throw t0b::InvalidArgument("device descriptor table is not 16-byte aligned");
  }
}

const t0b::TableHeader& Header(const t0b_plan* plan) {
  return *reinterpret_cast<const t0b::TableHeader*>(plan->plan.table.data());
}

void RequirePlan(const t0b_plan* plan, int32_t operation, int32_t dtype, int64_t batches) {
  if (plan == nullptr) throw t0b::InvalidArgument("plan is null");
  if (plan->plan.operation != operation) throw t0b::InvalidArgument("plan was built for another operation");
  if (ElementBytes(dtype) != plan->plan.element_bytes) {
    throw t0b::InvalidArgument("storage dtype does not match the plan's element size");
  }
  if (batches < 0) throw t0b::InvalidArgument("batch count must be nonnegative");
}

uint64_t CoefficientCount(int64_t count, int64_t batches) {
  if (count != 1 && count != batches) {
    throw t0b::InvalidArgument("coefficients must be shared (one value) or one value per batch");
  }
  return static_cast<uint64_t>(count);
}

void RunMap(const t0b_plan* plan, int op, int32_t dtype, int32_t ca_dtype, int32_t cb_dtype,
            const void* src, const void* base, void* out, int64_t batches, const void* ca, int64_t ca_count,
            const void* cb, int64_t cb_count, const int64_t* table, cudaStream_t stream) {
  const auto& h = Header(plan);
  t0b::MapArgs args{};
  args.recs = reinterpret_cast<const t0b::MapRecord*>(table + h.map_offset);
  args.nrec = h.map_records;
  args.tiles_per_batch = h.map_tiles;
  args.batches = batches;
  args.src = src;
  args.base = base;
  args.out = out;
  args.src_size = static_cast<int64_t>(plan->plan.source_size);
  args.out_size = static_cast<int64_t>(plan->plan.output_size);
  args.tile_elems = plan->tile_elems;
  args.ca = ca;
  args.ca_count = ca_count;
  args.cb = cb;
  args.cb_count = cb_count;
  args.conjugate = plan->plan.conjugate ? 1 : 0;
  t0b::LaunchMap(op, dtype, ca_dtype, cb_dtype, args, plan->map_smem, plan->plan.map_wide, stream);
}

void RunReduce(const t0b_plan* plan, int32_t dtype, int32_t ca_dtype, const void* src, void* out,
               int64_t batches, const void* ca, int64_t ca_count, void* scratch, const int64_t* table,
               cudaStream_t stream) {
  const auto& h = Header(plan);
  for (const auto& wave : plan->plan.waves) {
    t0b::ReduceArgs args{};
    args.groups = reinterpret_cast<const t0b::ReduceGroup*>(table + h.group_offset);
    args.records = reinterpret_cast<const t0b::ReduceRecord*>(table + h.reduce_offset);
    args.group_begin = wave.group_begin;
    args.group_end = wave.group_end;
    args.task_begin = wave.task_begin;
    args.task_end = wave.task_end;
    args.owner_begin = wave.owner_begin;
    args.owner_end = wave.owner_end;
    args.batches = batches;
    args.src = src;
    args.out = out;
    args.scratch = scratch;
    args.scratch_stride = h.scratch;
    args.src_size = static_cast<int64_t>(plan->plan.source_size);
    args.out_size = static_cast<int64_t>(plan->plan.output_size);
    args.ca = ca;
    args.ca_count = ca_count;
    args.conjugate = plan->plan.conjugate ? 1 : 0;
    args.assign = plan->plan.reduce_assign ? 1 : 0;
    t0b::LaunchReduce(dtype, ca_dtype, args, stream);
  }
}

// Shared body of accumulation and reduction.
void Sum(const t0b_plan* plan, int32_t operation, int32_t dtype, const void* source, void* output,
         int64_t batches, const void* coefficients, int32_t coefficient_dtype, int64_t coefficient_count,
         void* scratch, const int64_t* table, cudaStream_t stream) {
  RequirePlan(plan, operation, dtype, batches);
  const auto& p = plan->plan;
  const int eb = p.element_bytes;
  const uint64_t b = static_cast<uint64_t>(batches);
  const uint64_t out_bytes = Bytes(b * p.output_size, eb);
  const uint64_t src_bytes = Bytes(b * p.source_size, eb);
  const uint64_t scratch_bytes = Bytes(b * p.scratch, eb);
  if (b != 0 && p.output_size != 0 && output == nullptr) throw t0b::InvalidArgument("output buffer is null");
  if (b != 0 && p.source_size != 0 && source == nullptr) throw t0b::InvalidArgument("source buffer is null");
  RequireAligned(source, eb, "source");
  RequireAligned(output, eb, "output");
  Disjoint(source, src_bytes, output, out_bytes);
  const size_t table_bytes = p.table.size() * sizeof(int64_t);
  if (table == nullptr) throw t0b::InvalidArgument("device descriptor table is null");
  RequireTableAligned(table);
  Disjoint(table, table_bytes, output, out_bytes);
  uint64_t count = 1;
  int coef_bytes = 4;
  if (p.coefficient_rows != 0) {
    coef_bytes = CoefficientBytes(coefficient_dtype, dtype);
    count = CoefficientCount(coefficient_count, batches);
    if (coefficients == nullptr) throw t0b::InvalidArgument("coefficient buffer is null");
    RequireAligned(coefficients, coef_bytes, "coefficient");
    Disjoint(coefficients, Bytes(p.coefficient_rows * count, coef_bytes), output, out_bytes);
  } else {
    coefficient_dtype = T0B_S32;
  }
  if (p.scratch != 0 && b != 0) {
    if (scratch == nullptr) throw t0b::InvalidArgument("scratch buffer is null but the plan needs scratch");
    Disjoint(scratch, scratch_bytes, output, out_bytes);
    Disjoint(scratch, scratch_bytes, source, src_bytes);
    Disjoint(scratch, scratch_bytes, table, table_bytes);
  }
  if (b == 0 || p.output_size == 0) return;
  if (!p.full_coverage) {
    t0b::Check(cudaMemsetAsync(output, 0, out_bytes, stream), "memset");
  }
  if (p.has_map) {
    RunMap(plan, t0b::kOpAccumulation, dtype, coefficient_dtype, T0B_S32, source, nullptr, output, batches,
           coefficients, static_cast<int64_t>(count), nullptr, 1, table, stream);
  }
  if (p.has_reduce) {
    RunReduce(plan, dtype, coefficient_dtype, source, output, batches, coefficients,
              static_cast<int64_t>(count), scratch, table, stream);
  }
}

}  // namespace

extern "C" {

const char* t0b_version(void) { return "tensor0-b200 0.1 (sm_100a)"; }

int t0b_plan_create(int32_t operation, const int64_t* words, size_t word_count,
                    const int64_t* coefficient_records, size_t coefficient_count,
                    int32_t element_bytes, uint32_t flags, t0b_plan** plan,
                    char* error, size_t error_size) {
  return Guard(error, error_size, [&] {
    if (plan == nullptr) throw t0b::InvalidArgument("plan output pointer is null");
    *plan = nullptr;
    if (coefficient_records == nullptr && coefficient_count != 0) {
      throw t0b::InvalidArgument("coefficient record list is null");
    }
    auto built = std::make_unique<t0b_plan>();
    built->plan = t0b::BuildPlan(operation, words, word_count, coefficient_records, coefficient_count,
                                 element_bytes, flags);
    const auto& h = *reinterpret_cast<const t0b::TableHeader*>(built->plan.table.data());
    int64_t tile = 0, box = 0;
    t0b::MapTileElements(reinterpret_cast<const t0b::MapRecord*>(built->plan.table.data() + h.map_offset),
                         h.map_records, element_bytes, &tile, &box);
    // Update plans also stage the destination's base values, in the tile's layout.
    built->tile_elems = tile;
    built->map_smem = static_cast<int>(t0b::MapSharedBytes(operation, tile, element_bytes));
    *plan = built.release();
    g_created.fetch_add(1, std::memory_order_relaxed);
  });
}

void t0b_plan_destroy(t0b_plan* plan) {
  if (plan == nullptr) return;
  delete plan;
  g_destroyed.fetch_add(1, std::memory_order_relaxed);
}

const int64_t* t0b_plan_table(const t0b_plan* plan, size_t* word_count) {
  if (plan == nullptr) { if (word_count) *word_count = 0; return nullptr; }
  if (word_count) *word_count = plan->plan.table.size();
  return plan->plan.table.data();
}

uint64_t t0b_plan_scratch_elements(const t0b_plan* plan) { return plan ? plan->plan.scratch : 0; }

void t0b_plan_query(const t0b_plan* plan, t0b_plan_info* info) {
  if (plan == nullptr || info == nullptr) return;
  const auto& p = plan->plan;
  info->source_size = p.source_size;
  info->output_size = p.output_size;
  info->records = p.records;
  info->tiles = p.map_tiles;
  info->kernels_per_call = p.operation == 2   ? 2
                           : p.operation == 5 ? (p.grouped_units != 0 ? 1 : 0)
                                              : (p.has_map ? 1 : 0) + 2 * p.waves.size();
  info->full_coverage = p.full_coverage ? 1 : 0;
  info->bytes_moved = p.bytes_moved;
}

uint64_t t0b_plan_matrix_elements(const t0b_plan* plan) {
  return plan != nullptr && plan->plan.operation == 5 ? plan->plan.coefficient_rows : 0;
}

uint64_t t0b_plan_created_count(void) { return g_created.load(std::memory_order_relaxed); }
uint64_t t0b_plan_destroyed_count(void) { return g_destroyed.load(std::memory_order_relaxed); }

int t0b_copy(const t0b_plan* plan, int32_t dtype, const void* source, void* output, int64_t batches,
             const int64_t* device_table, void* stream, char* error, size_t error_size) {
  return Guard(error, error_size, [&] {
    RequirePlan(plan, T0B_OP_COPY, dtype, batches);
    const auto& p = plan->plan;
    const uint64_t b = static_cast<uint64_t>(batches);
    const uint64_t out_bytes = Bytes(b * p.output_size, p.element_bytes);
    const uint64_t src_bytes = Bytes(b * p.source_size, p.element_bytes);
    if (b != 0 && p.output_size != 0 && output == nullptr) throw t0b::InvalidArgument("output buffer is null");
    if (b != 0 && p.source_size != 0 && source == nullptr) throw t0b::InvalidArgument("source buffer is null");
    if (device_table == nullptr) throw t0b::InvalidArgument("device descriptor table is null");
    RequireTableAligned(device_table);
    RequireAligned(source, p.element_bytes, "source");
    RequireAligned(output, p.element_bytes, "output");
    Disjoint(source, src_bytes, output, out_bytes);
    Disjoint(device_table, p.table.size() * sizeof(int64_t), output, out_bytes);
    if (b == 0 || p.output_size == 0) return;
    auto s = static_cast<cudaStream_t>(stream);
    if (!p.full_coverage) t0b::Check(cudaMemsetAsync(output, 0, out_bytes, s), "memset");
    if (p.has_map) {
      RunMap(plan, t0b::kOpCopy, dtype, T0B_S32, T0B_S32, source, nullptr, output, batches, nullptr, 1,
             nullptr, 1, device_table, s);
    }
  });
}

int t0b_accumulation(const t0b_plan* plan, int32_t dtype, const void* source, void* output, int64_t batches,
                     const void* coefficients, int32_t coefficient_dtype, int64_t coefficient_count,
                     void* scratch, const int64_t* device_table, void* stream, char* error, size_t error_size) {
  return Guard(error, error_size, [&] {
    Sum(plan, T0B_OP_ACCUMULATION, dtype, source, output, batches, coefficients, coefficient_dtype,
        coefficient_count, scratch, device_table, static_cast<cudaStream_t>(stream));
  });
}

int t0b_reduction(const t0b_plan* plan, int32_t dtype, const void* source, void* output, int64_t batches,
                  const void* coefficients, int32_t coefficient_dtype, int64_t coefficient_count,
                  void* scratch, const int64_t* device_table, void* stream, char* error, size_t error_size) {
  return Guard(error, error_size, [&] {
    Sum(plan, T0B_OP_REDUCTION, dtype, source, output, batches, coefficients, coefficient_dtype,
        coefficient_count, scratch, device_table, static_cast<cudaStream_t>(stream));
  });
}

int t0b_update(const t0b_plan* plan, int32_t dtype, const void* source, const void* base, void* output,
               int64_t batches, const void* alpha, int32_t alpha_dtype, int64_t alpha_count,
               const void* beta, int32_t beta_dtype, int64_t beta_count, const int64_t* device_table,
               void* stream, char* error, size_t error_size) {
  return Guard(error, error_size, [&] {
    RequirePlan(plan, T0B_OP_UPDATE, dtype, batches);
    const auto& p = plan->plan;
    const uint64_t b = static_cast<uint64_t>(batches);
    const int eb = p.element_bytes;
    const uint64_t out_bytes = Bytes(b * p.output_size, eb);
    const uint64_t src_bytes = Bytes(b * p.source_size, eb);
    if (b != 0 && p.output_size != 0 && (output == nullptr || base == nullptr)) {
      throw t0b::InvalidArgument("base or output buffer is null");
    }
    if (b != 0 && p.source_size != 0 && source == nullptr) throw t0b::InvalidArgument("source buffer is null");
    if (device_table == nullptr) throw t0b::InvalidArgument("device descriptor table is null");
    RequireTableAligned(device_table);
    RequireAligned(source, eb, "source");
    RequireAligned(base, eb, "base");
    RequireAligned(output, eb, "output");
    if (alpha == nullptr || beta == nullptr) throw t0b::InvalidArgument("update coefficient buffer is null");
    const int ab = CoefficientBytes(alpha_dtype, dtype);
    const int bb = CoefficientBytes(beta_dtype, dtype);
    RequireAligned(alpha, ab, "alpha");
    RequireAligned(beta, bb, "beta");
    const uint64_t a_count = CoefficientCount(alpha_count, batches);
    const uint64_t b_count = CoefficientCount(beta_count, batches);
    if (base != output) Disjoint(base, out_bytes, output, out_bytes);
    // A source aliasing the result is the reference's in-place form only
    // (update_impl.h:155-167): identical storage and per-element addresses.
    if (src_bytes != 0 && out_bytes != 0 && source == output) {
      throw t0b::InvalidArgument("unsupported source/result alias: requires identical source/base/result storage");
    }
    Disjoint(source, src_bytes, output, out_bytes);
    Disjoint(alpha, Bytes(a_count, ab), output, out_bytes);
    Disjoint(beta, Bytes(b_count, bb), output, out_bytes);
    Disjoint(device_table, p.table.size() * sizeof(int64_t), output, out_bytes);
    if (b == 0 || p.output_size == 0) return;
    auto s = static_cast<cudaStream_t>(stream);
    if (base != output && !p.full_coverage) {
      t0b::Check(cudaMemcpyAsync(output, base, out_bytes, cudaMemcpyDeviceToDevice, s), "base copy");
    }
    if (p.has_map) {
      RunMap(plan, t0b::kOpUpdate, dtype, alpha_dtype, beta_dtype, source, base, output, batches, alpha,
             static_cast<int64_t>(a_count), beta, static_cast<int64_t>(b_count), device_table, s);
    }
  });
}

int t0b_dot(const t0b_plan* plan, int32_t dtype, const void* left, const void* right, void* output,
            int64_t batches, int32_t conjugate_left, void* scratch, const int64_t* device_table, void* stream,
            char* error, size_t error_size) {
  return Guard(error, error_size, [&] {
    RequirePlan(plan, 2, dtype, batches);
    if (conjugate_left != 0 && conjugate_left != 1) throw t0b::InvalidArgument("dot conjugate_left must be zero or one");
    const auto& p = plan->plan;
    const int eb = p.element_bytes;
    const uint64_t b = static_cast<uint64_t>(batches);
    const uint64_t out_bytes = Bytes(b, eb);
    const uint64_t left_bytes = Bytes(b * p.source_size, eb);
    const uint64_t right_bytes = Bytes(b * p.output_size, eb);
    const uint64_t scratch_bytes = Bytes(b * p.scratch, eb);
    if (b == 0) return;
    if (output == nullptr || scratch == nullptr) throw t0b::InvalidArgument("dot output or scratch buffer is null");
    if ((p.source_size != 0 && left == nullptr) || (p.output_size != 0 && right == nullptr)) {
      throw t0b::InvalidArgument("dot input buffer is null");
    }
    if (device_table == nullptr) throw t0b::InvalidArgument("device descriptor table is null");
    RequireTableAligned(device_table);
    for (const void* buffer : {left, right, static_cast<const void*>(output)}) RequireAligned(buffer, eb, "dot");
    // Single-precision partial sums are kept in double precision.
    RequireAligned(scratch, 16, "dot scratch");
    const size_t table_bytes = p.table.size() * sizeof(int64_t);
    for (const auto& target : {std::pair<const void*, uint64_t>{output, out_bytes}, {scratch, scratch_bytes}}) {
      Disjoint(left, left_bytes, target.first, target.second);
      Disjoint(right, right_bytes, target.first, target.second);
      Disjoint(device_table, table_bytes, target.first, target.second);
    }
    Disjoint(output, out_bytes, scratch, scratch_bytes);
    const auto& h = Header(plan);
    t0b::DotArgs args{};
    args.recs = reinterpret_cast<const t0b::DotRecord*>(device_table + h.dot_offset);
    args.nrec = h.dot_records;
    args.units = h.dot_units;
    args.batches = batches;
    args.left = left;
    args.right = right;
    args.out = output;
    args.partials = scratch;
    args.left_size = static_cast<int64_t>(p.source_size);
    args.right_size = static_cast<int64_t>(p.output_size);
    args.conjugate_left = conjugate_left;
    t0b::LaunchDot(dtype, args, static_cast<cudaStream_t>(stream));
  });
}

int t0b_grouped_transform(const t0b_plan* plan, int32_t dtype, const void* source, void* output,
                          int64_t batches, const void* matrices, int32_t matrix_dtype,
                          const int64_t* device_table, void* stream, char* error, size_t error_size) {
  return Guard(error, error_size, [&] {
    RequirePlan(plan, 5, dtype, batches);
    const auto& p = plan->plan;
    const int eb = p.element_bytes;
    const uint64_t b = static_cast<uint64_t>(batches);
    const uint64_t out_bytes = Bytes(b * p.output_size, eb);
    const uint64_t src_bytes = Bytes(b * p.source_size, eb);
    if (matrix_dtype == T0B_S32) throw t0b::InvalidArgument("grouped matrices must be floating point");
    const int mb = CoefficientBytes(matrix_dtype, dtype);
    const uint64_t matrix_bytes = Bytes(p.coefficient_rows, mb);
    if (b == 0 || p.output_size == 0) return;
    if (output == nullptr) throw t0b::InvalidArgument("output buffer is null");
    if (p.source_size != 0 && source == nullptr) throw t0b::InvalidArgument("source buffer is null");
    if (p.coefficient_rows != 0 && matrices == nullptr) throw t0b::InvalidArgument("grouped matrix buffer is null");
    if (device_table == nullptr) throw t0b::InvalidArgument("device descriptor table is null");
    RequireTableAligned(device_table);
    RequireAligned(source, eb, "source");
    RequireAligned(output, eb, "output");
    RequireAligned(matrices, mb, "grouped matrix");
    Disjoint(source, src_bytes, output, out_bytes);
    Disjoint(matrices, matrix_bytes, output, out_bytes);
    Disjoint(device_table, p.table.size() * sizeof(int64_t), output, out_bytes);
    const auto launch_stream = static_cast<cudaStream_t>(stream);
    if (!p.full_coverage) t0b::Check(cudaMemsetAsync(output, 0, out_bytes, launch_stream), "memset");
    const auto& h = Header(plan);
    t0b::GroupedArgs args{};
    args.groups = reinterpret_cast<const t0b::GroupedGroup*>(device_table + h.grouped_offset);
    args.operands = reinterpret_cast<const t0b::GroupedOperand*>(device_table + h.operand_offset);
    args.ngroups = h.grouped;
    args.units = h.grouped_units;
    args.batches = batches;
    args.src = source;
    args.out = output;
    args.matrices = matrices;
    args.src_size = static_cast<int64_t>(p.source_size);
    args.out_size = static_cast<int64_t>(p.output_size);
    t0b::LaunchGrouped(dtype, matrix_dtype, args, static_cast<int64_t>(p.grouped_stage) * eb, launch_stream);
  });
}

int t0b_axpby(int32_t dtype, int64_t n, double alpha_real, double alpha_imag, const void* x,
              double beta_real, double beta_imag, const void* y, void* output, void* stream,
              char* error, size_t error_size) {
  return Guard(error, error_size, [&] {
    const int eb = ElementBytes(dtype);
    if (n < 0) throw t0b::InvalidArgument("element count must be nonnegative");
    if (n != 0 && (x == nullptr || y == nullptr || output == nullptr)) throw t0b::InvalidArgument("buffer is null");
    const uint64_t bytes = Bytes(static_cast<uint64_t>(n), eb);
    if (x != output) Disjoint(x, bytes, output, bytes);
    if (y != output) Disjoint(y, bytes, output, bytes);
    t0b::LaunchAxpby(dtype, n, alpha_real, alpha_imag, x, beta_real, beta_imag, y, output,
                     static_cast<cudaStream_t>(stream));
  });
}

size_t t0b_gemm_table_words(int64_t sectors) {
  return sectors < 0 ? 0 : static_cast<size_t>(sectors) * t0b::kGemmRow;
}

int t0b_gemm_table_build(int64_t sectors, const int64_t* spec, int64_t* table, char* error, size_t error_size) {
  return Guard(error, error_size, [&] {
    if (sectors < 0) throw t0b::InvalidArgument("sector count must be nonnegative");
    if (sectors != 0 && (spec == nullptr || table == nullptr)) throw t0b::InvalidArgument("GEMM table is null");
    t0b::BuildGemmTable(sectors, spec, table);
  });
}

int t0b_sector_gemm(int32_t dtype, int64_t sectors, const int64_t* host_table, const int64_t* device_table,
                    const void* left, int64_t left_size, const void* right, int64_t right_size, void* output,
                    int64_t output_size, void* stream, char* error, size_t error_size) {
  return Guard(error, error_size, [&] {
    t0b::SectorGemm(dtype, sectors, host_table, device_table, left, left_size, right, right_size, output,
                    output_size, static_cast<cudaStream_t>(stream));
  });
}

uint64_t t0b_kernel_launches(void) { return t0b::g_kernel_launches.load(std::memory_order_relaxed); }

}  // extern "C"
