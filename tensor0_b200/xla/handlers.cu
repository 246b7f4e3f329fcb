// XLA FFI handlers with the symbol table of the reference's CUDA companion
// library (crates/tensor0-py/src/stride.rs:284-330), forwarding to the engine's
// C ABI (include/tensor0_b200.h).  A JAX process loads this library where it
// loads the companion today and registers the same targets
// (_ffi/_registration.py:57-242); the public API above is unchanged.
//
// Bindings follow the reference's handlers attribute for attribute and operand
// for operand (copy.cu:154-162, update.cu:198-212, accumulation.cu:191-206,
// reduction.cu:199-215, dot.cu:123-160).  Two things differ inside:
//   - the descriptor operand carries this engine's packed table for the
//     handler's element size (t0b_plan_table), which the lowering computes in
//     place of the reference's owner/fiber words;
//   - the scratch result is sized by t0b_plan_scratch_elements.
// Coefficients arrive as one device buffer per coefficient record (scalar,
// [1] or [batch]); the handler gathers them into a table that lives in this
// library (no allocation, no synchronisation) with kernels that receive the
// buffer addresses as parameters.  Calls that overlap on the GPU share that
// table, as XLA's one stream per device never does.
#include "../../include/tensor0_b200.h"
#include "../../include/tensor0_b200_xla.h"

#include "xla/ffi/api/ffi.h"

#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstdio>
#include <functional>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

namespace ffi = xla::ffi;

namespace {

constexpr size_t kCoefficientTableBytes = size_t{32} << 20;   // 32 MiB per device
constexpr int kMaxDevices = 64;
__device__ __align__(256) unsigned char g_coefficient_table[kCoefficientTableBytes];

ffi::Error Failure(int status, const char* message) {
  return status == 1 ? ffi::Error::InvalidArgument(message) : ffi::Error::Internal(message);
}

int StorageDtype(ffi::DataType type) {
  switch (type) {
    case ffi::DataType::F32: return T0B_F32;
    case ffi::DataType::F64: return T0B_F64;
    case ffi::DataType::C64: return T0B_C64;
    case ffi::DataType::C128: return T0B_C128;
    default: return 0;
  }
}

int ElementBytes(int dtype) { return dtype == T0B_F32 ? 4 : dtype == T0B_C128 ? 16 : 8; }

// The instantiated state of one call site: the layout words and, per element
// size, the engine plan built on first use.
struct Prepared {
  int32_t operation = 0;
  std::vector<int64_t> words;
  std::vector<int64_t> records;
  uint32_t flags = 0;
  int64_t conjugate_left = 0;
  std::mutex mutex;
  t0b_plan* plans[3] = {nullptr, nullptr, nullptr};   // 4, 8 and 16 bytes

  ~Prepared() {
    for (t0b_plan* plan : plans) t0b_plan_destroy(plan);
  }

  // Build (once) the plan for an element size; status and message as the C ABI.
  int Plan(int element_bytes, t0b_plan** out, char* error, size_t size) {
    const int index = element_bytes == 4 ? 0 : element_bytes == 8 ? 1 : 2;
    std::lock_guard<std::mutex> lock(mutex);
    if (plans[index] == nullptr) {
      const int status = t0b_plan_create(operation, words.data(), words.size(), records.data(), records.size(),
                                         element_bytes, flags, &plans[index], error, size);
      if (status != 0) return status;
    }
    *out = plans[index];
    return 0;
  }
};

std::atomic<uint64_t> g_created[5];
std::atomic<uint64_t> g_destroyed[5];

// One state type per operation: XLA tells states apart by the type id that the
// registration (PreparedTypeId) fills in.
template <int Operation>
struct Counted : Prepared {
  Counted() { g_created[Operation].fetch_add(1, std::memory_order_relaxed); }
  ~Counted() { g_destroyed[Operation].fetch_add(1, std::memory_order_relaxed); }
  static inline ffi::TypeId id = {};
};

using CopyState = Counted<T0B_OP_COPY>;
using UpdateState = Counted<T0B_OP_UPDATE>;
using DotState = Counted<T0B_OP_DOT>;
using AccumulationState = Counted<T0B_OP_ACCUMULATION>;
using ReductionState = Counted<T0B_OP_REDUCTION>;

const ffi::TypeInfo kCopyTypeInfo = ffi::MakeTypeInfo<CopyState>();
const ffi::TypeInfo kUpdateTypeInfo = ffi::MakeTypeInfo<UpdateState>();
const ffi::TypeInfo kDotTypeInfo = ffi::MakeTypeInfo<DotState>();
const ffi::TypeInfo kAccumulationTypeInfo = ffi::MakeTypeInfo<AccumulationState>();
const ffi::TypeInfo kReductionTypeInfo = ffi::MakeTypeInfo<ReductionState>();

// Validate the words once at instantiation with a plan for 8-byte elements,
// before any prepared state exists: a rejected call site creates none, as in
// the reference (copy.cu:130-152).
template <typename S>
ffi::ErrorOr<std::unique_ptr<S>> Instantiate(int32_t operation, ffi::Span<const int64_t> layout,
                                              ffi::Span<const int64_t> records, uint32_t flags,
                                              int64_t conjugate_left) {
  std::vector<int64_t> words(layout.begin(), layout.end());
  std::vector<int64_t> selected(records.begin(), records.end());
  char error[512] = {0};
  t0b_plan* plan = nullptr;
  const int status = t0b_plan_create(operation, words.data(), words.size(), selected.data(), selected.size(), 8,
                                     flags, &plan, error, sizeof error);
  if (status != 0) return ffi::Unexpected(Failure(status, error));
  std::unique_ptr<S> state;
  try {
    state = std::make_unique<S>();
  } catch (...) {
    t0b_plan_destroy(plan);
    throw;
  }
  state->operation = operation;
  state->words = std::move(words);
  state->records = std::move(selected);
  state->flags = flags;
  state->conjugate_left = conjugate_left;
  state->plans[1] = plan;   // the 8-byte plan
  return std::move(state);
}

ffi::ErrorOr<std::unique_ptr<CopyState>> InstantiateCopy(ffi::Span<const int64_t> layout) {
  return Instantiate<CopyState>(T0B_OP_COPY, layout, {}, 0, 0);
}
ffi::ErrorOr<std::unique_ptr<UpdateState>> InstantiateUpdate(ffi::Span<const int64_t> layout) {
  return Instantiate<UpdateState>(T0B_OP_UPDATE, layout, {}, 0, 0);
}
ffi::ErrorOr<std::unique_ptr<DotState>> InstantiateDot(ffi::Span<const int64_t> layout, int64_t conjugate_left) {
  if (conjugate_left != 0 && conjugate_left != 1) {
    return ffi::Unexpected(ffi::Error::InvalidArgument("CUDA dot conjugate_left must be zero or one"));
  }
  return Instantiate<DotState>(T0B_OP_DOT, layout, {}, 0, conjugate_left);
}
ffi::ErrorOr<std::unique_ptr<AccumulationState>> InstantiateAccumulation(ffi::Span<const int64_t> layout,
                                                                         ffi::Span<const int64_t> records) {
  return Instantiate<AccumulationState>(T0B_OP_ACCUMULATION, layout, records, 0, 0);
}
ffi::ErrorOr<std::unique_ptr<ReductionState>> InstantiateReduction(ffi::Span<const int64_t> layout,
                                                                   ffi::Span<const int64_t> records) {
  return Instantiate<ReductionState>(T0B_OP_REDUCTION, layout, records, 0, 0);
}

// ---------------------------------------------------------------------------
// Coefficient gathering.

struct ScratchAddress {
  CUcontext context = nullptr;
  void* address = nullptr;
};
ScratchAddress g_table[kMaxDevices];
std::mutex g_table_mutex;

CUresult CurrentContext(CUcontext* context) {
  using Function = CUresult (*)(CUcontext*);
  static Function function = [] {
    void* pointer = nullptr;
    cudaDriverEntryPointQueryResult found{};
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &pointer, cudaEnableDefault, &found) != cudaSuccess ||
        found != cudaDriverEntryPointSuccess) {
      return static_cast<Function>(nullptr);
    }
    return reinterpret_cast<Function>(pointer);
  }();
  return function == nullptr ? CUDA_ERROR_NOT_FOUND : function(context);
}

// The table's device address for the current device and context.
void* TableAddress() {
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices) {
    throw std::runtime_error("cannot identify the current CUDA device");
  }
  CUcontext context = nullptr;
  if (CurrentContext(&context) != CUDA_SUCCESS) throw std::runtime_error("cannot identify the current CUDA context");
  std::lock_guard<std::mutex> lock(g_table_mutex);
  ScratchAddress& cached = g_table[device];
  if (cached.address == nullptr || context == nullptr || cached.context != context) {
    void* address = nullptr;
    if (cudaGetSymbolAddress(&address, g_coefficient_table) != cudaSuccess || address == nullptr) {
      throw std::runtime_error("cudaGetSymbolAddress of the coefficient table failed");
    }
    if (context == nullptr && (CurrentContext(&context) != CUDA_SUCCESS || context == nullptr)) {
      throw std::runtime_error("cannot identify the current CUDA context");
    }
    cached = {context, address};
  }
  return cached.address;
}

constexpr int kGatherChunk = 256;
struct GatherChunk {
  const void* source[kGatherChunk];
  int64_t count[kGatherChunk];     // 1 (shared by every batch) or the batch count
  int32_t dtype[kGatherChunk];
  int32_t size;
  int32_t first_row;
};

template <typename Real> struct Pair { Real x, y; };

template <typename Real, bool kComplexTable>
__device__ void ReadAs(const void* source, int32_t dtype, int64_t index, Real* x, Real* y) {
  *y = Real(0);
  switch (dtype) {
    case T0B_S32: *x = static_cast<Real>(static_cast<const int32_t*>(source)[index]); break;
    case T0B_F32: *x = static_cast<Real>(static_cast<const float*>(source)[index]); break;
    case T0B_F64: *x = static_cast<Real>(static_cast<const double*>(source)[index]); break;
    case T0B_C64: {
      const float2 v = static_cast<const float2*>(source)[index];
      *x = static_cast<Real>(v.x); *y = static_cast<Real>(v.y);
      break;
    }
    default: {
      const double2 v = static_cast<const double2*>(source)[index];
      *x = static_cast<Real>(v.x); *y = static_cast<Real>(v.y);
      break;
    }
  }
}

// table[(first_row + i) * columns + b] = coefficient i for batch b.
template <typename Real, bool kComplexTable>
__global__ void GatherCoefficients(GatherChunk chunk, void* table, int64_t columns) {
  const int64_t total = static_cast<int64_t>(chunk.size) * columns;
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int i = static_cast<int>(t / columns);
    const int64_t b = t - static_cast<int64_t>(i) * columns;
    Real x, y;
    ReadAs<Real, kComplexTable>(chunk.source[i], chunk.dtype[i], chunk.count[i] == 1 ? 0 : b, &x, &y);
    const int64_t at = (chunk.first_row + i) * columns + b;
    if constexpr (kComplexTable) {
      static_cast<Pair<Real>*>(table)[at] = Pair<Real>{x, y};
    } else {
      static_cast<Real*>(table)[at] = x;
    }
  }
}

int CoefficientDtype(ffi::DataType type) {
  switch (type) {
    case ffi::DataType::S32: return T0B_S32;
    case ffi::DataType::F32: return T0B_F32;
    case ffi::DataType::F64: return T0B_F64;
    case ffi::DataType::C64: return T0B_C64;
    case ffi::DataType::C128: return T0B_C128;
    default: return 0;
  }
}

// Gather the coefficient operands into the table; returns the table, its
// element dtype and columns (1 or batches) for the engine.
struct Gathered {
  const void* table = nullptr;
  int32_t dtype = T0B_S32;
  int64_t columns = 1;
};

Gathered GatherAll(ffi::RemainingArgs coefficients, int storage, int64_t batches, size_t expected,
                   const char* what, cudaStream_t stream) {
  if (coefficients.size() != expected) {
    throw std::invalid_argument(std::string("CUDA ") + what + " coefficient record count does not match operands");
  }
  Gathered out;
  if (expected == 0) return out;
  const bool single = storage == T0B_F32 || storage == T0B_C64;
  const bool complex_storage = storage == T0B_C64 || storage == T0B_C128;
  bool any_complex = false;
  std::vector<GatherChunk> chunks((expected + kGatherChunk - 1) / kGatherChunk);
  for (size_t i = 0; i < expected; ++i) {
    auto buffer = coefficients.get<ffi::AnyBuffer>(i);
    if (!buffer) throw std::invalid_argument(std::string("CUDA ") + what + " coefficient must be a buffer");
    const auto dims = buffer->dimensions();
    int64_t count = 1;
    if (dims.size() == 1) {
      if (dims[0] != 1 && dims[0] != batches) {
        throw std::invalid_argument(std::string("CUDA ") + what +
                                    " coefficients must be scalar, length-one, or match batch count");
      }
      count = dims[0];
    } else if (dims.size() != 0) {
      throw std::invalid_argument(std::string("CUDA ") + what +
                                  " coefficients must be scalar, length-one, or match batch count");
    }
    const int dtype = CoefficientDtype(buffer->element_type());
    const bool complex_coefficient = dtype == T0B_C64 || dtype == T0B_C128;
    const bool allowed = dtype == T0B_S32 || dtype == (single ? T0B_F32 : T0B_F64) ||
                         (complex_storage && dtype == (single ? T0B_C64 : T0B_C128));
    if (!allowed) {
      throw std::invalid_argument("unsupported CUDA coefficient dtype; expected S32 or matching real/complex precision");
    }
    any_complex = any_complex || complex_coefficient;
    if (count != 1) out.columns = batches;
    GatherChunk& chunk = chunks[i / kGatherChunk];
    const int k = static_cast<int>(i % kGatherChunk);
    chunk.source[k] = buffer->untyped_data();
    chunk.count[k] = count;
    chunk.dtype[k] = dtype;
    chunk.size = k + 1;
    chunk.first_row = static_cast<int32_t>(i - k);
  }
  const size_t real_bytes = single ? 4 : 8;
  const size_t element = any_complex ? 2 * real_bytes : real_bytes;
  if (static_cast<double>(expected) * static_cast<double>(out.columns) * element > kCoefficientTableBytes) {
    throw std::invalid_argument(std::string("CUDA ") + what + " has more coefficients than the handler's 32 MiB table holds");
  }
  void* table = TableAddress();
  for (const GatherChunk& chunk : chunks) {
    const int64_t total = static_cast<int64_t>(chunk.size) * out.columns;
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>((total + 255) / 256, 1024));
    if (single) {
      if (any_complex) GatherCoefficients<float, true><<<grid, 256, 0, stream>>>(chunk, table, out.columns);
      else GatherCoefficients<float, false><<<grid, 256, 0, stream>>>(chunk, table, out.columns);
    } else {
      if (any_complex) GatherCoefficients<double, true><<<grid, 256, 0, stream>>>(chunk, table, out.columns);
      else GatherCoefficients<double, false><<<grid, 256, 0, stream>>>(chunk, table, out.columns);
    }
    const cudaError_t status = cudaGetLastError();
    if (status != cudaSuccess) throw std::runtime_error(std::string("coefficient gather launch: ") + cudaGetErrorString(status));
  }
  out.table = table;
  out.dtype = any_complex ? (single ? T0B_C64 : T0B_C128) : (single ? T0B_F32 : T0B_F64);
  return out;
}

// ---------------------------------------------------------------------------
// Execute handlers.

ffi::Error Contain(const std::function<void()>& body) {
  try {
    body();
    return ffi::Error::Success();
  } catch (const std::invalid_argument& e) {
    return ffi::Error::InvalidArgument(e.what());
  } catch (const std::exception& e) {
    return ffi::Error::Internal(e.what());
  }
}

struct Engine {
  t0b_plan* plan = nullptr;
  size_t words = 0;
};

Engine PlanFor(Prepared* state, int dtype, ffi::BufferR1<ffi::S64> descriptor, const char* what) {
  char error[512] = {0};
  Engine engine;
  const int status = state->Plan(ElementBytes(dtype), &engine.plan, error, sizeof error);
  if (status == 1) throw std::invalid_argument(error);
  if (status != 0) throw std::runtime_error(error);
  t0b_plan_table(engine.plan, &engine.words);
  if (descriptor.dimensions()[0] < 0 || static_cast<size_t>(descriptor.dimensions()[0]) != engine.words) {
    throw std::invalid_argument(std::string("CUDA ") + what + " descriptor operand shape does not match layout");
  }
  return engine;
}

void Check(int status, const char* error) {
  if (status == 1) throw std::invalid_argument(error);
  if (status != 0) throw std::runtime_error(error);
}

template <ffi::DataType Dtype>
ffi::Error Copy(CopyState* state, ffi::AnyBuffer source, ffi::BufferR1<ffi::S64> descriptor,
                ffi::ResultBufferR2<Dtype> result, cudaStream_t stream) {
  return Contain([&] {
    if (source.element_type() != Dtype) {
      throw std::invalid_argument("CUDA copy supports only same-dtype F32/F64/C64/C128; conversion is unsupported");
    }
    if (source.dimensions().size() != 2) throw std::invalid_argument("CUDA copy storage must be rank-two");
    const int dtype = StorageDtype(Dtype);
    const Engine engine = PlanFor(state, dtype, descriptor, "copy");
    t0b_plan_info info{};
    t0b_plan_query(engine.plan, &info);
    if (source.dimensions()[0] != result->dimensions()[0] ||
        static_cast<uint64_t>(source.dimensions()[1]) != info.source_size ||
        static_cast<uint64_t>(result->dimensions()[1]) != info.output_size) {
      throw std::invalid_argument("CUDA copy buffer dimensions do not match layout");
    }
    char error[512] = {0};
    Check(t0b_copy(engine.plan, dtype, source.untyped_data(), result->untyped_data(), result->dimensions()[0],
                   descriptor.typed_data(), stream, error, sizeof error), error);
  });
}

template <ffi::DataType Dtype>
ffi::Error Update(UpdateState* state, ffi::AnyBuffer source, ffi::BufferR2<Dtype> base, ffi::AnyBuffer alpha,
                  ffi::AnyBuffer beta, ffi::BufferR1<ffi::S64> descriptor, ffi::ResultBufferR2<Dtype> result,
                  cudaStream_t stream) {
  return Contain([&] {
    if (source.element_type() != Dtype) {
      throw std::invalid_argument("CUDA update supports only same-dtype F32/F64/C64/C128 storage");
    }
    if (source.dimensions().size() != 2) throw std::invalid_argument("CUDA update source storage must be rank-two");
    const int dtype = StorageDtype(Dtype);
    const Engine engine = PlanFor(state, dtype, descriptor, "update");
    t0b_plan_info info{};
    t0b_plan_query(engine.plan, &info);
    const int64_t batches = result->dimensions()[0];
    if (source.dimensions()[0] != batches || base.dimensions()[0] != batches ||
        static_cast<uint64_t>(source.dimensions()[1]) != info.source_size ||
        static_cast<uint64_t>(result->dimensions()[1]) != info.output_size ||
        base.dimensions()[1] != result->dimensions()[1]) {
      throw std::invalid_argument("CUDA update buffer dimensions do not match layout");
    }
    auto count = [&](const ffi::AnyBuffer& b) -> int64_t {
      const auto dims = b.dimensions();
      if (dims.size() == 0) return 1;
      if (dims.size() == 1 && (dims[0] == 1 || dims[0] == batches)) return dims[0];
      throw std::invalid_argument("CUDA update coefficients must be scalar, length-one, or match batch count");
    };
    char error[512] = {0};
    Check(t0b_update(engine.plan, dtype, source.untyped_data(), base.untyped_data(), result->untyped_data(), batches,
                     alpha.untyped_data(), CoefficientDtype(alpha.element_type()), count(alpha), beta.untyped_data(),
                     CoefficientDtype(beta.element_type()), count(beta), descriptor.typed_data(), stream, error,
                     sizeof error), error);
  });
}

template <ffi::DataType Dtype, int Operation>
ffi::Error Sum(Counted<Operation>* state, ffi::AnyBuffer source, ffi::BufferR1<ffi::S64> descriptor,
               ffi::RemainingArgs coefficients, ffi::ResultBufferR2<Dtype> result,
               ffi::ResultBufferR2<Dtype> scratch, cudaStream_t stream) {
  const char* what = Operation == T0B_OP_ACCUMULATION ? "accumulation" : "reduction";
  return Contain([&] {
    if (source.element_type() != Dtype) {
      throw std::invalid_argument(std::string("CUDA ") + what + " supports only same-dtype F32/F64/C64/C128 storage");
    }
    if (source.dimensions().size() != 2) throw std::invalid_argument(std::string("CUDA ") + what + " source must be rank-two");
    const int dtype = StorageDtype(Dtype);
    const Engine engine = PlanFor(state, dtype, descriptor, what);
    t0b_plan_info info{};
    t0b_plan_query(engine.plan, &info);
    const int64_t batches = result->dimensions()[0];
    if (source.dimensions()[0] != batches || static_cast<uint64_t>(source.dimensions()[1]) != info.source_size ||
        static_cast<uint64_t>(result->dimensions()[1]) != info.output_size) {
      throw std::invalid_argument(std::string("CUDA ") + what + " buffer dimensions do not match layout");
    }
    if (scratch->dimensions()[0] != batches ||
        static_cast<uint64_t>(scratch->dimensions()[1]) != t0b_plan_scratch_elements(engine.plan)) {
      throw std::invalid_argument(std::string("CUDA ") + what + " scratch capacity does not match layout");
    }
    const Gathered table = GatherAll(coefficients, dtype, batches, state->records.size(), what, stream);
    char error[512] = {0};
    auto function = Operation == T0B_OP_ACCUMULATION ? t0b_accumulation : t0b_reduction;
    Check(function(engine.plan, dtype, source.untyped_data(), result->untyped_data(), batches, table.table,
                   table.dtype, table.columns, scratch->untyped_data(), descriptor.typed_data(), stream, error,
                   sizeof error), error);
  });
}

template <ffi::DataType Dtype>
ffi::Error Dot(DotState* state, ffi::AnyBuffer left, ffi::AnyBuffer right, ffi::BufferR1<ffi::S64> descriptor,
               ffi::ResultBufferR1<Dtype> result, ffi::ResultBufferR2<Dtype> scratch, cudaStream_t stream) {
  return Contain([&] {
    if (left.element_type() != Dtype || right.element_type() != Dtype) {
      throw std::invalid_argument("CUDA dot supports only same-dtype F32/F64/C64/C128 inputs and result");
    }
    if (left.dimensions().size() != 2 || right.dimensions().size() != 2) {
      throw std::invalid_argument("CUDA dot inputs must be rank-two");
    }
    const int dtype = StorageDtype(Dtype);
    const Engine engine = PlanFor(state, dtype, descriptor, "dot");
    t0b_plan_info info{};
    t0b_plan_query(engine.plan, &info);
    const int64_t batches = result->dimensions()[0];
    if (left.dimensions()[0] != batches || right.dimensions()[0] != batches ||
        static_cast<uint64_t>(left.dimensions()[1]) != info.source_size ||
        static_cast<uint64_t>(right.dimensions()[1]) != info.output_size || scratch->dimensions()[0] != batches) {
      throw std::invalid_argument("CUDA dot buffer dimensions do not match layout");
    }
    if (static_cast<uint64_t>(scratch->dimensions()[1]) != t0b_plan_scratch_elements(engine.plan)) {
      throw std::invalid_argument("CUDA dot scratch capacity does not match layout");
    }
    char error[512] = {0};
    Check(t0b_dot(engine.plan, dtype, left.untyped_data(), right.untyped_data(), result->untyped_data(), batches,
                  static_cast<int32_t>(state->conjugate_left), scratch->untyped_data(), descriptor.typed_data(), stream,
                  error, sizeof error), error);
  });
}

}  // namespace

// ---------------------------------------------------------------------------
// The symbol table (stride.rs:284-330).

#define T0B_XLA_EXPORT extern "C" __attribute__((visibility("default")))

#define T0B_XLA_STATE(Name, Type, Info, Op)                                                               \
  T0B_XLA_EXPORT void* Tensor0StrideCuda##Name##PreparedTypeId() { return &Type::id; }                     \
  T0B_XLA_EXPORT const void* Tensor0StrideCuda##Name##PreparedTypeInfo() { return &Info; }                 \
  T0B_XLA_EXPORT uint64_t Tensor0StrideCuda##Name##PreparedCreatedCount() {                                \
    return g_created[Op].load(std::memory_order_relaxed);                                                 \
  }                                                                                                       \
  T0B_XLA_EXPORT uint64_t Tensor0StrideCuda##Name##PreparedDestroyedCount() {                              \
    return g_destroyed[Op].load(std::memory_order_relaxed);                                               \
  }

XLA_FFI_DEFINE_HANDLER_SYMBOL(T0bXlaCopyInstantiate, InstantiateCopy,
                              ffi::Ffi::BindInstantiate().Attr<ffi::Span<const int64_t>>("layout"));
XLA_FFI_DEFINE_HANDLER_SYMBOL(T0bXlaUpdateInstantiate, InstantiateUpdate,
                              ffi::Ffi::BindInstantiate().Attr<ffi::Span<const int64_t>>("layout"));
XLA_FFI_DEFINE_HANDLER_SYMBOL(T0bXlaDotInstantiate, InstantiateDot,
                              ffi::Ffi::BindInstantiate().Attr<ffi::Span<const int64_t>>("layout")
                                  .Attr<int64_t>("conjugate_left"));
XLA_FFI_DEFINE_HANDLER_SYMBOL(T0bXlaAccumulationInstantiate, InstantiateAccumulation,
                              ffi::Ffi::BindInstantiate().Attr<ffi::Span<const int64_t>>("layout")
                                  .Attr<ffi::Span<const int64_t>>("coefficient_records"));
XLA_FFI_DEFINE_HANDLER_SYMBOL(T0bXlaReductionInstantiate, InstantiateReduction,
                              ffi::Ffi::BindInstantiate().Attr<ffi::Span<const int64_t>>("layout")
                                  .Attr<ffi::Span<const int64_t>>("coefficient_records"));

T0B_XLA_EXPORT void* Tensor0StrideCudaCopyInstantiateV1Handler() { return reinterpret_cast<void*>(&T0bXlaCopyInstantiate); }
T0B_XLA_EXPORT void* Tensor0StrideCudaUpdateInstantiateV1Handler() { return reinterpret_cast<void*>(&T0bXlaUpdateInstantiate); }
T0B_XLA_EXPORT void* Tensor0StrideCudaDotInstantiateV1Handler() { return reinterpret_cast<void*>(&T0bXlaDotInstantiate); }
T0B_XLA_EXPORT void* Tensor0StrideCudaAccumulationInstantiateV1Handler() {
  return reinterpret_cast<void*>(&T0bXlaAccumulationInstantiate);
}
T0B_XLA_EXPORT void* Tensor0StrideCudaReductionInstantiateV1Handler() {
  return reinterpret_cast<void*>(&T0bXlaReductionInstantiate);
}

T0B_XLA_STATE(Copy, CopyState, kCopyTypeInfo, T0B_OP_COPY)
T0B_XLA_STATE(Update, UpdateState, kUpdateTypeInfo, T0B_OP_UPDATE)
T0B_XLA_STATE(Dot, DotState, kDotTypeInfo, T0B_OP_DOT)
T0B_XLA_STATE(Accumulation, AccumulationState, kAccumulationTypeInfo, T0B_OP_ACCUMULATION)
T0B_XLA_STATE(Reduction, ReductionState, kReductionTypeInfo, T0B_OP_REDUCTION)

#define T0B_XLA_DTYPE(Suffix, Dtype)                                                                          \
  XLA_FFI_DEFINE_HANDLER_SYMBOL(T0bXlaCopy##Suffix, Copy<ffi::Dtype>,                                       \
                                ffi::Ffi::BindExecute().Ctx<ffi::State<CopyState>>().Arg<ffi::AnyBuffer>()  \
                                    .Arg<ffi::BufferR1<ffi::S64>>().Ret<ffi::BufferR2<ffi::Dtype>>()         \
                                    .Ctx<ffi::PlatformStream<cudaStream_t>>());                             \
  XLA_FFI_DEFINE_HANDLER_SYMBOL(T0bXlaUpdate##Suffix, Update<ffi::Dtype>,                                   \
                                ffi::Ffi::BindExecute().Ctx<ffi::State<UpdateState>>().Arg<ffi::AnyBuffer>() \
                                    .Arg<ffi::BufferR2<ffi::Dtype>>().Arg<ffi::AnyBuffer>()                  \
                                    .Arg<ffi::AnyBuffer>().Arg<ffi::BufferR1<ffi::S64>>()                    \
                                    .Ret<ffi::BufferR2<ffi::Dtype>>().Ctx<ffi::PlatformStream<cudaStream_t>>()); \
  XLA_FFI_DEFINE_HANDLER_SYMBOL(T0bXlaAccumulation##Suffix, (Sum<ffi::Dtype, T0B_OP_ACCUMULATION>),          \
                                ffi::Ffi::BindExecute().Ctx<ffi::State<AccumulationState>>()                \
                                    .Arg<ffi::AnyBuffer>().Arg<ffi::BufferR1<ffi::S64>>().RemainingArgs()   \
                                    .Ret<ffi::BufferR2<ffi::Dtype>>().Ret<ffi::BufferR2<ffi::Dtype>>()       \
                                    .Ctx<ffi::PlatformStream<cudaStream_t>>());                             \
  XLA_FFI_DEFINE_HANDLER_SYMBOL(T0bXlaReduction##Suffix, (Sum<ffi::Dtype, T0B_OP_REDUCTION>),                \
                                ffi::Ffi::BindExecute().Ctx<ffi::State<ReductionState>>()                   \
                                    .Arg<ffi::AnyBuffer>().Arg<ffi::BufferR1<ffi::S64>>().RemainingArgs()   \
                                    .Ret<ffi::BufferR2<ffi::Dtype>>().Ret<ffi::BufferR2<ffi::Dtype>>()       \
                                    .Ctx<ffi::PlatformStream<cudaStream_t>>());                             \
  XLA_FFI_DEFINE_HANDLER_SYMBOL(T0bXlaDot##Suffix, Dot<ffi::Dtype>,                                         \
                                ffi::Ffi::BindExecute().Ctx<ffi::State<DotState>>().Arg<ffi::AnyBuffer>()   \
                                    .Arg<ffi::AnyBuffer>().Arg<ffi::BufferR1<ffi::S64>>()                    \
                                    .Ret<ffi::BufferR1<ffi::Dtype>>().Ret<ffi::BufferR2<ffi::Dtype>>()       \
                                    .Ctx<ffi::PlatformStream<cudaStream_t>>());                             \
  T0B_XLA_EXPORT void* Tensor0StrideCudaCopy##Suffix##V1Handler() { return reinterpret_cast<void*>(&T0bXlaCopy##Suffix); } \
  T0B_XLA_EXPORT void* Tensor0StrideCudaUpdate##Suffix##V1Handler() { return reinterpret_cast<void*>(&T0bXlaUpdate##Suffix); } \
  T0B_XLA_EXPORT void* Tensor0StrideCudaAccumulation##Suffix##V1Handler() {                                 \
    return reinterpret_cast<void*>(&T0bXlaAccumulation##Suffix);                                            \
  }                                                                                                         \
  T0B_XLA_EXPORT void* Tensor0StrideCudaReduction##Suffix##V1Handler() {                                    \
    return reinterpret_cast<void*>(&T0bXlaReduction##Suffix);                                               \
  }                                                                                                         \
  T0B_XLA_EXPORT void* Tensor0StrideCudaDot##Suffix##V1Handler() { return reinterpret_cast<void*>(&T0bXlaDot##Suffix); }

T0B_XLA_DTYPE(F32, F32)
T0B_XLA_DTYPE(F64, F64)
T0B_XLA_DTYPE(C64, C64)
T0B_XLA_DTYPE(C128, C128)
