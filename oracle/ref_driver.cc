// Test infrastructure only: a C driver around the reference's own native CPU
// stride executors, compiled from the reference sources where they lie (see
// oracle/Makefile).  Nothing in the product links or loads this file; tests,
// the smoke check and the CPU-baseline leg of bench.py use it as the checker.
//
// The reference's JAX CPU path reaches these executors through XLA FFI
// handlers (crates/tensor0-py/native/ffi/{copy.cc,update_impl.h,
// reduction_impl.h}).  JAX is not available here, so this driver binds the
// same handler templates directly with hand-built XLA_FFI_Buffer structs and
// an XLA_FFI_Api whose thread pool is a real std::thread pool (the pattern of
// tests/stride/native/cpp/thread_pool_test_support.h:9-40).  The one-shot
// calls run instantiate (descriptor decode, validation, sort/fuse preparation)
// and then execute; the t0ref_prepare / t0ref_execute_* pair keeps the
// instantiated state across executions, as one XLA executable does, so that
// timing covers execution only.

#define TENSOR0_STRIDE_TEST_NO_HANDLERS
#include "ffi/dot_impl.h"
#include "ffi/reduction_impl.h"
#include "ffi/update_impl.h"
#include "execute/copy.h"
#undef TENSOR0_STRIDE_TEST_NO_HANDLERS

#include <condition_variable>
#include <cstring>
#include <deque>
#include <functional>
#include <memory>
#include <mutex>
#include <optional>
#include <thread>
#include <vector>

namespace native = tensor0::stride;

extern "C" void Tensor0StrideSetWorkerLimit(uint64_t);

namespace {

// A fixed pool of workers behind XLA_FFI_ThreadPool_{NumThreads,Schedule}.
class WorkerPool {
 public:
  explicit WorkerPool(int64_t threads) : threads_(threads < 1 ? 1 : threads) {
    api_.XLA_FFI_ThreadPool_NumThreads = [](XLA_FFI_ThreadPool_NumThreads_Args* args) -> XLA_FFI_Error* {
      *args->num_threads = reinterpret_cast<WorkerPool*>(args->ctx)->threads_;
      return nullptr;
    };
    api_.XLA_FFI_ThreadPool_Schedule = [](XLA_FFI_ThreadPool_Schedule_Args* args) -> XLA_FFI_Error* {
      reinterpret_cast<WorkerPool*>(args->ctx)->Push(args->task, args->data);
      return nullptr;
    };
    for (int64_t i = 0; i < threads_; ++i) workers_.emplace_back([this] { Run(); });
  }
  ~WorkerPool() {
    {
      std::lock_guard lock(mutex_);
      stopping_ = true;
    }
    ready_.notify_all();
    for (auto& worker : workers_) worker.join();
  }

  ffi::ThreadPool Get() {
    return *ffi::CtxDecoding<ffi::ThreadPool>::Decode(
        &api_, reinterpret_cast<XLA_FFI_ExecutionContext*>(this), diagnostic_);
  }

 private:
  void Push(XLA_FFI_Task* task, void* data) {
    {
      std::lock_guard lock(mutex_);
      queue_.emplace_back(task, data);
    }
    ready_.notify_one();
  }
  void Run() {
    for (;;) {
      std::pair<XLA_FFI_Task*, void*> item;
      {
        std::unique_lock lock(mutex_);
        ready_.wait(lock, [&] { return stopping_ || !queue_.empty(); });
        if (queue_.empty()) return;
        item = queue_.front();
        queue_.pop_front();
      }
      item.first(item.second);
    }
  }

  XLA_FFI_Api api_{};
  ffi::DiagnosticEngine diagnostic_;
  int64_t threads_;
  std::mutex mutex_;
  std::condition_variable ready_;
  std::deque<std::pair<XLA_FFI_Task*, void*>> queue_;
  std::vector<std::thread> workers_;
  bool stopping_ = false;
};

WorkerPool& Pool(int64_t threads) {
  static std::mutex guard;
  static std::unique_ptr<WorkerPool> pool;
  static int64_t size = 0;
  std::lock_guard lock(guard);
  if (!pool || size != threads) {
    pool.reset();
    pool = std::make_unique<WorkerPool>(threads);
    size = threads;
  }
  return *pool;
}

int Wait(ffi::Future future, char* error, size_t error_size) {
  std::mutex mutex;
  std::condition_variable done;
  bool ready = false;
  std::optional<ffi::Error> result;
  future.OnReady([&](const std::optional<ffi::Error>& value) {
    std::lock_guard lock(mutex);
    if (value) result = *value;
    ready = true;
    done.notify_all();
  });
  std::unique_lock lock(mutex);
  done.wait(lock, [&] { return ready; });
  if (result && result->failure()) {
    const auto message = result->message();
    if (error && error_size) {
      std::snprintf(error, error_size, "%s", message.c_str());
    }
    return result->errc() == ffi::ErrorCode::kInvalidArgument ? 1 : 2;
  }
  return 0;
}

int Report(const ffi::Error& status, char* error, size_t error_size) {
  if (!status.failure()) return 0;
  if (error && error_size) std::snprintf(error, error_size, "%s", status.message().c_str());
  return status.errc() == ffi::ErrorCode::kInvalidArgument ? 1 : 2;
}

XLA_FFI_Buffer MakeBuffer(int dtype, const void* data, int64_t rank, int64_t* dims) {
  return XLA_FFI_Buffer{XLA_FFI_Buffer_STRUCT_SIZE, nullptr, static_cast<XLA_FFI_DataType>(dtype),
                        const_cast<void*>(data), rank, dims};
}

template <typename Function>
int DispatchStorage(int dtype, Function function) {
  switch (dtype) {
    case XLA_FFI_DataType_F32: return function(std::integral_constant<ffi::DataType, ffi::F32>{});
    case XLA_FFI_DataType_F64: return function(std::integral_constant<ffi::DataType, ffi::F64>{});
    case XLA_FFI_DataType_C64: return function(std::integral_constant<ffi::DataType, ffi::C64>{});
    case XLA_FFI_DataType_C128: return function(std::integral_constant<ffi::DataType, ffi::C128>{});
    default: return -1;
  }
}

// Coefficient operands: each is scalar (count 0 -> rank 0), length one, or per batch.
struct CoefficientArgs {
  std::vector<XLA_FFI_Buffer> buffers;
  std::vector<std::array<int64_t, 1>> dims;
  std::vector<XLA_FFI_ArgType> kinds;
  std::vector<void*> pointers;
  XLA_FFI_Args args{};

  CoefficientArgs(size_t count, const void* const* data, const int* dtypes, const int64_t* counts) {
    buffers.reserve(count);
    dims.resize(count);
    for (size_t i = 0; i < count; ++i) {
      dims[i][0] = counts[i];
      const int64_t rank = counts[i] < 0 ? 0 : 1;
      buffers.push_back(MakeBuffer(dtypes[i], data[i], rank, rank ? dims[i].data() : nullptr));
    }
    kinds.assign(count, XLA_FFI_ArgType_BUFFER);
    for (auto& buffer : buffers) pointers.push_back(&buffer);
    args = XLA_FFI_Args{XLA_FFI_Args_STRUCT_SIZE, nullptr, static_cast<int64_t>(count),
                        kinds.data(), pointers.data()};
  }
};

}  // namespace

extern "C" {

// Set the process-wide worker limit the reference's scheduler honours.
void t0ref_set_worker_limit(uint64_t limit) { Tensor0StrideSetWorkerLimit(limit); }

// The reference's own layout preparation bridge (descriptor.cc:294-351).
int t0ref_prepare_layout(int32_t operation, const int64_t* words, size_t word_count,
                         int64_t* output, size_t capacity, size_t* output_count,
                         char* error, size_t error_size) {
  struct Context { int64_t* output; size_t capacity; size_t* count; char* error; size_t error_size; int status; };
  Context context{output, capacity, output_count, error, error_size, 0};
  Tensor0StridePrepareLayout(operation, words, word_count, &context,
      [](void* raw, int32_t status, const int64_t* result, size_t n, const char* message, size_t message_size) {
        auto* ctx = static_cast<Context*>(raw);
        ctx->status = status;
        if (status == 0) {
          *ctx->count = n;
          if (n <= ctx->capacity) std::memcpy(ctx->output, result, n * sizeof(int64_t));
          else ctx->status = 3;
        } else if (ctx->error && ctx->error_size) {
          std::snprintf(ctx->error, ctx->error_size, "%.*s", static_cast<int>(message_size), message);
        }
      });
  return context.status;
}

// Copy: InstantiatePrepared (prepared.cc:37-45) + ExecuteCopy (execute/copy.h:119-134).
int t0ref_copy(int dtype, const int64_t* words, size_t word_count, const void* source,
               int64_t source_size, void* output, int64_t output_size, int64_t batches,
               int64_t threads, char* error, size_t error_size) {
  auto prepared = native::InstantiatePrepared({words, word_count});
  if (!prepared.has_value()) return Report(prepared.error(), error, error_size);
  const auto& state = **prepared;
  if (static_cast<uint64_t>(source_size) != state.source_size ||
      static_cast<uint64_t>(output_size) != state.output_size) {
    std::snprintf(error, error_size, "buffer dimensions do not match layout");
    return 1;
  }
  return DispatchStorage(dtype, [&](auto tag) {
    using Scalar = native::ScalarDtype<decltype(tag)::value>;
    using Value = native::scalar::Value<Scalar>;
    auto future = native::ExecuteCopy<Scalar, Scalar>(Pool(threads).Get(), state.records,
        static_cast<const Value*>(source), static_cast<Value*>(output),
        state.source_size, state.output_size, static_cast<uint64_t>(batches));
    return Wait(std::move(future), error, error_size);
  });
}

// Accumulation: InstantiateAccumulation (prepared.cc:69-81) + Accumulation
// (ffi/reduction_impl.h:162-172) with coefficient operands bound per record.
int t0ref_accumulation(int dtype, const int64_t* words, size_t word_count,
                       const int64_t* coefficient_records, size_t coefficient_count,
                       const void* const* coefficient_data, const int* coefficient_dtypes,
                       const int64_t* coefficient_counts, int64_t outputs_disjoint,
                       const void* source, int64_t source_size, void* output, int64_t output_size,
                       int64_t batches, int64_t threads, char* error, size_t error_size) {
  auto prepared = native::InstantiateAccumulation({words, word_count},
      {coefficient_records, coefficient_count}, outputs_disjoint);
  if (!prepared.has_value()) return Report(prepared.error(), error, error_size);
  CoefficientArgs coefficients(coefficient_count, coefficient_data, coefficient_dtypes, coefficient_counts);
  return DispatchStorage(dtype, [&](auto tag) {
    constexpr auto Dtype = decltype(tag)::value;
    int64_t source_dims[2] = {batches, source_size};
    int64_t output_dims[2] = {batches, output_size};
    auto input = MakeBuffer(dtype, source, 2, source_dims);
    auto result = MakeBuffer(dtype, output, 2, output_dims);
    auto future = native::Accumulation<Dtype>({words, word_count},
        {coefficient_records, coefficient_count}, prepared->get(), ffi::AnyBuffer(&input),
        ffi::RemainingArgs(&coefficients.args, 0), ffi::BufferR2<Dtype>(&result),
        Pool(threads).Get(), outputs_disjoint);
    return Wait(std::move(future), error, error_size);
  });
}

// Reduction (partial trace): InstantiateReduction (prepared.cc:47-61) + Reduction
// (ffi/reduction_impl.h:152-160).
int t0ref_reduction(int dtype, const uint8_t* bytes, size_t byte_count,
                    const int64_t* coefficient_records, size_t coefficient_count,
                    const void* const* coefficient_data, const int* coefficient_dtypes,
                    const int64_t* coefficient_counts, const void* source, int64_t source_size,
                    void* output, int64_t output_size, int64_t batches, int64_t threads,
                    char* error, size_t error_size) {
  auto prepared = native::InstantiateReduction({bytes, byte_count}, {coefficient_records, coefficient_count});
  if (!prepared.has_value()) return Report(prepared.error(), error, error_size);
  CoefficientArgs coefficients(coefficient_count, coefficient_data, coefficient_dtypes, coefficient_counts);
  return DispatchStorage(dtype, [&](auto tag) {
    constexpr auto Dtype = decltype(tag)::value;
    int64_t source_dims[2] = {batches, source_size};
    int64_t output_dims[2] = {batches, output_size};
    auto input = MakeBuffer(dtype, source, 2, source_dims);
    auto result = MakeBuffer(dtype, output, 2, output_dims);
    auto future = native::Reduction<Dtype>({bytes, byte_count}, {coefficient_records, coefficient_count},
        prepared->get(), ffi::AnyBuffer(&input), ffi::RemainingArgs(&coefficients.args, 0),
        ffi::BufferR2<Dtype>(&result), Pool(threads).Get());
    return Wait(std::move(future), error, error_size);
  });
}

// Update: InstantiatePrepared + Update (ffi/update_impl.h:87-190).  The result
// may alias the base buffer, as in the handler's operand_output_aliases {1:0}.
int t0ref_update(int dtype, const int64_t* words, size_t word_count,
                 const void* source, int64_t source_size, const void* base, void* output,
                 int64_t output_size, const void* alpha, int alpha_dtype, int64_t alpha_count,
                 const void* beta, int beta_dtype, int64_t beta_count, int64_t batches,
                 int64_t threads, char* error, size_t error_size) {
  auto prepared = native::InstantiatePrepared({words, word_count});
  if (!prepared.has_value()) return Report(prepared.error(), error, error_size);
  return DispatchStorage(dtype, [&](auto tag) {
    constexpr auto Dtype = decltype(tag)::value;
    int64_t source_dims[2] = {batches, source_size};
    int64_t output_dims[2] = {batches, output_size};
    int64_t alpha_dims[1] = {alpha_count};
    int64_t beta_dims[1] = {beta_count};
    auto input = MakeBuffer(dtype, source, 2, source_dims);
    auto old = MakeBuffer(dtype, base, 2, output_dims);
    auto result = MakeBuffer(dtype, output, 2, output_dims);
    auto a = MakeBuffer(alpha_dtype, alpha, alpha_count < 0 ? 0 : 1, alpha_count < 0 ? nullptr : alpha_dims);
    auto b = MakeBuffer(beta_dtype, beta, beta_count < 0 ? 0 : 1, beta_count < 0 ? nullptr : beta_dims);
    auto future = native::Update<Dtype>({words, word_count}, prepared->get(), ffi::AnyBuffer(&input),
        ffi::BufferR2<Dtype>(&old), ffi::AnyBuffer(&a), ffi::AnyBuffer(&b),
        ffi::BufferR2<Dtype>(&result), Pool(threads).Get());
    return Wait(std::move(future), error, error_size);
  });
}

// Dot: InstantiateDot (prepared.cc:66-75) + Dot (ffi/dot_impl.h:51-110).
int t0ref_dot(int dtype, const int64_t* words, size_t word_count, int64_t conjugate_left, const void* left,
              int64_t left_size, const void* right, int64_t right_size, void* output, int64_t batches,
              int64_t threads, char* error, size_t error_size) {
  auto prepared = native::InstantiateDot({words, word_count}, conjugate_left);
  if (!prepared.has_value()) return Report(prepared.error(), error, error_size);
  return DispatchStorage(dtype, [&](auto tag) {
    constexpr auto Dtype = decltype(tag)::value;
    int64_t left_dims[2] = {batches, left_size};
    int64_t right_dims[2] = {batches, right_size};
    int64_t output_dims[1] = {batches};
    auto a = MakeBuffer(dtype, left, 2, left_dims);
    auto b = MakeBuffer(dtype, right, 2, right_dims);
    auto result = MakeBuffer(dtype, output, 1, output_dims);
    auto future = native::Dot<Dtype>({words, word_count}, conjugate_left, prepared->get(), ffi::AnyBuffer(&a),
                                     ffi::AnyBuffer(&b), ffi::BufferR1<Dtype>(&result), Pool(threads).Get());
    return Wait(std::move(future), error, error_size);
  });
}

// A prepared call: instantiated once, executed many times.
struct t0ref_call {
  int32_t operation = 0;          // 1 update, 3 accumulation
  std::vector<int64_t> words;
  std::vector<int64_t> records;
  int64_t outputs_disjoint = 0;
  std::unique_ptr<native::PreparedState> state;
};

t0ref_call* t0ref_prepare(int32_t operation, const int64_t* words, size_t word_count,
                          const int64_t* coefficient_records, size_t coefficient_count,
                          int64_t outputs_disjoint, char* error, size_t error_size) {
  auto call = std::make_unique<t0ref_call>();
  call->operation = operation;
  call->words.assign(words, words + word_count);
  call->records.assign(coefficient_records, coefficient_records + coefficient_count);
  call->outputs_disjoint = outputs_disjoint;
  const ffi::Span<const int64_t> layout(call->words.data(), call->words.size());
  const ffi::Span<const int64_t> records(call->records.data(), call->records.size());
  auto prepared = operation == 3 ? native::InstantiateAccumulation(layout, records, outputs_disjoint)
                                 : native::InstantiatePrepared(layout);
  if (!prepared.has_value()) {
    Report(prepared.error(), error, error_size);
    return nullptr;
  }
  call->state = std::move(*prepared);
  return call.release();
}

void t0ref_release(t0ref_call* call) { delete call; }

int t0ref_execute_accumulation(const t0ref_call* call, int dtype, const void* const* coefficient_data,
                               const int* coefficient_dtypes, const int64_t* coefficient_counts,
                               const void* source, int64_t source_size, void* output, int64_t output_size,
                               int64_t batches, int64_t threads, char* error, size_t error_size) {
  CoefficientArgs coefficients(call->records.size(), coefficient_data, coefficient_dtypes, coefficient_counts);
  return DispatchStorage(dtype, [&](auto tag) {
    constexpr auto Dtype = decltype(tag)::value;
    int64_t source_dims[2] = {batches, source_size};
    int64_t output_dims[2] = {batches, output_size};
    auto input = MakeBuffer(dtype, source, 2, source_dims);
    auto result = MakeBuffer(dtype, output, 2, output_dims);
    auto future = native::Accumulation<Dtype>({call->words.data(), call->words.size()},
        {call->records.data(), call->records.size()}, call->state.get(), ffi::AnyBuffer(&input),
        ffi::RemainingArgs(&coefficients.args, 0), ffi::BufferR2<Dtype>(&result),
        Pool(threads).Get(), call->outputs_disjoint);
    return Wait(std::move(future), error, error_size);
  });
}

int t0ref_execute_update(const t0ref_call* call, int dtype, const void* source, int64_t source_size,
                         const void* base, void* output, int64_t output_size, const void* alpha,
                         int alpha_dtype, int64_t alpha_count, const void* beta, int beta_dtype,
                         int64_t beta_count, int64_t batches, int64_t threads, char* error, size_t error_size) {
  return DispatchStorage(dtype, [&](auto tag) {
    constexpr auto Dtype = decltype(tag)::value;
    int64_t source_dims[2] = {batches, source_size};
    int64_t output_dims[2] = {batches, output_size};
    int64_t alpha_dims[1] = {alpha_count};
    int64_t beta_dims[1] = {beta_count};
    auto input = MakeBuffer(dtype, source, 2, source_dims);
    auto old = MakeBuffer(dtype, base, 2, output_dims);
    auto result = MakeBuffer(dtype, output, 2, output_dims);
    auto a = MakeBuffer(alpha_dtype, alpha, alpha_count < 0 ? 0 : 1, alpha_count < 0 ? nullptr : alpha_dims);
    auto b = MakeBuffer(beta_dtype, beta, beta_count < 0 ? 0 : 1, beta_count < 0 ? nullptr : beta_dims);
    auto future = native::Update<Dtype>({call->words.data(), call->words.size()}, call->state.get(),
        ffi::AnyBuffer(&input), ffi::BufferR2<Dtype>(&old), ffi::AnyBuffer(&a), ffi::AnyBuffer(&b),
        ffi::BufferR2<Dtype>(&result), Pool(threads).Get());
    return Wait(std::move(future), error, error_size);
  });
}

}  // extern "C"
