// Partial-trace reduction whose scratch lives in the library itself, for
// callers that cannot allocate device memory.
//
// Such callers include an XLA FFI custom call: XLA owns every device buffer
// and a handler must not allocate (the reference's CUDA handlers allocate
// nothing per call).  Another is a host application whose device memory is
// fully reserved by its own pool, so a cudaMalloc would fail or would bypass
// that pool.  Those callers still pass the inputs, the output, the
// coefficients and the plan's device table; only the reduce engine's pass-1
// partials move into the file-scope array below.
//
// The array has a fixed size, kStaticScratchBytes per device.  Every GPU that
// loads this library holds it until the process exits.
#include "../../include/tensor0_b200.h"

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

namespace {

constexpr size_t kStaticScratchBytes = size_t{16} << 20;   // 16 MiB per device
constexpr int kMaxDevices = 64;

// Device-side storage.  In host code this name is only a stand-in: its device
// address must come from cudaGetSymbolAddress on each device.
__device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

// The array's device address per device, with the context it was looked up
// in.  A module is loaded per context, so a different current context (a
// driver-API context, or a primary context recreated after cudaDeviceReset
// under a new handle) gets its own lookup.
struct ScratchAddress {
  CUcontext context = nullptr;
  void* address = nullptr;
};
ScratchAddress g_scratch_address[kMaxDevices];
std::mutex g_setup;

// cuCtxGetCurrent through the runtime's driver entry point, so the library
// needs no link against the driver library.
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
  if (function == nullptr) return CUDA_ERROR_NOT_FOUND;
  return function(context);
}

int Fail(char* error, size_t size, int status, const char* text) {
  if (error != nullptr && size != 0) std::snprintf(error, size, "tensor0-b200: %s", text);
  return status;
}

int ElementBytes(int32_t dtype) {
  switch (dtype) {
    case T0B_F32: return 4;
    case T0B_F64: case T0B_C64: return 8;
    case T0B_C128: return 16;
    default: return 0;
  }
}

}  // namespace

extern "C" int t0b_reduction_static_scratch(const t0b_plan* plan, int32_t dtype, const void* source, void* output,
                                            int64_t batches, const void* coefficients, int32_t coefficient_dtype,
                                            int64_t coefficient_count, const int64_t* device_table, void* stream,
                                            char* error, size_t error_size) {
  if (plan == nullptr) return Fail(error, error_size, 1, "plan is null");
  if (batches < 0) return Fail(error, error_size, 1, "batch count must be nonnegative");
  const int bytes = ElementBytes(dtype);
  if (bytes == 0) return Fail(error, error_size, 1, "CUDA stride storage supports only F32/F64/C64/C128");
  const uint64_t per_batch = t0b_plan_scratch_elements(plan);
  const unsigned __int128 need = static_cast<unsigned __int128>(per_batch) * static_cast<uint64_t>(batches) * bytes;
  if (need > kStaticScratchBytes) {
    char text[256];
    std::snprintf(text, sizeof text,
                  "this reduction needs %llu bytes of scratch; the library's static scratch holds %llu bytes "
                  "(use t0b_reduction with caller-provided scratch)",
                  static_cast<unsigned long long>(need > ~0ull ? ~0ull : static_cast<unsigned long long>(need)),
                  static_cast<unsigned long long>(kStaticScratchBytes));
    return Fail(error, error_size, 1, text);
  }
  void* scratch = nullptr;
  if (need != 0) {
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices) {
      return Fail(error, error_size, 2, "cannot identify the current CUDA device");
    }
    // No context is current yet on a thread where the runtime has not touched
    // the device; the symbol lookup below then initialises the primary one.
    CUcontext context = nullptr;
    if (CurrentContext(&context) != CUDA_SUCCESS) {
      return Fail(error, error_size, 2, "cannot identify the current CUDA context");
    }
    std::lock_guard<std::mutex> lock(g_setup);
    ScratchAddress& cached = g_scratch_address[device];
    if (cached.address == nullptr || context == nullptr || cached.context != context) {
      // Once per device (and context), with that device current: resolve the
      // array's device address.
      void* address = nullptr;
      const cudaError_t status = cudaGetSymbolAddress(&address, g_static_scratch);
      if (status != cudaSuccess || address == nullptr) {
        char text[256];
        std::snprintf(text, sizeof text, "cudaGetSymbolAddress of the static scratch failed: %s",
                      cudaGetErrorString(status));
        return Fail(error, error_size, 2, text);
      }
      if (context == nullptr && (CurrentContext(&context) != CUDA_SUCCESS || context == nullptr)) {
        return Fail(error, error_size, 2, "cannot identify the current CUDA context");
      }
      cached.context = context;
      cached.address = address;
    }
    scratch = cached.address;
  }
  return t0b_reduction(plan, dtype, source, output, batches, coefficients, coefficient_dtype, coefficient_count,
                       scratch, device_table, stream, error, error_size);
}
