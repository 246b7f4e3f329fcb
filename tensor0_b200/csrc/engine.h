// Kernel launch interface of the map and reduce engines.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <stdexcept>
#include <string>

#include "layout.h"
#include "plan.h"

namespace t0b {

using InvalidArgumentError = InvalidArgument;

enum MapOp : int { kOpCopy = 0, kOpUpdate = 1, kOpAccumulation = 3 };

struct MapArgs {
  const MapRecord* recs;
  int64_t nrec;
  int64_t tiles_per_batch;
  int64_t batches;
  const void* src;
  const void* base;
  void* out;
  int64_t src_size;
  int64_t out_size;
  int64_t tile_elems;  // shared-memory elements of the staged tile (the base buffer follows)
  const void* ca;      // accumulation: coefficient rows; update: alpha
  int64_t ca_count;
  const void* cb;      // update: beta
  int64_t cb_count;
  int conjugate;       // accumulation: read conj(source) (complex storage)
};

struct ReduceArgs {
  const ReduceGroup* groups;
  const ReduceRecord* records;
  int64_t group_begin, group_end;   // wave
  int64_t task_begin, task_end;
  int64_t owner_begin, owner_end;
  int64_t batches;
  const void* src;
  void* out;
  void* scratch;
  int64_t scratch_stride;           // scratch elements per batch
  int64_t src_size;
  int64_t out_size;
  const void* ca;
  int64_t ca_count;
  int conjugate;                    // read conj(source) (complex storage)
  int assign;                       // pass 2 writes 0 + sum (the output was not zeroed) instead of adding
};

struct DotArgs {
  const DotRecord* recs;
  int64_t nrec;
  int64_t units;                    // per batch
  int64_t batches;
  const void* left;
  const void* right;
  void* out;                        // [batches]
  void* partials;                   // [batches][kDotPartials]
  int64_t left_size;
  int64_t right_size;
  int conjugate_left;
};

struct GroupedArgs {
  const GroupedGroup* groups;
  const GroupedOperand* operands;
  int64_t ngroups;
  int64_t units;                    // per batch
  int64_t batches;
  const void* src;
  void* out;
  const void* matrices;             // row-major [n_dst][n_src] per group, in group order
  int64_t src_size;
  int64_t out_size;
};

extern std::atomic<uint64_t> g_kernel_launches;

// Multiprocessors of the current device.
int SmCount();

// Throw std::runtime_error for a failed CUDA runtime call.
void Check(cudaError_t status, const char* what);

// Largest padded tile (shared-memory elements) and largest tile box over a plan's records.
void MapTileElements(const MapRecord* recs, int64_t count, int element_bytes, int64_t* tile, int64_t* box);
// Dynamic shared memory of one map CTA for an operation: every pipeline stage
// holds a staged tile (and, for update, the base values after it).
int64_t MapSharedBytes(int op, int64_t tile_elems, int element_bytes);
void LaunchMap(int op, int32_t dtype, int32_t ca_dtype, int32_t cb_dtype, const MapArgs& args,
               int smem, bool wide, cudaStream_t stream);
void LaunchReduce(int32_t dtype, int32_t ca_dtype, const ReduceArgs& args, cudaStream_t stream);
void LaunchDot(int32_t dtype, const DotArgs& args, cudaStream_t stream);
// One launch of the grouped-transform kernel; matrix_dtype is the storage's
// real type or (complex storage) its complex type; stage_bytes is the dynamic
// shared memory of a tiled unit (the plan's grouped_stage elements).
void LaunchGrouped(int32_t dtype, int32_t matrix_dtype, const GroupedArgs& args, int64_t stage_bytes,
                   cudaStream_t stream);
void LaunchAxpby(int32_t dtype, int64_t n, double ar, double ai, const void* x, double br, double bi,
                 const void* y, void* out, cudaStream_t stream);

}  // namespace t0b
