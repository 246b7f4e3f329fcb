// Grouped per-sector GEMM launch interface.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace t0b {

// Device table row: {m, n, k, a_off, b_off, c_off, tile_begin, tc_tile_begin}:
// prefixes over sectors of 64 x 64 tiles (DMMA and FMA kernels) and of
// 128 x 64 tiles (the tcgen05 FP32 kernel).
constexpr int kGemmRow = 8;

void BuildGemmTable(int64_t sectors, const int64_t* spec, int64_t* table);
// Validates every table row against the operand sizes (elements), the
// operands' alignment and overlaps, then launches; throws InvalidArgument.
void SectorGemm(int32_t dtype, int64_t sectors, const int64_t* host_table, const int64_t* device_table,
                const void* left, int64_t left_size, const void* right, int64_t right_size, void* output,
                int64_t output_size, cudaStream_t stream);

}  // namespace t0b
