// Element arithmetic with explicit IEEE round-to-nearest operations and no
// contraction, so results match the reference's CPU executors bit for bit
// where the reference defines the operation order:
//   products and sums:      numeric/scalar.h:268-320 (CPU),
//                           native/cuda/arithmetic.cuh:16-39 (CUDA);
//   complex x complex:      {fma(ar, br, -(ai*bi)), fma(ai, br, ar*bi)};
//   real x complex:         componentwise products;
//   accumulation into zero: 0 + x (turns -0 into +0, keeps NaN payloads).
#pragma once

#include <cuda_runtime.h>
#include <cstdint>

#include "plan.h"

namespace t0b {

// Division by a constant computed on the host (MakeDivision).
struct FastDiv {
  uint32_t m, l;
  __device__ __forceinline__ uint32_t Div(uint32_t n) const { return (__umulhi(n, m) + n) >> l; }
};

__device__ __forceinline__ FastDiv Division(const DivisionConstants& c) { return FastDiv{c.magic, c.shift}; }

template <typename T> struct Elem;
template <> struct Elem<float>   { using Real = float;  static constexpr bool kComplex = false; };
template <> struct Elem<double>  { using Real = double; static constexpr bool kComplex = false; };
template <> struct Elem<float2>  { using Real = float;  static constexpr bool kComplex = true; };
template <> struct Elem<double2> { using Real = double; static constexpr bool kComplex = true; };

__device__ __forceinline__ float Mul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ double Mul(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ float Add(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ double Add(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ float Fma(float a, float b, float c) { return __fmaf_rn(a, b, c); }
__device__ __forceinline__ double Fma(double a, double b, double c) { return __fma_rn(a, b, c); }

__device__ __forceinline__ float2 Add(float2 a, float2 b) { return {Add(a.x, b.x), Add(a.y, b.y)}; }
__device__ __forceinline__ double2 Add(double2 a, double2 b) { return {Add(a.x, b.x), Add(a.y, b.y)}; }

// Coefficient products.  A coefficient is the storage's real type, or (for
// complex storage) its complex type; S32 coefficients are converted to the
// real type when read.
__device__ __forceinline__ float Scale(float c, float v) { return Mul(c, v); }
__device__ __forceinline__ double Scale(double c, double v) { return Mul(c, v); }
__device__ __forceinline__ float2 Scale(float c, float2 v) { return {Mul(c, v.x), Mul(c, v.y)}; }
__device__ __forceinline__ double2 Scale(double c, double2 v) { return {Mul(c, v.x), Mul(c, v.y)}; }
__device__ __forceinline__ float2 Scale(float2 c, float2 v) {
  return {Fma(c.x, v.x, -Mul(c.y, v.y)), Fma(c.y, v.x, Mul(c.x, v.y))};
}
__device__ __forceinline__ double2 Scale(double2 c, double2 v) {
  return {Fma(c.x, v.x, -Mul(c.y, v.y)), Fma(c.y, v.x, Mul(c.x, v.y))};
}

__device__ __forceinline__ bool IsZero(float c) { return c == 0.0f; }
__device__ __forceinline__ bool IsZero(double c) { return c == 0.0; }
__device__ __forceinline__ bool IsZero(float2 c) { return c.x == 0.0f && c.y == 0.0f; }
__device__ __forceinline__ bool IsZero(double2 c) { return c.x == 0.0 && c.y == 0.0; }
__device__ __forceinline__ bool IsOne(float c) { return c == 1.0f; }
__device__ __forceinline__ bool IsOne(double c) { return c == 1.0; }
__device__ __forceinline__ bool IsOne(float2 c) { return c.x == 1.0f && c.y == 0.0f; }
__device__ __forceinline__ bool IsOne(double2 c) { return c.x == 1.0 && c.y == 0.0; }

// 0 + x: identical to x except that -0 becomes +0.
__device__ __forceinline__ float PlusZero(float v) { return v == 0.0f ? 0.0f : v; }
__device__ __forceinline__ double PlusZero(double v) { return v == 0.0 ? 0.0 : v; }
__device__ __forceinline__ float2 PlusZero(float2 v) { return {PlusZero(v.x), PlusZero(v.y)}; }
__device__ __forceinline__ double2 PlusZero(double2 v) { return {PlusZero(v.x), PlusZero(v.y)}; }

template <typename T> __device__ __forceinline__ T Zero() { return T{}; }

// Coefficient value types: S32 is read as the storage real type; real and
// complex coefficients are used as stored.
template <typename Real, typename Raw> struct BoundOf { using type = Raw; };
template <typename Real> struct BoundOf<Real, int32_t> { using type = Real; };

// Coefficient `row` for batch `batch` from a device array with `count`
// values per row (count 1: shared by every batch).
template <typename Real, typename Raw>
__device__ __forceinline__ typename BoundOf<Real, Raw>::type
ReadCoefficient(const Raw* data, int64_t row, int64_t count, int64_t batch) {
  const Raw raw = data[row * count + (count == 1 ? 0 : batch)];
  return static_cast<typename BoundOf<Real, Raw>::type>(raw);
}

}  // namespace t0b
