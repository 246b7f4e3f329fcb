// Grouped per-sector GEMM behind block-sparse contraction: for every coupled
// sector g, C_g = A_g @ B_g over row-major blocks sliced from flat storage
// (the reference loops over sectors with one XLA dot each,
// src/tensor0/tensor/linalg.py:533-566, then concatenates, _blocks.py:83-131).
// Here every 64x64 output tile of every sector is one task of a single
// persistent grid.
//
// F64 and C128 use the FP64 tensor-core MMA (mma.sync m8n8k4 f64, "DMMA");
// C128 uses four real products per complex product; operands are staged with
// cp.async (zero-filled at edges) in two stages.  F32 and C64 use the
// 5th-generation tensor cores (tcgen05.mma kind::tf32, accumulators in tensor
// memory) with a three-term TF32 split, each K slice summed in FP32 registers
// (TcGemm, TcGemmComplex).
#include "gemm.h"

#include "engine.h"

#include <algorithm>
#include <string>
#include <utility>
#include <vector>

namespace t0b {
namespace {

constexpr int kGemmThreads = 256;
constexpr int kTile = 64;

__device__ __forceinline__ int64_t FindSector(const int64_t* table, int64_t sectors, int64_t tile) {
  int64_t lo = 0, hi = sectors - 1;
  while (lo < hi) {
    const int64_t mid = (lo + hi + 1) >> 1;
    if (table[mid * kGemmRow + 6] <= tile) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ void CpAsync8(void* smem, const void* gmem, bool valid) {
  const unsigned dst = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  const int bytes = valid ? 8 : 0;
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n" ::"r"(dst), "l"(gmem), "r"(bytes));
}
__device__ __forceinline__ void CpAsync16(void* smem, const void* gmem, bool valid) {
  const unsigned dst = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  const int bytes = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(gmem), "r"(bytes));
}
__device__ __forceinline__ void CpCommit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void CpWait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

// D = A(8x4, row) * B(4x8, col) + D on the FP64 tensor cores.
__device__ __forceinline__ void Dmma(double (&d)[2], double a, double b) {
  asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0,%1}, {%2}, {%3}, {%0,%1};\n"
               : "+d"(d[0]), "+d"(d[1])
               : "d"(a), "d"(b));
}

struct Task {
  int64_t m, n, k, a, b, c;
  int64_t m0, n0;
};

__device__ __forceinline__ Task DecodeTask(const int64_t* table, int64_t sectors, int64_t tile) {
  const int64_t s = FindSector(table, sectors, tile);
  const int64_t* row = table + s * kGemmRow;
  Task t;
  t.m = row[0]; t.n = row[1]; t.k = row[2];
  t.a = row[3]; t.b = row[4]; t.c = row[5];
  const int64_t local = tile - row[6];
  const int64_t tiles_n = (t.n + kTile - 1) / kTile;
  t.m0 = (local / tiles_n) * kTile;
  t.n0 = (local % tiles_n) * kTile;
  return t;
}

// ---------------------------------------------------------------------------
// FP64 / complex128 on DMMA.  8 warps as 2 (M) x 4 (N); a warp owns 32x16 of
// the 64x64 tile = 4 x 2 fragments of 8x8.
template <bool kComplex>
__global__ void __launch_bounds__(kGemmThreads) DmmaGemm(const int64_t* __restrict__ table, int64_t sectors,
                                                         int64_t tiles, const double* __restrict__ left,
                                                         const double* __restrict__ right, double* out) {
  // Real: K tile 16, pads keep fragment loads conflict-free.  Complex: K tile
  // 8 complex values, stored interleaved.
  constexpr int BK = kComplex ? 8 : 16;
  constexpr int W = kComplex ? 2 : 1;              // doubles per element
  constexpr int APITCH = kComplex ? (BK + 4) : (BK + 4);
  constexpr int BPITCH = kComplex ? (kTile + 2) : (kTile + 4);
  __shared__ __align__(16) double As[2][kTile * APITCH * W];
  __shared__ __align__(16) double Bs[2][BK * BPITCH * W];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int wm = warp & 1, wn = warp >> 1;
  const int fr = lane >> 2, fc = lane & 3;

  for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    const Task t = DecodeTask(table, sectors, tile);
    double acc[4][2][2] = {};
    double acci[4][2][2] = {};
    const int64_t ktiles = (t.k + BK - 1) / BK;

    auto stage = [&](int buf, int64_t k0) {
      if constexpr (!kComplex) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {            // A: 64 x 16 doubles
          const int e = tid + i * kGemmThreads;
          const int r = e >> 4, c = e & 15;
          const bool ok = t.m0 + r < t.m && k0 + c < t.k;
          const double* g = ok ? left + t.a + (t.m0 + r) * t.k + k0 + c : left;
          CpAsync8(&As[buf][r * APITCH + c], g, ok);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {            // B: 16 x 64 doubles
          const int e = tid + i * kGemmThreads;
          const int r = e >> 6, c = e & 63;
          const bool ok = k0 + r < t.k && t.n0 + c < t.n;
          const double* g = ok ? right + t.b + (k0 + r) * t.n + t.n0 + c : right;
          CpAsync8(&Bs[buf][r * BPITCH + c], g, ok);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 2; ++i) {            // A: 64 x 8 complex
          const int e = tid + i * kGemmThreads;
          const int r = e >> 3, c = e & 7;
          const bool ok = t.m0 + r < t.m && k0 + c < t.k;
          const double* g = ok ? left + 2 * (t.a + (t.m0 + r) * t.k + k0 + c) : left;
          CpAsync16(&As[buf][2 * (r * APITCH + c)], g, ok);
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {            // B: 8 x 64 complex
          const int e = tid + i * kGemmThreads;
          const int r = e >> 6, c = e & 63;
          const bool ok = k0 + r < t.k && t.n0 + c < t.n;
          const double* g = ok ? right + 2 * (t.b + (k0 + r) * t.n + t.n0 + c) : right;
          CpAsync16(&Bs[buf][2 * (r * BPITCH + c)], g, ok);
        }
      }
      CpCommit();
    };

    if (ktiles > 0) stage(0, 0);
    for (int64_t kt = 0; kt < ktiles; ++kt) {
      const int buf = static_cast<int>(kt & 1);
      if (kt + 1 < ktiles) { stage(buf ^ 1, (kt + 1) * BK); CpWait<1>(); } else { CpWait<0>(); }
      __syncthreads();
#pragma unroll
      for (int kk = 0; kk < BK; kk += 4) {
        if constexpr (!kComplex) {
          double a[4], b[2];
#pragma unroll
          for (int f = 0; f < 4; ++f) a[f] = As[buf][(wm * 32 + f * 8 + fr) * APITCH + kk + fc];
#pragma unroll
          for (int g = 0; g < 2; ++g) b[g] = Bs[buf][(kk + fc) * BPITCH + wn * 16 + g * 8 + fr];
#pragma unroll
          for (int f = 0; f < 4; ++f)
#pragma unroll
            for (int g = 0; g < 2; ++g) Dmma(acc[f][g], a[f], b[g]);
        } else {
          double ar[4], ai[4], br[2], bi[2];
#pragma unroll
          for (int f = 0; f < 4; ++f) {
            const double2 v = *reinterpret_cast<const double2*>(&As[buf][2 * ((wm * 32 + f * 8 + fr) * APITCH + kk + fc)]);
            ar[f] = v.x; ai[f] = v.y;
          }
#pragma unroll
          for (int g = 0; g < 2; ++g) {
            const double2 v = *reinterpret_cast<const double2*>(&Bs[buf][2 * ((kk + fc) * BPITCH + wn * 16 + g * 8 + fr)]);
            br[g] = v.x; bi[g] = v.y;
          }
#pragma unroll
          for (int f = 0; f < 4; ++f)
#pragma unroll
            for (int g = 0; g < 2; ++g) {
              Dmma(acc[f][g], ar[f], br[g]);
              Dmma(acc[f][g], -ai[f], bi[g]);
              Dmma(acci[f][g], ar[f], bi[g]);
              Dmma(acci[f][g], ai[f], br[g]);
            }
        }
      }
      __syncthreads();
    }
    // Epilogue: fragment (f, g) holds rows fr, columns 2*fc + {0, 1}.
#pragma unroll
    for (int f = 0; f < 4; ++f) {
      const int64_t row = t.m0 + wm * 32 + f * 8 + fr;
      if (row >= t.m) continue;
#pragma unroll
      for (int g = 0; g < 2; ++g) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int64_t col = t.n0 + wn * 16 + g * 8 + 2 * fc + j;
          if (col >= t.n) continue;
          const int64_t at = t.c + row * t.n + col;
          if constexpr (kComplex) {
            reinterpret_cast<double2*>(out)[at] = double2{acc[f][g][j], acci[f][g][j]};
          } else {
            out[at] = acc[f][g][j];
          }
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// FP32 on tcgen05 (kind::tf32).  A CTA of 128 threads owns 128 x 64 output
// tiles (the table's second tile prefix).  Each operand value x is split into
// hi = tf32(x) and lo = tf32(x - hi); a 32-deep K slice issues, per 8-deep MMA
// step, lo(A) hi(B) + hi(A) lo(B) + hi(A) hi(B) into one of two tensor-memory
// accumulators (the dropped lo lo term is below 2^-22 relative).  The tensor
// core's accumulation over long K is not IEEE: measured 2e-6 (K = 256) and
// 7e-6 (K = 1000) relative error when all of K stays in tensor memory.  So
// every slice starts from zero and is added into FP32 registers: thread r
// reads tensor-memory lane r (its output row) after the slice's MMAs
// complete.  Two stages: slice s + 1 is copied (cp.async) while slice s is
// split and multiplied, and the two accumulators alternate.
// Shared-memory tiles are K-major without swizzle: 16-byte chunks of four k
// values, chunk-major over the tile's rows (leading byte offset = one chunk of
// all rows, stride byte offset = 8 rows).
constexpr int kTcM = 128, kTcN = 64, kTcK = 32;
constexpr int kTcThreads = 256;   // warp w drains lanes 32 (w % 4).. and columns 32 (w / 4)..
constexpr uint32_t kTcABytes = kTcM * kTcK * 4;   // 16 KB: one part (hi or lo) of an A slice
constexpr uint32_t kTcBBytes = kTcN * kTcK * 4;   // 8 KB
constexpr uint32_t kTcStageBytes = 2 * kTcABytes + 2 * kTcBBytes;
constexpr int kTcSmem = 2 * kTcStageBytes;        // two stages: 96 KB
constexpr uint32_t kTcTmemColumns = 2 * kTcN;     // two accumulators
constexpr uint32_t kTcSpinLimit = 1u << 24;       // mbarrier polls before a wait gives up

__device__ __forceinline__ uint32_t Tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

// Asynchronous 4-byte copy into shared memory; zero-filled when !valid.
__device__ __forceinline__ void TcCopy4(uint32_t dst, const float* src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(valid ? 4 : 0) : "memory");
}

__device__ __forceinline__ uint64_t SmemDescriptor(uint32_t addr, uint32_t leading, uint32_t stride) {
  return static_cast<uint64_t>((addr >> 4) & 0x3FFF) | (static_cast<uint64_t>((leading >> 4) & 0x3FFF) << 16) |
         (static_cast<uint64_t>((stride >> 4) & 0x3FFF) << 32) | (uint64_t{1} << 46);
}

__device__ __forceinline__ void MmaTf32(uint32_t tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  const uint32_t mask = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}\n"
      :: "r"(tmem), "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(mask));
}

// Bounded wait for an mbarrier phase; false if it gave up.
__device__ __forceinline__ bool WaitPhase(uint32_t mbar, uint32_t parity) {
  for (uint32_t i = 0; i < kTcSpinLimit; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done) : "r"(mbar), "r"(parity) : "memory");
    if (done) return true;
  }
  return false;
}

__device__ __forceinline__ void TmemLoad32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
}

struct TcTask {
  int64_t m, n, k, a, b, c, m0, n0;
};

__device__ __forceinline__ TcTask DecodeTcTask(const int64_t* table, int64_t sectors, int64_t tile) {
  int64_t lo = 0, hi = sectors - 1;
  while (lo < hi) {
    const int64_t mid = (lo + hi + 1) >> 1;
    if (table[mid * kGemmRow + 7] <= tile) lo = mid; else hi = mid - 1;
  }
  const int64_t* row = table + lo * kGemmRow;
  TcTask t;
  t.m = row[0]; t.n = row[1]; t.k = row[2];
  t.a = row[3]; t.b = row[4]; t.c = row[5];
  const int64_t local = tile - row[7];
  const int64_t tiles_n = (t.n + kTcN - 1) / kTcN;
  t.m0 = (local / tiles_n) * kTcM;
  t.n0 = (local % tiles_n) * kTcN;
  return t;
}

__global__ void __launch_bounds__(kTcThreads, 1) TcGemm(const int64_t* __restrict__ table, int64_t sectors,
                                                       int64_t tiles, const float* __restrict__ left,
                                                       const float* __restrict__ right, float* out) {
  extern __shared__ __align__(1024) unsigned char tc_smem[];
  __shared__ __align__(8) uint64_t mbar_storage[2];
  __shared__ uint32_t tmem_slot;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, half = warp >> 2;   // tensor-memory lane quarter, accumulator column half
  const uint32_t smem = static_cast<uint32_t>(__cvta_generic_to_shared(tc_smem));
  const uint32_t mbar0 = static_cast<uint32_t>(__cvta_generic_to_shared(&mbar_storage[0]));
  if (warp == 0) {
    const uint32_t slot = static_cast<uint32_t>(__cvta_generic_to_shared(&tmem_slot));
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" :: "r"(slot), "r"(kTcTmemColumns));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" :: "r"(mbar0));
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" :: "r"(mbar0 + 8));
    asm volatile("fence.mbarrier_init.release.cluster;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;");
  const uint32_t tmem = tmem_slot;
  // kind::tf32, F32 accumulate, A and B K-major, N = 64, M = 128.
  const uint32_t idesc = (1u << 4) | (2u << 7) | (2u << 10) | ((kTcN >> 3) << 17) | ((kTcM >> 4) << 24);
  uint32_t parity[2] = {0, 0};
  bool ok = true;
  for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    const TcTask t = DecodeTcTask(table, sectors, tile);
    float acc[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) acc[j] = 0.0f;
    const int64_t slices = (t.k + kTcK - 1) / kTcK;
    // Add slice `s`'s accumulator (buffer s & 1) into the registers.
    auto drain = [&](int64_t s) {
      const int buf = static_cast<int>(s & 1);
      ok = WaitPhase(mbar0 + 8 * buf, parity[buf]) && ok;
      parity[buf] ^= 1u;
      asm volatile("tcgen05.fence::after_thread_sync;");
      float v[32];
      TmemLoad32(tmem + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(buf * kTcN + half * 32), v);
#pragma unroll
      for (int j = 0; j < 32; ++j) acc[j] = __fadd_rn(acc[j], v[j]);
    };
    // Slice s lands in stage s & 1: raw values by cp.async at their K-major
    // positions in the hi buffers; each thread then splits the values it
    // copied itself (hi in place, lo beside it).  A warp's A piece is 8 rows x
    // one 4-value chunk (coalesced 16-byte pieces, one contiguous 128-byte run
    // of shared memory); its B piece is 8 columns x 4 k rows.
    auto a_position = [&](int e, int& m, int& k) -> uint32_t {
      const int k_in = e & 3, m_lo = (e >> 2) & 7, chunk = (e >> 5) & 7, m_hi = e >> 8;
      m = m_hi * 8 + m_lo;
      k = chunk * 4 + k_in;
      return ((static_cast<uint32_t>(chunk) * kTcM + m) << 4) + (k_in << 2);
    };
    auto b_position = [&](int e, int& n, int& k) -> uint32_t {
      const int l = e & 31, w = e >> 5;
      const int k_in = l >> 3, chunk = w >> 3;
      n = (w & 7) * 8 + (l & 7);
      k = chunk * 4 + k_in;
      return ((static_cast<uint32_t>(chunk) * kTcN + n) << 4) + (k_in << 2);
    };
    // A moves in 16-byte chunks (four k values of one row) when every row of
    // the sector starts on a 16-byte boundary; a thread copies and splits the
    // same chunks.  A warp's chunks are 8 rows x 4 chunks.
    const bool a_vector = (t.k & 3) == 0 && (t.a & 3) == 0 && (reinterpret_cast<uintptr_t>(left) & 15) == 0;
    auto a_chunk = [&](int e, int& m, int& c) -> uint32_t {
      const int l = e & 31, w = e >> 5;
      m = (w & 15) * 8 + (l & 7);
      c = (w >> 4) * 4 + (l >> 3);
      return (static_cast<uint32_t>(c) * kTcM + m) << 4;
    };
    auto issue = [&](int64_t s) {
      const uint32_t a_hi = smem + static_cast<uint32_t>(s & 1) * kTcStageBytes;
      const uint32_t b_hi = a_hi + 2 * kTcABytes;
      const int64_t k0 = s * kTcK;
      if (a_vector) {
        for (int e = tid; e < kTcM * kTcK / 4; e += kTcThreads) {
          int m, c;
          const uint32_t off = a_chunk(e, m, c);
          const int64_t row = t.m0 + m, col = k0 + 4 * c;
          if (row < t.m && col + 4 <= t.k) {
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(a_hi + off), "l"(left + t.a + row * t.k + col)
                         : "memory");
          } else {
            for (int j = 0; j < 4; ++j) {
              const bool valid = row < t.m && col + j < t.k;
              TcCopy4(a_hi + off + 4 * j, valid ? left + t.a + row * t.k + col + j : left, valid);
            }
          }
        }
      } else {
        for (int e = tid; e < kTcM * kTcK; e += kTcThreads) {
          int m, k;
          const uint32_t off = a_position(e, m, k);
          const int64_t row = t.m0 + m, col = k0 + k;
          const bool valid = row < t.m && col < t.k;
          TcCopy4(a_hi + off, valid ? left + t.a + row * t.k + col : left, valid);
        }
      }
      for (int e = tid; e < kTcN * kTcK; e += kTcThreads) {
        int n, k;
        const uint32_t off = b_position(e, n, k);
        const int64_t row = k0 + k, col = t.n0 + n;
        const bool valid = row < t.k && col < t.n;
        TcCopy4(b_hi + off, valid ? right + t.b + row * t.n + col : right, valid);
      }
      asm volatile("cp.async.commit_group;" ::: "memory");
    };
    auto split = [&](int64_t s) {
      const uint32_t a_hi = smem + static_cast<uint32_t>(s & 1) * kTcStageBytes;
      const uint32_t a_lo = a_hi + kTcABytes, b_hi = a_lo + kTcABytes, b_lo = b_hi + kTcBBytes;
      if (a_vector) {
        for (int e = tid; e < kTcM * kTcK / 4; e += kTcThreads) {
          int m, c;
          const uint32_t off = a_chunk(e, m, c);
          float x[4];
          asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                       : "=f"(x[0]), "=f"(x[1]), "=f"(x[2]), "=f"(x[3]) : "r"(a_hi + off));
          uint32_t hi[4], lo[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            hi[j] = Tf32(x[j]);
            lo[j] = Tf32(x[j] - __uint_as_float(hi[j]));
          }
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" :: "r"(a_hi + off), "r"(hi[0]), "r"(hi[1]), "r"(hi[2]),
                       "r"(hi[3]));
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" :: "r"(a_lo + off), "r"(lo[0]), "r"(lo[1]), "r"(lo[2]),
                       "r"(lo[3]));
        }
      } else {
        for (int e = tid; e < kTcM * kTcK; e += kTcThreads) {
          int m, k;
          const uint32_t off = a_position(e, m, k);
          float x;
          asm volatile("ld.shared.f32 %0, [%1];" : "=f"(x) : "r"(a_hi + off));
          const uint32_t hi = Tf32(x), lo = Tf32(x - __uint_as_float(hi));
          asm volatile("st.shared.b32 [%0], %1;" :: "r"(a_hi + off), "r"(hi));
          asm volatile("st.shared.b32 [%0], %1;" :: "r"(a_lo + off), "r"(lo));
        }
      }
      for (int e = tid; e < kTcN * kTcK; e += kTcThreads) {
        int n, k;
        const uint32_t off = b_position(e, n, k);
        float x;
        asm volatile("ld.shared.f32 %0, [%1];" : "=f"(x) : "r"(b_hi + off));
        const uint32_t hi = Tf32(x), lo = Tf32(x - __uint_as_float(hi));
        asm volatile("st.shared.b32 [%0], %1;" :: "r"(b_hi + off), "r"(hi));
        asm volatile("st.shared.b32 [%0], %1;" :: "r"(b_lo + off), "r"(lo));
      }
    };
    if (slices > 0) issue(0);
    for (int64_t s = 0; s < slices; ++s) {
      const int buf = static_cast<int>(s & 1);
      // Slice s - 1's MMAs are done once its accumulator is drained, so its
      // stage (the one slice s + 1 uses) is free.
      if (s > 0) drain(s - 1);
      if (s + 1 < slices) {
        issue(s + 1);
        asm volatile("cp.async.wait_group 1;" ::: "memory");
      } else {
        asm volatile("cp.async.wait_group 0;" ::: "memory");
      }
      split(s);
      asm volatile("fence.proxy.async.shared::cta;");
      asm volatile("tcgen05.fence::before_thread_sync;");
      __syncthreads();
      asm volatile("tcgen05.fence::after_thread_sync;");
      if (tid == 0) {
        const uint32_t a_hi = smem + static_cast<uint32_t>(buf) * kTcStageBytes, a_lo = a_hi + kTcABytes;
        const uint32_t b_hi = a_lo + kTcABytes, b_lo = b_hi + kTcBBytes;
        const uint32_t d = tmem + static_cast<uint32_t>(buf * kTcN);
#pragma unroll
        for (int step = 0; step < kTcK / 8; ++step) {
          const uint32_t a_step = static_cast<uint32_t>(step) * 2 * kTcM * 16;
          const uint32_t b_step = static_cast<uint32_t>(step) * 2 * kTcN * 16;
          const uint64_t ah = SmemDescriptor(a_hi + a_step, kTcM * 16, 128);
          const uint64_t al = SmemDescriptor(a_lo + a_step, kTcM * 16, 128);
          const uint64_t bh = SmemDescriptor(b_hi + b_step, kTcN * 16, 128);
          const uint64_t bl = SmemDescriptor(b_lo + b_step, kTcN * 16, 128);
          MmaTf32(d, al, bh, idesc, step == 0 ? 0u : 1u);
          MmaTf32(d, ah, bl, idesc, 1u);
          MmaTf32(d, ah, bh, idesc, 1u);
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                     :: "r"(mbar0 + 8 * buf) : "memory");
      }
    }
    if (slices > 0) drain(slices - 1);
    // Epilogue: a thread writes 32 columns of row m0 + 32 (w % 4) + lane.  A wait that gave up (the
    // tensor cores never signalled) leaves NaN in the tile instead of a
    // partial sum.
    if (!ok) {
#pragma unroll
      for (int j = 0; j < 32; ++j) acc[j] = __int_as_float(0x7fc00000);
    }
    const int64_t row = t.m0 + quarter * 32 + lane;
    if (row < t.m) {
      float* dst = out + t.c + row * t.n + t.n0 + half * 32;
      const int64_t width = t.n - t.n0 - half * 32;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (j < width) dst[j] = acc[j];
      }
    }
    // Every thread's tensor-memory reads of this tile precede the next
    // tile's MMAs into the same accumulators.
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(kTcTmemColumns));
}

// ---------------------------------------------------------------------------
// Complex64 on tcgen05: the same pipeline as TcGemm with real and imaginary
// planes.  Per 8-deep step, Cr += Ar Br - Ai Bi and Ci += Ar Bi + Ai Br, each
// product as three TF32 terms (the minus by the instruction descriptor's A
// negate bit): 12 MMAs into two accumulators (re, im) per buffer.  A slice is
// 16 deep so that a stage (four A planes of 128 x 16, four B planes of
// 64 x 16) stays 48 KB.  Raw interleaved values land in the lo planes and the
// copying thread splits them into the four planes.
constexpr int kTcKc = 16;
constexpr uint32_t kTcAPlane = kTcM * kTcKc * 4;   // 8 KB
constexpr uint32_t kTcBPlane = kTcN * kTcKc * 4;   // 4 KB
static_assert(4 * kTcAPlane + 4 * kTcBPlane == kTcStageBytes, "complex stage must match the real stage size");
constexpr uint32_t kTcTmemColumnsComplex = 4 * kTcN;   // two buffers of (re, im)

__global__ void __launch_bounds__(kTcThreads, 2) TcGemmComplex(const int64_t* __restrict__ table, int64_t sectors,
                                                              int64_t tiles, const float* __restrict__ left,
                                                              const float* __restrict__ right, float* out) {
  extern __shared__ __align__(1024) unsigned char tc_smem[];
  __shared__ __align__(8) uint64_t mbar_storage[2];
  __shared__ uint32_t tmem_slot;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, half = warp >> 2;
  const uint32_t smem = static_cast<uint32_t>(__cvta_generic_to_shared(tc_smem));
  const uint32_t mbar0 = static_cast<uint32_t>(__cvta_generic_to_shared(&mbar_storage[0]));
  if (warp == 0) {
    const uint32_t slot = static_cast<uint32_t>(__cvta_generic_to_shared(&tmem_slot));
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" :: "r"(slot),
                 "r"(kTcTmemColumnsComplex));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" :: "r"(mbar0));
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" :: "r"(mbar0 + 8));
    asm volatile("fence.mbarrier_init.release.cluster;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;");
  const uint32_t tmem = tmem_slot;
  // kind::tf32, F32 accumulate, A and B K-major, N = 64, M = 128; bit 13 negates A.
  const uint32_t idesc = (1u << 4) | (2u << 7) | (2u << 10) | ((kTcN >> 3) << 17) | ((kTcM >> 4) << 24);
  const uint32_t idesc_negate = idesc | (1u << 13);
  uint32_t parity[2] = {0, 0};
  bool ok = true;
  // Planes of stage s: A re hi, re lo, im hi, im lo, then B in the same order.
  auto plane_a = [&](int64_t s, int p) { return smem + static_cast<uint32_t>(s & 1) * kTcStageBytes + p * kTcAPlane; };
  auto plane_b = [&](int64_t s, int p) {
    return smem + static_cast<uint32_t>(s & 1) * kTcStageBytes + 4 * kTcAPlane + p * kTcBPlane;
  };
  for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    const TcTask t = DecodeTcTask(table, sectors, tile);
    float acc_re[32], acc_im[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) acc_re[j] = acc_im[j] = 0.0f;
    const int64_t slices = (t.k + kTcKc - 1) / kTcKc;
    auto drain = [&](int64_t s) {
      const int buf = static_cast<int>(s & 1);
      ok = WaitPhase(mbar0 + 8 * buf, parity[buf]) && ok;
      parity[buf] ^= 1u;
      asm volatile("tcgen05.fence::after_thread_sync;");
      const uint32_t lanes = static_cast<uint32_t>(quarter * 32) << 16;
      float v[32];
      TmemLoad32(tmem + lanes + static_cast<uint32_t>(buf * 2 * kTcN + half * 32), v);
#pragma unroll
      for (int j = 0; j < 32; ++j) acc_re[j] = __fadd_rn(acc_re[j], v[j]);
      TmemLoad32(tmem + lanes + static_cast<uint32_t>(buf * 2 * kTcN + kTcN + half * 32), v);
#pragma unroll
      for (int j = 0; j < 32; ++j) acc_im[j] = __fadd_rn(acc_im[j], v[j]);
    };
    auto a_position = [&](int e, int& m, int& k) -> uint32_t {
      const int k_in = e & 3, m_lo = (e >> 2) & 7, chunk = (e >> 5) & 3, m_hi = e >> 7;
      m = m_hi * 8 + m_lo;
      k = chunk * 4 + k_in;
      return ((static_cast<uint32_t>(chunk) * kTcM + m) << 4) + (k_in << 2);
    };
    auto a_chunk = [&](int e, int& m, int& c) -> uint32_t {
      const int l = e & 31, w = e >> 5;
      m = w * 8 + (l & 7);
      c = l >> 3;
      return (static_cast<uint32_t>(c) * kTcM + m) << 4;
    };
    auto b_position = [&](int e, int& n, int& k) -> uint32_t {
      const int l = e & 31, w = e >> 5;
      const int k_in = l >> 3, chunk = w >> 3;
      n = (w & 7) * 8 + (l & 7);
      k = chunk * 4 + k_in;
      return ((static_cast<uint32_t>(chunk) * kTcN + n) << 4) + (k_in << 2);
    };
    // A moves as 32-byte chunks (four complex values of one row: two 16-byte
    // copies, parked interleaved in the two lo planes) when its rows start on
    // 16-byte boundaries; otherwise, and at the K edge, value by value into
    // the lo planes as re / im.
    const bool a_vector = (t.k & 1) == 0 && (t.a & 1) == 0 && (reinterpret_cast<uintptr_t>(left) & 15) == 0;
    auto whole_chunk = [&](int64_t row, int64_t col) { return row < t.m && col + 4 <= t.k; };
    auto issue = [&](int64_t s) {
      const uint32_t are_lo = plane_a(s, 1), aim_lo = plane_a(s, 3);
      const uint32_t bre_lo = plane_b(s, 1), bim_lo = plane_b(s, 3);
      const int64_t k0 = s * kTcKc;
      if (a_vector) {
        for (int e = tid; e < kTcM * kTcKc / 4; e += kTcThreads) {
          int m, c;
          const uint32_t off = a_chunk(e, m, c);
          const int64_t row = t.m0 + m, col = k0 + 4 * c;
          if (whole_chunk(row, col)) {
            const float* src = left + 2 * (t.a + row * t.k + col);
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(are_lo + off), "l"(src) : "memory");
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(aim_lo + off), "l"(src + 4) : "memory");
          } else {
            for (int j = 0; j < 4; ++j) {
              const bool valid = row < t.m && col + j < t.k;
              const float* src = valid ? left + 2 * (t.a + row * t.k + col + j) : left;
              TcCopy4(are_lo + off + 4 * j, src, valid);
              TcCopy4(aim_lo + off + 4 * j, valid ? src + 1 : left, valid);
            }
          }
        }
      } else {
        for (int e = tid; e < kTcM * kTcKc; e += kTcThreads) {
          int m, k;
          const uint32_t off = a_position(e, m, k);
          const int64_t row = t.m0 + m, col = k0 + k;
          const bool valid = row < t.m && col < t.k;
          const float* src = valid ? left + 2 * (t.a + row * t.k + col) : left;
          TcCopy4(are_lo + off, src, valid);
          TcCopy4(aim_lo + off, valid ? src + 1 : left, valid);
        }
      }
      for (int e = tid; e < kTcN * kTcKc; e += kTcThreads) {
        int n, k;
        const uint32_t off = b_position(e, n, k);
        const int64_t row = k0 + k, col = t.n0 + n;
        const bool valid = row < t.k && col < t.n;
        const float* src = valid ? right + 2 * (t.b + row * t.n + col) : right;
        TcCopy4(bre_lo + off, src, valid);
        TcCopy4(bim_lo + off, valid ? src + 1 : right, valid);
      }
      asm volatile("cp.async.commit_group;" ::: "memory");
    };
    // Split one complex value (read from the raw lo planes by the caller)
    // into the four planes at one 4-byte position.
    auto put = [&](uint32_t re_hi, uint32_t re_lo, uint32_t im_hi, uint32_t im_lo, uint32_t off, float re, float im) {
      const uint32_t rh = Tf32(re), rl = Tf32(re - __uint_as_float(rh));
      const uint32_t ih = Tf32(im), il = Tf32(im - __uint_as_float(ih));
      asm volatile("st.shared.b32 [%0], %1;" :: "r"(re_hi + off), "r"(rh));
      asm volatile("st.shared.b32 [%0], %1;" :: "r"(re_lo + off), "r"(rl));
      asm volatile("st.shared.b32 [%0], %1;" :: "r"(im_hi + off), "r"(ih));
      asm volatile("st.shared.b32 [%0], %1;" :: "r"(im_lo + off), "r"(il));
    };
    auto ld = [](uint32_t address) {
      float x;
      asm volatile("ld.shared.f32 %0, [%1];" : "=f"(x) : "r"(address));
      return x;
    };
    auto split = [&](int64_t s) {
      const uint32_t are_hi = plane_a(s, 0), are_lo = plane_a(s, 1), aim_hi = plane_a(s, 2), aim_lo = plane_a(s, 3);
      const uint32_t bre_hi = plane_b(s, 0), bre_lo = plane_b(s, 1), bim_hi = plane_b(s, 2), bim_lo = plane_b(s, 3);
      const int64_t k0 = s * kTcKc;
      if (a_vector) {
        for (int e = tid; e < kTcM * kTcKc / 4; e += kTcThreads) {
          int m, c;
          const uint32_t off = a_chunk(e, m, c);
          float re[4], im[4];
          if (whole_chunk(t.m0 + m, k0 + 4 * c)) {
            // Raw interleaved: (re0 im0 re1 im1) in the re lo plane, (re2 im2 re3 im3) in the im lo plane.
            re[0] = ld(are_lo + off); im[0] = ld(are_lo + off + 4); re[1] = ld(are_lo + off + 8); im[1] = ld(are_lo + off + 12);
            re[2] = ld(aim_lo + off); im[2] = ld(aim_lo + off + 4); re[3] = ld(aim_lo + off + 8); im[3] = ld(aim_lo + off + 12);
          } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              re[j] = ld(are_lo + off + 4 * j);
              im[j] = ld(aim_lo + off + 4 * j);
            }
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) put(are_hi, are_lo, aim_hi, aim_lo, off + 4 * j, re[j], im[j]);
        }
      } else {
        for (int e = tid; e < kTcM * kTcKc; e += kTcThreads) {
          int m, k;
          const uint32_t off = a_position(e, m, k);
          put(are_hi, are_lo, aim_hi, aim_lo, off, ld(are_lo + off), ld(aim_lo + off));
        }
      }
      for (int e = tid; e < kTcN * kTcKc; e += kTcThreads) {
        int n, k;
        const uint32_t off = b_position(e, n, k);
        put(bre_hi, bre_lo, bim_hi, bim_lo, off, ld(bre_lo + off), ld(bim_lo + off));
      }
    };
    if (slices > 0) issue(0);
    for (int64_t s = 0; s < slices; ++s) {
      const int buf = static_cast<int>(s & 1);
      if (s > 0) drain(s - 1);
      if (s + 1 < slices) {
        issue(s + 1);
        asm volatile("cp.async.wait_group 1;" ::: "memory");
      } else {
        asm volatile("cp.async.wait_group 0;" ::: "memory");
      }
      split(s);
      asm volatile("fence.proxy.async.shared::cta;");
      asm volatile("tcgen05.fence::before_thread_sync;");
      __syncthreads();
      asm volatile("tcgen05.fence::after_thread_sync;");
      if (tid == 0) {
        const uint32_t d_re = tmem + static_cast<uint32_t>(buf * 2 * kTcN), d_im = d_re + kTcN;
#pragma unroll
        for (int step = 0; step < kTcKc / 8; ++step) {
          const uint32_t a_step = static_cast<uint32_t>(step) * 2 * kTcM * 16;
          const uint32_t b_step = static_cast<uint32_t>(step) * 2 * kTcN * 16;
          uint64_t a[4], b[4];   // re hi, re lo, im hi, im lo
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            a[p] = SmemDescriptor(plane_a(s, p) + a_step, kTcM * 16, 128);
            b[p] = SmemDescriptor(plane_b(s, p) + b_step, kTcN * 16, 128);
          }
          const uint32_t first = step == 0 ? 0u : 1u;
          // re: Ar Br - Ai Bi
          MmaTf32(d_re, a[1], b[0], idesc, first);
          MmaTf32(d_re, a[0], b[1], idesc, 1u);
          MmaTf32(d_re, a[0], b[0], idesc, 1u);
          MmaTf32(d_re, a[3], b[2], idesc_negate, 1u);
          MmaTf32(d_re, a[2], b[3], idesc_negate, 1u);
          MmaTf32(d_re, a[2], b[2], idesc_negate, 1u);
          // im: Ar Bi + Ai Br
          MmaTf32(d_im, a[1], b[2], idesc, first);
          MmaTf32(d_im, a[0], b[3], idesc, 1u);
          MmaTf32(d_im, a[0], b[2], idesc, 1u);
          MmaTf32(d_im, a[3], b[0], idesc, 1u);
          MmaTf32(d_im, a[2], b[1], idesc, 1u);
          MmaTf32(d_im, a[2], b[0], idesc, 1u);
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                     :: "r"(mbar0 + 8 * buf) : "memory");
      }
    }
    if (slices > 0) drain(slices - 1);
    if (!ok) {
#pragma unroll
      for (int j = 0; j < 32; ++j) acc_re[j] = acc_im[j] = __int_as_float(0x7fc00000);
    }
    const int64_t row = t.m0 + quarter * 32 + lane;
    if (row < t.m) {
      float* dst = out + 2 * (t.c + row * t.n + t.n0 + half * 32);
      const int64_t width = t.n - t.n0 - half * 32;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (j < width) {
          dst[2 * j] = acc_re[j];
          dst[2 * j + 1] = acc_im[j];
        }
      }
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(kTcTmemColumnsComplex));
  }
}

int SmCountGemm() {
  static int count = [] {
    int device = 0, sms = 148;
    if (cudaGetDevice(&device) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    return sms;
  }();
  return count;
}

}  // namespace

void BuildGemmTable(int64_t sectors, const int64_t* spec, int64_t* table) {
  int64_t tiles = 0, tc_tiles = 0;
  for (int64_t s = 0; s < sectors; ++s) {
    const int64_t* in = spec + s * 6;
    int64_t* row = table + s * kGemmRow;
    for (int i = 0; i < 6; ++i) row[i] = in[i];
    row[6] = tiles;
    row[7] = tc_tiles;
    tiles += ((in[0] + kTile - 1) / kTile) * ((in[1] + kTile - 1) / kTile);
    tc_tiles += ((in[0] + kTcM - 1) / kTcM) * ((in[1] + kTcN - 1) / kTcN);
  }
}

// Bytes of one element of a GEMM operand, or 0 for an unsupported dtype.
int GemmElementBytes(int32_t dtype) {
  switch (dtype) {
    case 11: return 4;
    case 12: case 15: return 8;
    case 18: return 16;
    default: return 0;
  }
}

void SectorGemm(int32_t dtype, int64_t sectors, const int64_t* host_table, const int64_t* device_table,
                const void* left, int64_t left_size, const void* right, int64_t right_size, void* output,
                int64_t output_size, cudaStream_t stream) {
  const int eb = GemmElementBytes(dtype);
  if (eb == 0) throw InvalidArgument("sector GEMM supports only F32/F64/C64/C128");
  if (sectors < 0) throw InvalidArgument("sector count must be nonnegative");
  if (left_size < 0 || right_size < 0 || output_size < 0) throw InvalidArgument("GEMM operand sizes must be nonnegative");
  if (sectors == 0) return;
  if (host_table == nullptr || device_table == nullptr) throw InvalidArgument("GEMM table is null");
  // Every row must address inside the operands, and output blocks must not
  // overlap one another: all checks run before the launch.
  auto span = [](int64_t offset, int64_t rows, int64_t cols, int64_t size, const char* what) {
    uint64_t count = 0, end = 0;
    if (!CheckedMul(static_cast<uint64_t>(rows), static_cast<uint64_t>(cols), &count) ||
        !CheckedAdd(static_cast<uint64_t>(offset), count, &end) || (count != 0 && end > static_cast<uint64_t>(size))) {
      throw InvalidArgument(std::string("GEMM ") + what + " block lies outside its operand");
    }
    return count;
  };
  int64_t tiles = 0, tc_tiles = 0;
  std::vector<std::pair<int64_t, int64_t>> blocks;
  blocks.reserve(static_cast<std::size_t>(sectors));
  for (int64_t s = 0; s < sectors; ++s) {
    const int64_t* row = host_table + s * kGemmRow;
    for (int i = 0; i < 6; ++i) {
      if (row[i] < 0) throw InvalidArgument("GEMM sizes and offsets must be nonnegative");
    }
    if (row[0] > (int64_t{1} << 31) || row[1] > (int64_t{1} << 31) || row[2] > (int64_t{1} << 40)) {
      throw InvalidArgument("GEMM block extents are too large");
    }
    if (row[6] != tiles || row[7] != tc_tiles) {
      throw InvalidArgument("GEMM table tile prefix is inconsistent; build it with t0b_gemm_table_build");
    }
    const uint64_t c_count = span(row[5], row[0], row[1], output_size, "output");
    if (row[2] != 0) {
      span(row[3], row[0], row[2], left_size, "left");
      span(row[4], row[2], row[1], right_size, "right");
    }
    if (c_count != 0) blocks.emplace_back(row[5], row[5] + static_cast<int64_t>(c_count));
    tiles += ((row[0] + kTile - 1) / kTile) * ((row[1] + kTile - 1) / kTile);
    tc_tiles += ((row[0] + kTcM - 1) / kTcM) * ((row[1] + kTcN - 1) / kTcN);
  }
  std::sort(blocks.begin(), blocks.end());
  for (std::size_t i = 1; i < blocks.size(); ++i) {
    if (blocks[i].first < blocks[i - 1].second) throw InvalidArgument("GEMM output blocks overlap");
  }
  if (tiles == 0) return;
  if (left == nullptr || right == nullptr || output == nullptr) throw InvalidArgument("GEMM operand is null");
  // Operands are staged with element-sized asynchronous copies (16 bytes for C128).
  for (const void* buffer : {static_cast<const void*>(left), static_cast<const void*>(right),
                             static_cast<const void*>(output)}) {
    if (reinterpret_cast<uintptr_t>(buffer) % static_cast<uintptr_t>(eb) != 0) {
      throw InvalidArgument("GEMM operand buffer is not aligned to its element size");
    }
  }
  auto overlap = [](const void* a, uint64_t a_bytes, const void* b, uint64_t b_bytes) {
    if (a_bytes == 0 || b_bytes == 0) return false;
    const auto x = reinterpret_cast<uintptr_t>(a), y = reinterpret_cast<uintptr_t>(b);
    return x <= y ? y - x < a_bytes : x - y < b_bytes;
  };
  const uint64_t out_bytes = static_cast<uint64_t>(output_size) * eb;
  if (overlap(left, static_cast<uint64_t>(left_size) * eb, output, out_bytes) ||
      overlap(right, static_cast<uint64_t>(right_size) * eb, output, out_bytes)) {
    throw InvalidArgument("input and output buffers overlap");
  }
  if (overlap(device_table, static_cast<uint64_t>(sectors) * kGemmRow * sizeof(int64_t), output, out_bytes)) {
    throw InvalidArgument("device descriptor table overlaps the output");
  }
  const int64_t grid = std::min<int64_t>(tiles, int64_t{SmCountGemm()} * 4);
  switch (dtype) {
    case 12:
      DmmaGemm<false><<<static_cast<unsigned>(grid), kGemmThreads, 0, stream>>>(
          device_table, sectors, tiles, static_cast<const double*>(left), static_cast<const double*>(right),
          static_cast<double*>(output));
      break;
    case 18:
      DmmaGemm<true><<<static_cast<unsigned>(grid), kGemmThreads, 0, stream>>>(
          device_table, sectors, tiles, static_cast<const double*>(left), static_cast<const double*>(right),
          static_cast<double*>(output));
      break;
    case 11: {
      Check(cudaFuncSetAttribute(TcGemm, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem), "tcgen05 GEMM shared memory");
      const int64_t tc_grid = std::min<int64_t>(tc_tiles, int64_t{SmCountGemm()} * 2);
      TcGemm<<<static_cast<unsigned>(tc_grid), kTcThreads, kTcSmem, stream>>>(
          device_table, sectors, tc_tiles, static_cast<const float*>(left), static_cast<const float*>(right),
          static_cast<float*>(output));
      break;
    }
    case 15: {
      Check(cudaFuncSetAttribute(TcGemmComplex, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem),
            "tcgen05 GEMM shared memory");
      const int64_t tc_grid = std::min<int64_t>(tc_tiles, int64_t{SmCountGemm()} * 2);
      TcGemmComplex<<<static_cast<unsigned>(tc_grid), kTcThreads, kTcSmem, stream>>>(
          device_table, sectors, tc_tiles, static_cast<const float*>(left), static_cast<const float*>(right),
          static_cast<float*>(output));
      break;
    }
    default:
      throw InvalidArgument("sector GEMM supports only F32/F64/C64/C128");
  }
  Check(cudaGetLastError(), "sector gemm launch");
  g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
}

}  // namespace t0b
