/*
 * tensor0_b200 — C ABI of the B200 (sm_100a) block-sparse stride engine.
 *
 * Plain C: pointers, sizes and a CUDA stream.  No framework types cross this
 * boundary.  The entry points replace the CUDA execute handlers of the
 * reference's companion library (crates/tensor0-cuda12/native/cuda/*.cu) and
 * keep their calling contract:
 *
 *   - a plan ("prepared state") is built once from the same i64 layout words
 *     the reference lowers as the `layout` attribute (wire format v1,
 *     src/tensor0/_stride/_ffi/_descriptor.py:8-76) and validated with the
 *     reference's rules (crates/tensor0-py/native/layout/descriptor.cc:14-165);
 *   - the plan exposes ONE packed device descriptor table (host words); the
 *     caller owns the device copy exactly as XLA owns the reference's packed
 *     owner/fiber constant (_ffi/_calls.py:230-240);
 *   - execute calls validate every argument before any write, enqueue work on
 *     the caller's stream, never synchronize, never read device data on the
 *     host, and allocate nothing (docs/cuda.md:336-341, 365-369);
 *   - status 0 = success, 1 = invalid argument, 2 = internal error, with a
 *     message (ffi/errors.h:12-24 maps the same two classes).
 *
 * Element types use the XLA_FFI_DataType numbering so an XLA FFI adapter can
 * pass the buffer element type through unchanged.
 */
#ifndef TENSOR0_B200_H_
#define TENSOR0_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* Element types (values of XLA_FFI_DataType). */
#define T0B_S32 4
#define T0B_F32 11
#define T0B_F64 12
#define T0B_C64 15
#define T0B_C128 18

/* Plan operations (the reference's operation codes, descriptor.h:69-78). */
#define T0B_OP_COPY 0
#define T0B_OP_UPDATE 1
#define T0B_OP_DOT 2
#define T0B_OP_ACCUMULATION 3
#define T0B_OP_REDUCTION 4
#define T0B_OP_GROUPED 5

/* Plan flags. */
/* The producer guarantees that distinct records write disjoint output
 * addresses (the reference's `outputs_disjoint` attribute,
 * ffi/reduction_impl.h:193-200).  Without it the planner proves disjointness
 * itself or falls back to record-ordered execution. */
#define T0B_PLAN_OUTPUTS_DISJOINT 1u
/* Run the map engine with 64-bit in-tile offsets even when every record's
 * strides fit 32 bits (the planner selects them by itself for records whose
 * tile spans exceed 2^31 elements); results are identical. */
#define T0B_PLAN_WIDE_OFFSETS 2u
/* Accumulation and reduction plans: read the complex conjugate of every
 * source element (real storage is unaffected).  This fuses the conjugation
 * the reference applies to a source before an adjoint-destination transform
 * (operations/transforms.py:190-259: jnp.conj, then the strided accumulation)
 * into the same pass; conjugation is exact, so results are identical. */
#define T0B_PLAN_CONJUGATE_SOURCE 4u

typedef struct t0b_plan t0b_plan;

/* Library version string. */
const char* t0b_version(void);

/*
 * Build a plan from layout words.
 *   operation: T0B_OP_COPY / UPDATE / DOT / ACCUMULATION take i64 words (v1;
 *              for DOT the record's source side addresses the left operand
 *              and its destination side the right one, both only bounds-checked);
 *              T0B_OP_REDUCTION takes the reduction protocol's u64 words
 *              (little-endian bit patterns carried as i64), as the reference's
 *              Tensor0StridePrepareLayout bridge does (descriptor.cc:321-340);
 *              T0B_OP_GROUPED takes this library's grouped-transform words
 *              (see t0b_grouped_transform).
 *   coefficient_records: strictly increasing record indices that carry a
 *              coefficient (accumulation / reduction only; others factor 1),
 *              as the `coefficient_records` attribute (accumulation.cu:54-70).
 *   element_bytes: storage element size (4, 8 or 16); tiles are sized for it.
 * Replaces: Tensor0StrideCuda{Copy,Update,Accumulation,Reduction}InstantiateV1
 *   (copy.cu:52-71, update.cu:28-51, accumulation.cu:54-80, reduction.cu:54-90).
 */
int t0b_plan_create(int32_t operation, const int64_t* words, size_t word_count,
                    const int64_t* coefficient_records, size_t coefficient_count,
                    int32_t element_bytes, uint32_t flags, t0b_plan** plan,
                    char* error, size_t error_size);
void t0b_plan_destroy(t0b_plan* plan);

/* Packed device descriptor table: host words the caller copies to device
 * memory it owns, then passes to every execute call.  16-byte aligned. */
const int64_t* t0b_plan_table(const t0b_plan* plan, size_t* word_count);

/* Scratch elements (of the storage type) one batch needs; 0 if none.
 * The reference sizes its XLA-owned second result the same way
 * (accumulation.cu:191-206, layout/owner_fiber.h:27-39). */
uint64_t t0b_plan_scratch_elements(const t0b_plan* plan);

/* Plan statistics: sizes, record count, engine kernels per call. */
typedef struct {
  uint64_t source_size;
  uint64_t output_size;
  uint64_t records;
  uint64_t tiles;
  uint64_t kernels_per_call;
  uint64_t full_coverage;     /* 1: every output element is written once, no zeroing pass */
  uint64_t bytes_moved;       /* algorithmic bytes of one batch */
} t0b_plan_info;
void t0b_plan_query(const t0b_plan* plan, t0b_plan_info* info);

/* Prepared-state counters (the reference exports the same per handler,
 * copy.cu:130-152). */
uint64_t t0b_plan_created_count(void);
uint64_t t0b_plan_destroyed_count(void);

/*
 * Storage buffers (source, output, base) must be aligned to their element
 * size (4, 8, 8 and 16 bytes for F32, F64, C64 and C128); execute calls reject
 * others with status 1.
 *
 * Copy: out[b, dst(i)] = src[b, src(i)], bit-preserving; outputs no record
 * writes are zero.  Replaces Tensor0StrideCudaCopy{F32,F64,C64,C128}V1
 * (copy.cu:73-126).  source [batches, source_size], output [batches, output_size].
 */
int t0b_copy(const t0b_plan* plan, int32_t dtype, const void* source, void* output,
             int64_t batches, const int64_t* device_table, void* stream,
             char* error, size_t error_size);

/*
 * Accumulation: out = 0; for each record in order out[dst] += c_r * src[src],
 * c_r = coefficients[slot(r) * coefficient_count + (coefficient_count == 1 ? 0 : b)]
 * for records listed in coefficient_records, 1 otherwise; a zero coefficient
 * skips its record, a unit one skips the multiply.  Coefficients are a device
 * array of dtype S32, the storage's real type or (complex storage) its complex
 * type.  Replaces Tensor0StrideCudaAccumulation*V1 (accumulation.cu:92-163).
 * scratch: device buffer of batches * t0b_plan_scratch_elements() elements
 * (may be NULL when that is 0).
 */
int t0b_accumulation(const t0b_plan* plan, int32_t dtype, const void* source, void* output,
                     int64_t batches, const void* coefficients, int32_t coefficient_dtype,
                     int64_t coefficient_count, void* scratch, const int64_t* device_table,
                     void* stream, char* error, size_t error_size);

/*
 * Reduction (strided partial trace): out = 0; per record, per output owner,
 * out[owner] += c_r * sum over the record's reduction axes of src.
 * Same coefficient and scratch rules as t0b_accumulation.
 * Replaces Tensor0StrideCudaReduction*V1 (reduction.cu:92-190).
 */
int t0b_reduction(const t0b_plan* plan, int32_t dtype, const void* source, void* output,
                  int64_t batches, const void* coefficients, int32_t coefficient_dtype,
                  int64_t coefficient_count, void* scratch, const int64_t* device_table,
                  void* stream, char* error, size_t error_size);

/*
 * t0b_reduction without a scratch argument, for callers that cannot allocate
 * device memory (no counterpart in the reference: its reductions receive
 * XLA-owned scratch).  An XLA FFI handler may not allocate (XLA owns every
 * buffer), and an application whose device memory is fully reserved by its own
 * pool cannot call cudaMalloc; both still pass inputs, output, coefficients
 * and the device table, and the reduce engine's partials go to a 16 MiB array
 * compiled into this library (held by every GPU that loads it until exit).
 * Calls needing more than 16 MiB of scratch (batches * scratch elements *
 * element size) are rejected with status 1.  The first call on a device looks
 * up the array's device address with that device current; make that first
 * call before any stream capture.  The address is looked up again whenever
 * the current CUDA context differs from the one it was found in; a primary
 * context recreated by cudaDeviceReset may return under the same handle, so a
 * device reset after the first call is not supported.  Every call shares the one array per device:
 * calls that overlap on the GPU (different streams, no ordering) race.  The
 * kernels write every partial they read, so nothing needs clearing between
 * calls.  Allocates nothing.
 */
int t0b_reduction_static_scratch(const t0b_plan* plan, int32_t dtype, const void* source, void* output,
                                 int64_t batches, const void* coefficients, int32_t coefficient_dtype,
                                 int64_t coefficient_count, const int64_t* device_table, void* stream,
                                 char* error, size_t error_size);

/*
 * Update (the fused add_transform): out = base; at each selected address
 * out[dst] = alpha * src[src] + beta * base[dst], with the reference's zero
 * and one short-circuits (map_reduce_policies.cuh:30-69).  output may alias
 * base.  alpha / beta are device arrays of 1 or `batches` values (count) of
 * dtype S32, real or complex of the storage precision.
 * Replaces Tensor0StrideCudaUpdate*V1 (update.cu:94-190).
 */
int t0b_update(const t0b_plan* plan, int32_t dtype, const void* source, const void* base,
               void* output, int64_t batches, const void* alpha, int32_t alpha_dtype,
               int64_t alpha_count, const void* beta, int32_t beta_dtype, int64_t beta_count,
               const int64_t* device_table, void* stream, char* error, size_t error_size);

/*
 * Dot (the reference's dot_p): out[b] = sum over every record and element of
 * conj?(left[b, src(i)]) * right[b, dst(i)], conjugating the left factor when
 * conjugate_left is 1 (complex storage).  left [batches, source_size], right
 * [batches, output_size], output [batches].  scratch: batches *
 * t0b_plan_scratch_elements() elements of the storage type for the partial
 * sums (XLA-owned in the reference, dot.cu:123-160), 16-byte aligned.  At most
 * 65535 batches.
 * Replaces Tensor0StrideCudaDot{F32,F64,C64,C128}V1 (dot.cu:97-160).
 */
int t0b_dot(const t0b_plan* plan, int32_t dtype, const void* left, const void* right, void* output,
            int64_t batches, int32_t conjugate_left, void* scratch, const int64_t* device_table,
            void* stream, char* error, size_t error_size);

/*
 * Grouped transform (the non-abelian permute's multi-tree groups): for each
 * group, destination block j = sum_i M[j][i] * source block i, elementwise over
 * one logical block shape; 1 x 1 groups follow the direct accumulation rule
 * (0 writes +0, 1 copies, others scale).  Output elements no destination
 * covers are zero.  The plan (T0B_OP_GROUPED, no coefficient records, no flags)
 * takes the words
 *   [1, source_size, output_size, groups,
 *    per group: rank, n_src, n_dst, shape[rank],
 *               n_src x (offset, strides[rank]),   (source strides in the shape's axis order)
 *               n_dst x (offset, strides[rank])]
 * with every address in bounds, each destination injective and all
 * destinations pairwise disjoint.  matrices: t0b_plan_matrix_elements()
 * values, each group's row-major [n_dst][n_src] matrix in group order, of the
 * storage's real type or (complex storage) its complex type.
 * source [batches, source_size], output [batches, output_size].
 * Replaces the pack (copy_p) -> small dense matmul -> unpack (update_p /
 * copy_p) sequence of _strided_grouped_transform (_stride/_tensor_ops.py:119-203).
 */
int t0b_grouped_transform(const t0b_plan* plan, int32_t dtype, const void* source, void* output,
                          int64_t batches, const void* matrices, int32_t matrix_dtype,
                          const int64_t* device_table, void* stream, char* error, size_t error_size);

/* Matrix elements a grouped plan's execute call reads; 0 for other plans. */
uint64_t t0b_plan_matrix_elements(const t0b_plan* plan);

/*
 * TensorMap.add: out[i] = alpha * x[i] + beta * y[i] over n elements, with
 * host scalars (tensor/tensor_map.py:434-455).  Real alpha/beta on complex
 * data scale both components.  alpha_imag / beta_imag are ignored for real
 * storage.
 */
int t0b_axpby(int32_t dtype, int64_t n, double alpha_real, double alpha_imag, const void* x,
              double beta_real, double beta_imag, const void* y, void* output, void* stream,
              char* error, size_t error_size);

/*
 * Grouped per-sector GEMM behind block-sparse contraction
 * (tensor/linalg.py:533-566): for each sector g, C_g = A_g @ B_g with
 * row-major A_g [m_g x k_g] at left + a_offset_g, B_g [k_g x n_g] at
 * right + b_offset_g and C_g [m_g x n_g] at output + c_offset_g (element
 * offsets).  Sectors absent from either operand are zero in the output
 * (pack_blocks, tensor/_blocks.py:83-131): the caller lists them with k = 0.
 * host_table / device_table: `sectors` rows of t0b_gemm_table_words(1) int64
 * words, built on the host by t0b_gemm_table_build from rows of 6 words
 * {m, n, k, a_off, b_off, c_off}; the caller copies the host words to device
 * memory it owns.  left_size / right_size / output_size are the operands'
 * lengths in elements: every row must address inside them, output blocks
 * must be pairwise disjoint, the output must not overlap either input, and
 * the operands must be aligned to their element size (16 bytes for C128);
 * otherwise status 1 and nothing is launched.  F64 and C128 run on the FP64
 * tensor cores (DMMA); F32 and C64 run on the tcgen05 tensor cores
 * (kind::tf32, three-term split, each K slice summed into FP32 registers;
 * C64 as four real products).
 */
size_t t0b_gemm_table_words(int64_t sectors);
int t0b_gemm_table_build(int64_t sectors, const int64_t* spec, int64_t* table, char* error,
                         size_t error_size);
int t0b_sector_gemm(int32_t dtype, int64_t sectors, const int64_t* host_table,
                    const int64_t* device_table, const void* left, int64_t left_size,
                    const void* right, int64_t right_size, void* output, int64_t output_size,
                    void* stream, char* error, size_t error_size);

/* Number of kernels this library launched since load (for launch accounting). */
uint64_t t0b_kernel_launches(void);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* TENSOR0_B200_H_ */
