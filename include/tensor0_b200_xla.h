/*
 * XLA FFI handler library (libtensor0_b200_xla.so) over the engine's C ABI.
 *
 * The symbol table of the reference's CUDA companion library, which its
 * Python extension resolves with dlsym (crates/tensor0-py/src/stride.rs:284-330)
 * and registers with JAX (src/tensor0/_stride/_ffi/_registration.py:57-242):
 *   *InstantiateV1Handler      XLA_FFI_Handler* of the instantiate stage
 *                              (copy.cu:154-156, update.cu:198-200, dot.cu:123-127,
 *                              accumulation.cu:191-195, reduction.cu:199-203)
 *   *{F32,F64,C64,C128}V1Handler XLA_FFI_Handler* of the execute stage
 *                              (copy.cu:158-167, update.cu:202-212, dot.cu:129-160,
 *                              accumulation.cu:197-206, reduction.cu:205-215)
 *   *PreparedTypeId            XLA_FFI_TypeId* of the prepared state, filled in
 *                              by the registration (jax.ffi.register_ffi_type)
 *   *PreparedTypeInfo          XLA_FFI_TypeInfo* (the state's deleter)
 *   *Prepared{Created,Destroyed}Count  prepared states made / deleted
 *                              (copy.cu:130-152)
 *
 * Execute operands as the reference's, except that the descriptor operand is
 * the engine's packed table (t0b_plan_table of a plan over the same words and
 * element size) and the scratch result is [batch, t0b_plan_scratch_elements].
 * Coefficient operands (accumulation, reduction) are one buffer per
 * coefficient record; they are gathered into a 32 MiB table inside the
 * library, so calls allocate nothing and never synchronize.
 */
#ifndef TENSOR0_B200_XLA_H_
#define TENSOR0_B200_XLA_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Copy */
void* Tensor0StrideCudaCopyInstantiateV1Handler(void);
void* Tensor0StrideCudaCopyF32V1Handler(void);
void* Tensor0StrideCudaCopyF64V1Handler(void);
void* Tensor0StrideCudaCopyC64V1Handler(void);
void* Tensor0StrideCudaCopyC128V1Handler(void);
void* Tensor0StrideCudaCopyPreparedTypeId(void);
const void* Tensor0StrideCudaCopyPreparedTypeInfo(void);
uint64_t Tensor0StrideCudaCopyPreparedCreatedCount(void);
uint64_t Tensor0StrideCudaCopyPreparedDestroyedCount(void);

/* Update */
void* Tensor0StrideCudaUpdateInstantiateV1Handler(void);
void* Tensor0StrideCudaUpdateF32V1Handler(void);
void* Tensor0StrideCudaUpdateF64V1Handler(void);
void* Tensor0StrideCudaUpdateC64V1Handler(void);
void* Tensor0StrideCudaUpdateC128V1Handler(void);
void* Tensor0StrideCudaUpdatePreparedTypeId(void);
const void* Tensor0StrideCudaUpdatePreparedTypeInfo(void);
uint64_t Tensor0StrideCudaUpdatePreparedCreatedCount(void);
uint64_t Tensor0StrideCudaUpdatePreparedDestroyedCount(void);

/* Dot */
void* Tensor0StrideCudaDotInstantiateV1Handler(void);
void* Tensor0StrideCudaDotF32V1Handler(void);
void* Tensor0StrideCudaDotF64V1Handler(void);
void* Tensor0StrideCudaDotC64V1Handler(void);
void* Tensor0StrideCudaDotC128V1Handler(void);
void* Tensor0StrideCudaDotPreparedTypeId(void);
const void* Tensor0StrideCudaDotPreparedTypeInfo(void);
uint64_t Tensor0StrideCudaDotPreparedCreatedCount(void);
uint64_t Tensor0StrideCudaDotPreparedDestroyedCount(void);

/* Accumulation */
void* Tensor0StrideCudaAccumulationInstantiateV1Handler(void);
void* Tensor0StrideCudaAccumulationF32V1Handler(void);
void* Tensor0StrideCudaAccumulationF64V1Handler(void);
void* Tensor0StrideCudaAccumulationC64V1Handler(void);
void* Tensor0StrideCudaAccumulationC128V1Handler(void);
void* Tensor0StrideCudaAccumulationPreparedTypeId(void);
const void* Tensor0StrideCudaAccumulationPreparedTypeInfo(void);
uint64_t Tensor0StrideCudaAccumulationPreparedCreatedCount(void);
uint64_t Tensor0StrideCudaAccumulationPreparedDestroyedCount(void);

/* Reduction */
void* Tensor0StrideCudaReductionInstantiateV1Handler(void);
void* Tensor0StrideCudaReductionF32V1Handler(void);
void* Tensor0StrideCudaReductionF64V1Handler(void);
void* Tensor0StrideCudaReductionC64V1Handler(void);
void* Tensor0StrideCudaReductionC128V1Handler(void);
void* Tensor0StrideCudaReductionPreparedTypeId(void);
const void* Tensor0StrideCudaReductionPreparedTypeInfo(void);
uint64_t Tensor0StrideCudaReductionPreparedCreatedCount(void);
uint64_t Tensor0StrideCudaReductionPreparedDestroyedCount(void);
#ifdef __cplusplus
}
#endif

#endif  /* TENSOR0_B200_XLA_H_ */
