/*
 * chelis_host_runtime.h -- the part of the Chelis host runtime that the
 * device owner and the generated host-array entries touch.
 *
 * Generated Chelis code and the reference's device owner
 * (crates/chelis-backend-hip/runtime/chelis_device_owner.cpp) talk to the
 * Rust runtime (crates/chelis-runtime, header
 * crates/chelis-runtime/include/chelis_runtime.h) through these functions:
 * tagged scalars, the metadata plan (shape / stride / byte arithmetic) and
 * host tensors with read views and write guards.
 *
 * libchelis_cuda exports every function below as a WEAK definition, so the
 * library links and runs alone (tests, a C host without the Rust runtime).
 * A process that links the real Chelis runtime resolves these names to the
 * runtime's own definitions instead (the executable's symbols come first in
 * the dynamic linker's search order), and the library then uses the
 * runtime's plans and tensors.  The stand-ins keep the runtime's checks and
 * failure behaviour: a metadata error prints the runtime's
 * "numeric trap: <kind> in metadata_plan at i64" line and exits with status
 * 1 (chelis_runtime.h:78-82, 127-130).
 *
 * When the real chelis_runtime.h is included first, its declarations are
 * used and this header adds nothing.
 */
#ifndef CHELIS_HOST_RUNTIME_H
#define CHELIS_HOST_RUNTIME_H

#include <stdint.h>

#include "chelis_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

#ifndef CHELIS_RUNTIME_H
/* chelis_runtime.h:18-19, 26 */
typedef struct chelis_tensor chelis_tensor;
typedef struct chelis_tensor_write chelis_tensor_write;
typedef struct { chelis_dtype dtype; uint8_t reserved[7]; uint64_t bits; } chelis_scalar;
/* chelis_runtime_views.h:7-18 */
typedef struct {
    const void *data;
    int64_t count;
    chelis_dtype dtype;
    uint8_t reserved[7];
} chelis_read_view;
typedef struct {
    void *data;
    int64_t count;
    chelis_dtype dtype;
    uint8_t reserved[7];
} chelis_write_view;
/* chelis_runtime.h:367 */
typedef struct chelis_metadata_plan chelis_metadata_plan;

/* chelis_runtime.h:328 (lib.rs:2583): a tagged scalar from raw bits. */
chelis_scalar chelis_scalar_from_bits(chelis_dtype dtype, uint64_t bits);
/* chelis_runtime.h:56: element width of a dtype id (0 for an unknown id). */
int64_t chelis_dtype_size(chelis_dtype dtype);

/* Metadata plan, chelis_runtime.h:368-378 (lib.rs:3022-3138).  `rank`,
 * shape and stride entries and byte counts are tagged i64 scalars; the
 * exemplar carries only the element dtype (reserved bytes zero).  _new is a
 * contiguous row-major plan; _view a forward strided view (non-negative
 * strides) whose reachable span must fit `byte_capacity`. */
chelis_metadata_plan *chelis_metadata_plan_new(chelis_scalar rank, const chelis_scalar *shape,
                                               chelis_scalar exemplar);
chelis_metadata_plan *chelis_metadata_plan_view(chelis_scalar rank, const chelis_scalar *shape,
                                                const chelis_scalar *strides,
                                                chelis_scalar exemplar,
                                                chelis_scalar byte_capacity);
int32_t chelis_metadata_plan_rank(const chelis_metadata_plan *plan);
const int64_t *chelis_metadata_plan_shape(const chelis_metadata_plan *plan);   /* NULL at rank 0 */
const int64_t *chelis_metadata_plan_strides(const chelis_metadata_plan *plan); /* NULL at rank 0 */
int64_t chelis_metadata_plan_count(const chelis_metadata_plan *plan);
int64_t chelis_metadata_plan_byte_count(const chelis_metadata_plan *plan);
int64_t chelis_metadata_plan_byte_offset(const chelis_metadata_plan *plan,
                                         chelis_scalar linear_index);
chelis_dtype chelis_metadata_plan_dtype(const chelis_metadata_plan *plan);
void chelis_metadata_plan_check_capacity(const chelis_metadata_plan *plan,
                                         chelis_scalar byte_capacity);
void chelis_metadata_plan_release(chelis_metadata_plan *plan);

/* Host tensors, chelis_runtime.h:38-49, 350-354 (lib.rs:2155-2534): runtime-owned
 * (zero-filled, 32-byte aligned) or borrowed storage, reference counted.
 * A write guard gives the one owner a writable view until end_write. */
chelis_tensor *chelis_alloc(int32_t rank, const int64_t *shape, chelis_dtype dtype);
chelis_tensor *chelis_tensor_entry_borrow(int32_t rank, const int64_t *shape, chelis_dtype dtype,
                                          const void *data, int64_t byte_capacity);
void chelis_tensor_retain(const chelis_tensor *tensor);
void chelis_tensor_release(const chelis_tensor *tensor);
chelis_read_view chelis_tensor_read_view(const chelis_tensor *tensor);
chelis_tensor_write *chelis_tensor_begin_write(chelis_tensor *tensor);
chelis_write_view chelis_tensor_write_view(const chelis_tensor_write *guard);
void chelis_tensor_end_write(chelis_tensor_write *guard);
int32_t chelis_tensor_rank(const chelis_tensor *tensor);
int64_t chelis_tensor_shape(const chelis_tensor *tensor, int32_t axis);
int64_t chelis_tensor_numel(const chelis_tensor *tensor);
int64_t chelis_tensor_byte_count(const chelis_tensor *tensor);
#endif /* CHELIS_RUNTIME_H */

/* =========================================================================
 * Device owner under the reference's names and argument types
 * crates/chelis-backend-hip/runtime/chelis_device_owner.h:16-24
 * (implementation chelis_device_owner.cpp:184-274).
 *
 * alloc and borrow take over `plan` (it is released, also on failure).
 * alloc: owned, zero-filled storage of the plan's byte count on the current
 * device.  borrow: `data` must be device memory of the current device,
 * aligned to the element width, with `byte_capacity` (tagged i64) covering
 * the plan's reach.  copy_from_host: the destination must own canonical
 * row-major storage and match the host tensor's count and dtype.
 * copy_to_host: any source layout (strided sources are gathered on the
 * device first), into a host write guard of equal count and dtype.
 * Each returns with its device work complete.
 *
 * Errors as in the reference: argument and metadata errors print
 * "numeric trap: domain in metadata_plan at i64" and exit(1); CUDA failures
 * print "CUDA device owner failure: ..." and abort().  The `_status` forms
 * return CHELIS_CUDA_OK or a CHELIS_CUDA_ERR_* code instead (message in
 * chelis_cuda_last_error()) and write the owner through `out`.
 * ========================================================================= */
chelis_device_tensor_owner *chelis_device_tensor_alloc(chelis_metadata_plan *plan);
chelis_device_tensor_owner *chelis_device_tensor_borrow(chelis_metadata_plan *plan, void *data,
                                                        chelis_scalar byte_capacity);
void chelis_device_tensor_copy_from_host(chelis_device_tensor_owner *destination,
                                         const chelis_tensor *source);
void chelis_device_tensor_copy_to_host(chelis_tensor_write *destination,
                                       const chelis_device_tensor_owner *source);
int chelis_device_tensor_alloc_status(chelis_metadata_plan *plan,
                                      chelis_device_tensor_owner **out);
int chelis_device_tensor_borrow_status(chelis_metadata_plan *plan, void *data,
                                       chelis_scalar byte_capacity,
                                       chelis_device_tensor_owner **out);
int chelis_device_tensor_copy_from_host_status(chelis_device_tensor_owner *destination,
                                               const chelis_tensor *source);
int chelis_device_tensor_copy_to_host_status(chelis_tensor_write *destination,
                                             const chelis_device_tensor_owner *source);

/* =========================================================================
 * Generated-entry host-array ABI of the shipped programs
 * `extern "C" void f(chelis_tensor **inputs, int n_in, chelis_tensor
 * **outputs, int n_out)` (crates/chelis-backend-hip/src/emit.rs:660-800,
 * header string src/lib.rs:117).  Inputs are borrowed host tensors; each
 * output is a new runtime-owned host tensor (chelis_alloc) that the caller
 * releases.  The program is the one of the matching `*_device` entry in
 * chelis_cuda.h (same inputs, outputs and constants).
 * A wrong input or output count prints "<f>: expected N inputs, got M" and
 * aborts (emit.rs:677-693); an input of the wrong dtype is
 * "numeric trap: domain in load at i64" (emit.rs:1112) and exits 1; other
 * failures as the owner's.  `f_status` returns a code instead and leaves
 * the outputs NULL on failure.
 * ========================================================================= */
void chelis_chain_fwd(chelis_tensor **inputs, int n_in, chelis_tensor **outputs, int n_out);
void chelis_chain_grad(chelis_tensor **inputs, int n_in, chelis_tensor **outputs, int n_out);
void chelis_portfolio(chelis_tensor **inputs, int n_in, chelis_tensor **outputs, int n_out);
void chelis_matmul(chelis_tensor **inputs, int n_in, chelis_tensor **outputs, int n_out);
int chelis_chain_fwd_status(chelis_tensor **inputs, int n_in, chelis_tensor **outputs, int n_out);
int chelis_chain_grad_status(chelis_tensor **inputs, int n_in, chelis_tensor **outputs, int n_out);
int chelis_portfolio_status(chelis_tensor **inputs, int n_in, chelis_tensor **outputs, int n_out);
int chelis_matmul_status(chelis_tensor **inputs, int n_in, chelis_tensor **outputs, int n_out);

#ifdef __cplusplus
}
#endif
#endif /* CHELIS_HOST_RUNTIME_H */
