/*
 * A C host written against the reference's runtime and device-owner
 * interfaces (chelis_runtime.h, chelis_device_owner.h), linked against
 * libchelis_cuda alone.  It runs the call sequence generated Chelis code
 * runs (crates/chelis-backend-hip/src/emit.rs:660-800, 3120-3200): metadata
 * plans, owned and borrowed device tensors, host tensors with write guards,
 * host <-> device copies, a program through the host-array entry.
 *
 *   owner_abi plan      metadata-plan and host-tensor arithmetic (no GPU)
 *   owner_abi trap-rank a negative plan rank: must print the runtime's
 *                       trap line and exit 1 (no GPU)
 *   owner_abi trap-view a view whose reach exceeds its capacity (no GPU)
 *   owner_abi status    _status forms report errors as codes (no GPU)
 *   owner_abi gpu       device owner round trip and chelis_matmul (GPU)
 */
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "chelis_host_runtime.h"

static chelis_scalar i64(int64_t v) { return chelis_scalar_from_bits(CHELIS_DTYPE_I64, (uint64_t)v); }
static chelis_scalar exemplar(chelis_dtype dt) { return chelis_scalar_from_bits(dt, 0); }

#define CHECK(cond)                                                            \
    do {                                                                       \
        if (!(cond)) {                                                         \
            fprintf(stderr, "check failed at line %d: %s\n", __LINE__, #cond); \
            return 1;                                                          \
        }                                                                      \
    } while (0)

static int plan_case(void) {
    chelis_scalar shape[3] = {i64(2), i64(3), i64(4)};
    chelis_metadata_plan *p = chelis_metadata_plan_new(i64(3), shape, exemplar(CHELIS_DTYPE_F64));
    CHECK(chelis_metadata_plan_rank(p) == 3);
    CHECK(chelis_metadata_plan_count(p) == 24);
    CHECK(chelis_metadata_plan_byte_count(p) == 192);
    CHECK(chelis_metadata_plan_dtype(p) == CHELIS_DTYPE_F64);
    const int64_t *st = chelis_metadata_plan_strides(p);
    CHECK(st[0] == 12 && st[1] == 4 && st[2] == 1);
    CHECK(chelis_metadata_plan_byte_offset(p, i64(23)) == 184);
    chelis_metadata_plan_check_capacity(p, i64(192));
    chelis_metadata_plan_release(p);

    /* a transposed view of a 3 x 5 f32 matrix: shape [5, 3], strides [1, 5] */
    chelis_scalar vshape[2] = {i64(5), i64(3)}, vstrides[2] = {i64(1), i64(5)};
    p = chelis_metadata_plan_view(i64(2), vshape, vstrides, exemplar(CHELIS_DTYPE_F32), i64(60));
    CHECK(chelis_metadata_plan_count(p) == 15);
    CHECK(chelis_metadata_plan_byte_offset(p, i64(1)) == 20);  /* (0, 1) -> element 5 */
    CHECK(chelis_metadata_plan_byte_offset(p, i64(3)) == 4);   /* (1, 0) -> element 1 */
    chelis_metadata_plan_release(p);

    /* rank 0 and an empty extent */
    p = chelis_metadata_plan_new(i64(0), NULL, exemplar(CHELIS_DTYPE_I32));
    CHECK(chelis_metadata_plan_count(p) == 1 && chelis_metadata_plan_shape(p) == NULL);
    chelis_metadata_plan_release(p);
    chelis_scalar zshape[2] = {i64(0), i64(7)};
    p = chelis_metadata_plan_new(i64(2), zshape, exemplar(CHELIS_DTYPE_F32));
    CHECK(chelis_metadata_plan_count(p) == 0 && chelis_metadata_plan_byte_count(p) == 0);
    chelis_metadata_plan_release(p);

    /* host tensors and the write guard */
    int64_t dims[2] = {2, 3};
    chelis_tensor *t = chelis_alloc(2, dims, CHELIS_DTYPE_F32);
    CHECK(chelis_tensor_rank(t) == 2 && chelis_tensor_shape(t, 1) == 3);
    CHECK(chelis_tensor_numel(t) == 6 && chelis_tensor_byte_count(t) == 24);
    chelis_tensor_write *g = chelis_tensor_begin_write(t);
    chelis_write_view w = chelis_tensor_write_view(g);
    CHECK(w.count == 6 && w.dtype == CHELIS_DTYPE_F32);
    for (int i = 0; i < 6; ++i) ((float *)w.data)[i] = (float)i;
    chelis_tensor_end_write(g);
    chelis_read_view r = chelis_tensor_read_view(t);
    CHECK(((const float *)r.data)[5] == 5.0f);
    chelis_tensor_retain(t);
    chelis_tensor_release(t);
    chelis_tensor_release(t);
    float raw[4] = {1, 2, 3, 4};
    int64_t bdims[1] = {4};
    t = chelis_tensor_entry_borrow(1, bdims, CHELIS_DTYPE_F32, raw, sizeof(raw));
    r = chelis_tensor_read_view(t);
    CHECK(r.data == raw && r.count == 4);
    chelis_tensor_release(t);
    printf("plan ok\n");
    return 0;
}

static int status_case(void) {
    /* the _status forms refuse a missing plan or owner with a code */
    chelis_device_tensor_owner *o = (chelis_device_tensor_owner *)1;
    CHECK(chelis_device_tensor_alloc_status(NULL, &o) == CHELIS_CUDA_ERR_DOMAIN && o == NULL);
    CHECK(strstr(chelis_cuda_last_error(), "numeric trap: domain in metadata_plan at i64") != NULL);
    CHECK(chelis_device_tensor_copy_from_host_status(NULL, NULL) != CHELIS_CUDA_OK);
    chelis_tensor *outs[1] = {NULL};
    CHECK(chelis_matmul_status(NULL, 2, outs, 1) == CHELIS_CUDA_ERR_DOMAIN);
    CHECK(chelis_matmul_status(NULL, 3, outs, 1) == CHELIS_CUDA_ERR_DOMAIN);
    printf("status ok\n");
    return 0;
}

static int gpu_case(void) {
    CHECK(chelis_cuda_init(0) == CHELIS_CUDA_OK);
    const int64_t m = 96, k = 80, n = 112;
    /* owned device tensor from a plan, filled from a host tensor */
    chelis_scalar ashape[2] = {i64(m), i64(k)};
    chelis_device_tensor_owner *da =
        chelis_device_tensor_alloc(chelis_metadata_plan_new(i64(2), ashape, exemplar(CHELIS_DTYPE_F64)));
    const chelis_gpu_tensor *va = chelis_device_tensor_view(da);
    CHECK(va->count == m * k && va->ownership == 1 && va->strides[0] == k);
    int64_t adims[2] = {m, k}, bdims[2] = {k, n};
    chelis_tensor *ha = chelis_alloc(2, adims, CHELIS_DTYPE_F64);
    chelis_tensor *hb = chelis_alloc(2, bdims, CHELIS_DTYPE_F64);
    chelis_tensor_write *g = chelis_tensor_begin_write(ha);
    double *A = (double *)chelis_tensor_write_view(g).data;
    for (int64_t i = 0; i < m * k; ++i) A[i] = sin(0.37 * (double)i);
    chelis_tensor_end_write(g);
    g = chelis_tensor_begin_write(hb);
    double *B = (double *)chelis_tensor_write_view(g).data;
    for (int64_t i = 0; i < k * n; ++i) B[i] = cos(0.11 * (double)i);
    chelis_tensor_end_write(g);
    chelis_device_tensor_copy_from_host(da, ha);

    /* a borrowed view of the same storage, transposed, copied back to the host */
    chelis_scalar tshape[2] = {i64(k), i64(m)}, tstrides[2] = {i64(1), i64(k)};
    chelis_device_tensor_owner *dt = chelis_device_tensor_borrow(
        chelis_metadata_plan_view(i64(2), tshape, tstrides, exemplar(CHELIS_DTYPE_F64), i64(m * k * 8)),
        va->data, i64(m * k * 8));
    CHECK(chelis_device_tensor_view(dt)->ownership == 0);
    int64_t tdims[2] = {k, m};
    chelis_tensor *ht = chelis_alloc(2, tdims, CHELIS_DTYPE_F64);
    g = chelis_tensor_begin_write(ht);
    chelis_device_tensor_copy_to_host(g, dt);
    const double *T = (const double *)chelis_tensor_write_view(g).data;
    for (int64_t i = 0; i < k; ++i)
        for (int64_t j = 0; j < m; ++j) CHECK(T[i * m + j] == A[j * k + i]);
    chelis_tensor_end_write(g);

    /* the host-array program entry */
    chelis_tensor *ins[2] = {ha, hb}, *outs[1] = {NULL};
    chelis_matmul(ins, 2, outs, 1);
    CHECK(outs[0] != NULL && chelis_tensor_rank(outs[0]) == 2 && chelis_tensor_shape(outs[0], 1) == n);
    const double *C = (const double *)chelis_tensor_read_view(outs[0]).data;
    double worst = 0.0;
    for (int64_t i = 0; i < m; ++i)
        for (int64_t j = 0; j < n; ++j) {
            double ref = 0.0, mag = 0.0;
            for (int64_t q = 0; q < k; ++q) {
                ref += A[i * k + q] * B[q * n + j];
                mag += fabs(A[i * k + q] * B[q * n + j]);
            }
            const double e = fabs(C[i * n + j] - ref) / (mag > 0 ? mag : 1.0);
            if (e > worst) worst = e;
        }
    CHECK(worst <= 1e-12);
    /* the same through the _status form, twice (outputs are fresh tensors) */
    chelis_tensor *outs2[1] = {NULL};
    CHECK(chelis_matmul_status(ins, 2, outs2, 1) == CHELIS_CUDA_OK);
    CHECK(memcmp(chelis_tensor_read_view(outs2[0]).data, C, (size_t)(m * n * 8)) == 0);
    /* a wrong dtype is refused with the load trap's wording */
    chelis_tensor *hf = chelis_alloc(2, adims, CHELIS_DTYPE_F32);
    chelis_tensor *bad[2] = {hf, hb}, *outs3[1] = {NULL};
    CHECK(chelis_matmul_status(bad, 2, outs3, 1) == CHELIS_CUDA_ERR_DOMAIN && outs3[0] == NULL);
    CHECK(strstr(chelis_cuda_last_error(), "numeric trap: domain in load at i64") != NULL);

    chelis_tensor_release(hf);
    chelis_tensor_release(outs2[0]);
    chelis_tensor_release(outs[0]);
    chelis_tensor_release(ht);
    chelis_tensor_release(ha);
    chelis_tensor_release(hb);
    chelis_device_tensor_release(dt);
    chelis_device_tensor_release(da);
    CHECK(chelis_cuda_shutdown() == CHELIS_CUDA_OK);
    printf("gpu ok (max rel err %.3g)\n", worst);
    return 0;
}

int main(int argc, char **argv) {
    const char *mode = argc > 1 ? argv[1] : "plan";
    if (!strcmp(mode, "plan")) return plan_case();
    if (!strcmp(mode, "status")) return status_case();
    if (!strcmp(mode, "gpu")) return gpu_case();
    if (!strcmp(mode, "trap-rank")) {
        chelis_metadata_plan_new(i64(-1), NULL, exemplar(CHELIS_DTYPE_F32));
        return 0; /* not reached */
    }
    if (!strcmp(mode, "trap-view")) {
        chelis_scalar s[1] = {i64(10)}, st[1] = {i64(1)};
        chelis_metadata_plan_view(i64(1), s, st, exemplar(CHELIS_DTYPE_F32), i64(36));
        return 0; /* not reached */
    }
    fprintf(stderr, "unknown mode %s\n", mode);
    return 2;
}
