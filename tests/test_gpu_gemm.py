"""GEMM parity on the GPU against the oracle (canonical tree over k).

Tolerances (stated per the north star: f32 rel <= 1e-5, f64 rel <= 1e-12
after reductions) are componentwise and scaled by the reduction's own
magnitude:  |C - C_ref|_ij <= rtol * (|A| . |B|)_ij.  That is the standard
bound of a length-k dot product; it does not blow up where C_ij cancels to
near zero.  The exact-tree mode is compared bit for bit.
"""
import numpy as np
import pytest

from chelis_b200 import lib as L
from chelis_b200 import workloads as W

pytestmark = pytest.mark.gpu

SHAPES = [(1, 1, 1), (17, 33, 45), (128, 256, 32), (300, 500, 700), (512, 512, 512),
          (129, 257, 1000), (64, 8, 4096)]


def _rel_err(c, ref, a, b, ta=False, tb=False):
    import torch
    A = torch.as_tensor(a, dtype=torch.float64).abs()
    B = torch.as_tensor(b, dtype=torch.float64).abs()
    A = A.T if ta else A
    B = B.T if tb else B
    bound = (A @ B).numpy()
    err = np.abs(c.astype(np.float64) - ref.astype(np.float64))
    return float((err / np.maximum(bound, 1e-300)).max())


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_sgemm_3xtf32_matches_oracle(cuda, orc, m, n, k):
    import torch
    a, b = W.gemm_inputs(m, n, k, np.float32, seed=m + n + k)
    c = cuda.matmul(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()).cpu().numpy()
    cuda.device_status()
    ref = orc.gemm(a, b)
    assert _rel_err(c, ref, a, b) <= 1e-5


@pytest.mark.parametrize("ta,tb", [(True, False), (False, True), (True, True)])
def test_sgemm_transposed_operands(cuda, orc, ta, tb):
    import torch
    m, n, k = 190, 130, 310
    a, b = W.gemm_inputs(m, n, k, np.float32, seed=5)
    at = a.T.copy() if ta else a
    bt = b.T.copy() if tb else b
    c = cuda.matmul(torch.from_numpy(at).cuda(), torch.from_numpy(bt).cuda(), ta, tb).cpu().numpy()
    ref = orc.gemm(a, b)
    assert _rel_err(c, ref, a, b) <= 1e-5


def test_sgemm_batched_matches_oracle(cuda, orc):
    import torch
    a, b = W.gemm_inputs(96, 160, 200, np.float32, seed=2, batch=5)
    c = cuda.matmul(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()).cpu().numpy()
    for i in range(5):
        assert _rel_err(c[i], orc.gemm(a[i], b[i]), a[i], b[i]) <= 1e-5


@pytest.mark.parametrize("m,n,k", [(1, 1, 1), (37, 45, 33), (64, 96, 100), (128, 64, 1025)])
def test_sgemm_exact_tree_is_bit_exact(cuda, orc, m, n, k):
    import torch
    a, b = W.gemm_inputs(m, n, k, np.float32, seed=k)
    with cuda.gemm_mode(L.GEMM_EXACT_TREE):
        c = cuda.matmul(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()).cpu().numpy()
    ref = orc.gemm(a, b)
    assert (c.view(np.uint32) == ref.view(np.uint32)).all()


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_dgemm_matches_oracle(cuda, orc, m, n, k):
    import torch
    a, b = W.gemm_inputs(m, n, k, np.float64, seed=m * 3 + k)
    c = cuda.matmul(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()).cpu().numpy()
    ref = orc.gemm(a, b)
    assert _rel_err(c, ref, a, b) <= 1e-12


def test_dgemm_transposed_and_batched(cuda, orc):
    import torch
    a, b = W.gemm_inputs(70, 90, 130, np.float64, seed=8, batch=3)
    c = cuda.matmul(torch.from_numpy(a.transpose(0, 2, 1).copy()).cuda(),
                    torch.from_numpy(b).cuda(), True, False).cpu().numpy()
    for i in range(3):
        assert _rel_err(c[i], orc.gemm(a[i], b[i]), a[i], b[i]) <= 1e-12


def test_dgemm_exact_tree_is_bit_exact(cuda, orc):
    import torch
    a, b = W.gemm_inputs(50, 70, 300, np.float64, seed=4)
    with cuda.gemm_mode(L.GEMM_EXACT_TREE):
        c = cuda.matmul(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()).cpu().numpy()
    assert (c.view(np.uint64) == orc.gemm(a, b).view(np.uint64)).all()


@pytest.mark.parametrize("dtype,rtol", [(np.float32, 1e-5), (np.float64, 1e-12)])
def test_full_size_8192_sampled_rows(cuda, orc, dtype, rtol):
    """BASELINE config 2 at its largest size: every output computed on the
    GPU, a bounded sample of rows checked against the oracle."""
    import torch
    n = 8192
    a, b = W.gemm_inputs(n, n, n, dtype, seed=1)
    c = cuda.matmul(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda())
    torch.cuda.synchronize()
    cuda.device_status()
    rows = [0, 1, 127, 128, 4095, 8191]
    for r in rows:
        ref = orc.gemm(a[r:r + 1], b)
        got = c[r:r + 1].cpu().numpy()
        assert _rel_err(got, ref, a[r:r + 1], b) <= rtol, r


def test_row_major_helper_abi(cuda, orc):
    """chelis_cuda_sgemm_row_major through chelis_gpu_tensor descriptors
    (the chelis_hipblas_sgemm_row_major slot)."""
    import ctypes
    import torch
    m, n, k = 33, 65, 47
    a, b = W.gemm_inputs(m, n, k, np.float32, seed=12)
    ta, tb = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    tc = torch.empty((m, n), dtype=torch.float32, device="cuda")
    keep = []

    def desc(t):
        shape = (ctypes.c_int64 * 2)(*t.shape)
        strides = (ctypes.c_int64 * 2)(*t.stride())
        keep.extend([shape, strides])
        d = L.GpuTensor()
        d.data, d.shape, d.strides = t.data_ptr(), shape, strides
        d.count, d.byte_capacity, d.rank, d.dtype = t.numel(), t.numel() * 4, 2, L.DTYPE_F32
        return d

    cuda._prepare(ta)
    da, db, dc = desc(ta), desc(tb), desc(tc)
    L.call("chelis_cuda_sgemm_row_major", ctypes.byref(da), ctypes.byref(db), ctypes.byref(dc), m, n, k)
    torch.cuda.synchronize()
    assert _rel_err(tc.cpu().numpy(), orc.gemm(a, b), a, b) <= 1e-5
    # non-contiguous slices are rejected like the reference's precondition
    bad = desc(tb)
    bad.strides = (ctypes.c_int64 * 2)(1, k)
    assert L.load().chelis_cuda_sgemm_row_major(ctypes.byref(da), ctypes.byref(bad), ctypes.byref(dc), m, n, k) == 1


@pytest.mark.parametrize("a_layout,b_layout", [(0, 0), (0, 1), (1, 0), (1, 1)])
def test_presplit_layouts(cuda, orc, a_layout, b_layout):
    """chelis_cuda_tf32x3_split + chelis_cuda_sgemm_tf32x3_presplit with each
    operand K-major (layout 0) or MN-major (layout 1), batched, ragged
    extents (m, n not multiples of 4 or of the tile; k not of 32)."""
    import torch
    m, n, k, batch = 131, 301, 97, 3
    a, b = W.gemm_inputs(m, n, k, np.float32, seed=21, batch=batch)
    ta = torch.from_numpy(a).cuda()                       # [batch][m][k]
    tbt = torch.from_numpy(b).cuda()                      # [batch][k][n]
    # A as m x k: layout 0 from the row-major copy, layout 1 from A^T ([k][m])
    at = ta.transpose(1, 2).contiguous()
    bt = tbt.transpose(1, 2).contiguous()                 # [batch][n][k]

    def split(src, trans, layout, rows):
        if layout == 0:
            shape = (batch, rows, (k + 31) // 32 * 32)
        else:
            shape = (batch, k, (rows + 3) // 4 * 4)
        hi = torch.full(shape, float("nan"), dtype=torch.float32, device="cuda")
        lo = torch.full(shape, float("nan"), dtype=torch.float32, device="cuda")
        ld = src.shape[2]
        cuda._prepare(src)
        L.call("chelis_cuda_tf32x3_split", trans, layout, rows, k, src.data_ptr(), ld,
               src.shape[1] * src.shape[2], batch, hi.data_ptr(), lo.data_ptr())
        return hi, lo

    # layout 0 for A: row-major A (trans 0); layout 1: A^T source (trans 1)
    ahi, alo = split(ta, 0, 0, m) if a_layout == 0 else split(at, 1, 1, m)
    # B as n x k: layout 0 from B^T rows (trans 0); layout 1 from row-major B (trans 1)
    bhi, blo = split(bt, 0, 0, n) if b_layout == 0 else split(tbt, 1, 1, n)
    c = torch.full((batch, m, n), float("nan"), dtype=torch.float32, device="cuda")
    L.call("chelis_cuda_sgemm_tf32x3_presplit", m, n, k, batch, a_layout, ahi.data_ptr(),
           alo.data_ptr(), b_layout, bhi.data_ptr(), blo.data_ptr(), c.data_ptr(), n, m * n)
    torch.cuda.synchronize()
    cuda.device_status()
    got = c.cpu().numpy()
    for i in range(batch):
        assert _rel_err(got[i], orc.gemm(a[i], b[i]), a[i], b[i]) <= 1e-5, i


def test_split_forced_kmajor_from_transposed_source(cuda, orc):
    """layout 0 on a transposed source goes through the tile-transposing
    split; MN-major from a row-contiguous source is rejected."""
    import torch
    m, n, k = 70, 90, 45
    a, b = W.gemm_inputs(m, n, k, np.float32, seed=22)
    at = torch.from_numpy(a.T.copy()).cuda()              # [k][m]
    tb = torch.from_numpy(b).cuda()                       # [k][n]
    kp = (k + 31) // 32 * 32
    ahi = torch.empty((m, kp), dtype=torch.float32, device="cuda")
    alo = torch.empty_like(ahi)
    bhi = torch.empty((n, kp), dtype=torch.float32, device="cuda")
    blo = torch.empty_like(bhi)
    cuda._prepare(at)
    L.call("chelis_cuda_tf32x3_split", 1, 0, m, k, at.data_ptr(), m, 0, 1, ahi.data_ptr(), alo.data_ptr())
    L.call("chelis_cuda_tf32x3_split", 1, 0, n, k, tb.data_ptr(), n, 0, 1, bhi.data_ptr(), blo.data_ptr())
    c = torch.empty((m, n), dtype=torch.float32, device="cuda")
    L.call("chelis_cuda_sgemm_tf32x3_presplit", m, n, k, 1, 0, ahi.data_ptr(), alo.data_ptr(),
           0, bhi.data_ptr(), blo.data_ptr(), c.data_ptr(), n, 0)
    torch.cuda.synchronize()
    assert _rel_err(c.cpu().numpy(), orc.gemm(a, b), a, b) <= 1e-5
    lib = L.load()
    assert lib.chelis_cuda_tf32x3_split(0, 1, m, k, at.data_ptr(), k, 0, 1, ahi.data_ptr(),
                                        alo.data_ptr()) == 1  # CHELIS_CUDA_ERR_DOMAIN


@pytest.mark.parametrize("pairs", [True, False])
@pytest.mark.parametrize("m,n,k,ta,tb,batch", [
    (300, 500, 700, False, False, 1),     # ragged pair: rows 300..383 of the second pair idle
    (256, 256, 32, False, False, 1),      # exactly one pair tile, one k-block
    (513, 129, 1000, True, False, 1),     # MN-major A on pairs
    (384, 300, 257, True, True, 2),       # MN-major A, K-major B, batched
    (1024, 768, 96, False, True, 3),      # K-major both, batched
    (2404, 600, 64, False, False, 1),     # 10 pair-rows: two tile-order groups, ragged last
])
def test_sgemm_pair_and_single_cta_tiles(cuda, orc, pairs, m, n, k, ta, tb, batch):
    """The CTA-pair (cta_group::2, 256 x 256) and single-CTA (128 x 256) main
    kernels against the oracle, over both operand majors and batches."""
    import torch
    a, b = W.gemm_inputs(m, n, k, np.float32, seed=m + n + k + batch, batch=batch)
    sw = (lambda x: np.ascontiguousarray(np.swapaxes(x, -1, -2)))
    at = sw(a) if ta else a
    bt = sw(b) if tb else b
    with cuda.gemm_pairs(pairs):
        c = cuda.matmul(torch.from_numpy(at).cuda(), torch.from_numpy(bt).cuda(), ta, tb)
        torch.cuda.synchronize()
    cuda.device_status()
    got = c.cpu().numpy().reshape(batch, m, n)
    a3, b3 = a.reshape(batch, m, k), b.reshape(batch, k, n)
    for i in range(batch):
        assert _rel_err(got[i], orc.gemm(a3[i], b3[i]), a3[i], b3[i]) <= 1e-5, i


@pytest.mark.parametrize("m,n,k,batch", [(256, 256, 8192, 1), (300, 200, 3000, 2), (1024, 1024, 4096, 1)])
def test_sgemm_split_k_matches_oracle(cuda, orc, m, n, k, batch):
    """Products whose tile grid underfills the GPU run as split-K (partial
    products reduced in split order); same bound as every 3xTF32 product."""
    import torch
    a, b = W.gemm_inputs(m, n, k, np.float32, seed=m + k + batch, batch=batch)
    c = cuda.matmul(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()).cpu().numpy()
    cuda.device_status()
    a3, b3, c3 = a.reshape(batch, m, k), b.reshape(batch, k, n), c.reshape(batch, m, n)
    for i in range(batch):
        rows = slice(0, min(m, 64))
        ref = orc.gemm(a3[i][rows], b3[i])
        assert _rel_err(c3[i][rows], ref, a3[i][rows], b3[i]) <= 1e-5, i


@pytest.mark.parametrize("m,n,k,ta,tb", [
    (128, 256, 8192, 0, 0),      # single-CTA tiles, 64 accumulator chunks
    (512, 512, 8192, 0, 0),      # CTA pairs, split-K
    (8192, 8192, 8192, 0, 0),    # the headline product (sampled rows)
    (8192, 1024, 4096, 0, 1),    # A . B^T (activation gradients)
    (1024, 4096, 2048, 1, 0),    # A^T . B (weight gradients, long K)
    (1000, 700, 3001, 0, 0),     # ragged everywhere, last chunk partial
])
def test_sgemm_error_grows_like_an_f32_sum(cuda, orc, m, n, k, ta, tb):
    """The tensor core's accumulator loses accuracy linearly in K when one
    accumulator spans the whole product (normwise 5.8e-5 at K = 8192).  With
    fresh 128-deep accumulator chunks folded in f32, the error must stay
    within normwise 1e-5 of the oracle's tree and within 3x the error of a
    float32 BLAS product (numpy) on the same rows."""
    import torch
    rng = np.random.default_rng(m + n + k)
    a = (rng.random((k, m) if ta else (m, k), dtype=np.float32) * 2 - 1)
    b = (rng.random((n, k) if tb else (k, n), dtype=np.float32) * 2 - 1)
    c = cuda.matmul(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda(), ta, tb)
    torch.cuda.synchronize()
    cuda.device_status()
    rows = np.arange(m) if m <= 1024 else np.linspace(0, m - 1, 96).astype(np.int64)
    A = np.ascontiguousarray(a.T if ta else a)[rows]
    B = np.ascontiguousarray(b.T if tb else b)
    ref = orc.gemm(A, B).astype(np.float64)
    got = c.cpu().numpy()[rows].astype(np.float64)
    blas = (A @ B).astype(np.float64)
    err = np.abs(got - ref).max() / np.abs(ref).max()
    err_blas = np.abs(blas - ref).max() / np.abs(ref).max()
    assert err <= 1e-5, (err, err_blas)
    assert err <= max(3.0 * err_blas, 2e-6), (err, err_blas)


F64_KERNEL_SHAPES = [(1, 1, 1), (17, 33, 45), (64, 8, 4096), (300, 500, 700), (512, 512, 512),
                     (129, 257, 1000), (1024, 1024, 256), (2048, 1536, 512)]


@pytest.mark.parametrize("kernel", [L.DGEMM_DMMA, L.DGEMM_FFMA, L.DGEMM_AUTO])
@pytest.mark.parametrize("m,n,k", F64_KERNEL_SHAPES)
def test_dgemm_kernels_match_oracle(cuda, orc, kernel, m, n, k):
    """DMMA, FFMA and the per-shape choice all meet f64 rel <= 1e-12."""
    import torch
    a, b = W.gemm_inputs(m, n, k, np.float64, seed=m + 7 * n + k)
    with cuda.dgemm_kernel(kernel):
        c = cuda.matmul(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()).cpu().numpy()
    assert _rel_err(c, orc.gemm(a, b), a, b) <= 1e-12


@pytest.mark.parametrize("kernel", [L.DGEMM_DMMA, L.DGEMM_FFMA])
@pytest.mark.parametrize("ta,tb", [(True, False), (False, True), (True, True)])
def test_dgemm_kernels_transposed_batched(cuda, orc, kernel, ta, tb):
    import torch
    a, b = W.gemm_inputs(70, 90, 131, np.float64, seed=9, batch=3)
    A = a.transpose(0, 2, 1).copy() if ta else a
    B = b.transpose(0, 2, 1).copy() if tb else b
    with cuda.dgemm_kernel(kernel):
        c = cuda.matmul(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda(), ta, tb).cpu().numpy()
    for i in range(3):
        assert _rel_err(c[i], orc.gemm(a[i], b[i]), a[i], b[i]) <= 1e-12


def test_dgemm_per_call_and_thread_modes(cuda, orc):
    """chelis_cuda_dgemm_ex / _sgemm_ex choose the arithmetic for one call and
    leave the thread's and the process's settings alone; the thread setting
    is the thread's own."""
    import ctypes
    import threading
    import torch
    lib = L.load()
    a, b = W.gemm_inputs(40, 60, 300, np.float64, seed=5)
    A, B = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    C = torch.empty(40, 60, dtype=torch.float64, device="cuda")
    L.call("chelis_cuda_dgemm_ex", L.GEMM_EXACT_TREE, L.DGEMM_AUTO, 0, 0, 40, 60, 300, A.data_ptr(),
           300, 0, B.data_ptr(), 60, 0, C.data_ptr(), 60, 0, 1)
    assert (C.cpu().numpy().view(np.uint64) == orc.gemm(a, b).view(np.uint64)).all()
    assert lib.chelis_cuda_get_gemm_mode() == L.GEMM_3XTF32
    g = ctypes.c_int()
    L.call("chelis_cuda_get_thread_modes", ctypes.byref(g), None, None)
    assert g.value == L.GEMM_3XTF32
    seen = {}

    def other():
        L.call("chelis_cuda_set_thread_modes", L.GEMM_EXACT_TREE, -1, -1)
        v = ctypes.c_int()
        L.call("chelis_cuda_get_thread_modes", ctypes.byref(v), None, None)
        seen["other"] = v.value

    t = threading.Thread(target=other)
    t.start()
    t.join()
    L.call("chelis_cuda_get_thread_modes", ctypes.byref(g), None, None)
    assert seen["other"] == L.GEMM_EXACT_TREE and g.value == L.GEMM_3XTF32
    assert lib.chelis_cuda_dgemm_kernel_for(0, 0, 8192, 8192, 8192, 1) == L.DGEMM_DMMA
    assert lib.chelis_cuda_dgemm_kernel_for(0, 0, 512, 512, 512, 1) == L.DGEMM_FFMA
    assert lib.chelis_cuda_dgemm_kernel_for(1, 0, 8192, 8192, 8192, 1) == L.DGEMM_DMMA
    assert lib.chelis_cuda_dgemm_kernel_for(0, 0, 256, 256, 4096, 1) == L.DGEMM_FFMA


def test_shutdown_releases_and_library_recovers(cuda, orc):
    import torch
    a, b = W.gemm_inputs(256, 384, 320, np.float32, seed=3)
    A, B = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    c1 = cuda.matmul(A, B).cpu().numpy()
    torch.cuda.synchronize()
    L.call("chelis_cuda_shutdown")
    c2 = cuda.matmul(A, B).cpu().numpy()
    assert (c1.view(np.uint32) == c2.view(np.uint32)).all()


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("m,n,k,ta,tb,batch", [(1, 1, 1, 0, 0, 1), (130, 70, 260, 0, 0, 1),
                                                (256, 384, 512, 0, 0, 1), (64, 96, 200, 1, 0, 1),
                                                (64, 96, 200, 0, 1, 3), (300, 129, 33, 1, 1, 2)])
def test_gemm16_f32_accumulate(cuda, dtype, m, n, k, ta, tb, batch):
    """bf16 / f16 storage, f32 products and sums, one rounding to the storage
    type: |C - round16(ref)| <= half an ulp of the storage type at |ref| plus
    the f32 accumulation bound k * 2^-23 * (|A| . |B|)."""
    import torch
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float16
    code = L.DTYPE_BF16 if dtype == "bf16" else L.DTYPE_F16
    g = torch.Generator(device="cuda").manual_seed(m + n + k)
    A = torch.randn((batch, k, m) if ta else (batch, m, k), device="cuda", generator=g).to(tdt)
    B = torch.randn((batch, n, k) if tb else (batch, k, n), device="cuda", generator=g).to(tdt)
    C = torch.empty((batch, m, n), device="cuda", dtype=tdt)
    lda, ldb = A.shape[2], B.shape[2]
    cuda._prepare(A)
    L.call("chelis_cuda_gemm16", code, ta, tb, m, n, k, A.data_ptr(), lda, A[0].numel(), B.data_ptr(),
           ldb, B[0].numel(), C.data_ptr(), n, m * n, batch)
    torch.cuda.synchronize()
    A64 = A.double().transpose(1, 2) if ta else A.double()
    B64 = B.double().transpose(1, 2) if tb else B.double()
    ref = A64 @ B64
    bound = A64.abs() @ B64.abs()
    ulp_half = (2.0 ** -8 if dtype == "bf16" else 2.0 ** -11) * ref.abs()
    err = (C.double() - ref).abs()
    assert bool((err <= ulp_half + (k + 2) * 2.0 ** -23 * bound + 1e-30).all())


def test_gemm16_row_major_helper(cuda):
    import ctypes
    import torch
    g = torch.Generator(device="cuda").manual_seed(7)
    A = torch.randn(70, 90, device="cuda", generator=g).to(torch.bfloat16)
    B = torch.randn(90, 50, device="cuda", generator=g).to(torch.bfloat16)
    C = torch.empty(70, 50, device="cuda", dtype=torch.bfloat16)

    keep = []

    def desc(t):
        shape = (ctypes.c_int64 * 2)(*t.shape)
        strides = (ctypes.c_int64 * 2)(*t.stride())
        keep.extend([shape, strides])
        d = L.GpuTensor()
        d.data, d.shape, d.strides = t.data_ptr(), shape, strides
        d.count, d.byte_capacity, d.rank, d.dtype = t.numel(), t.numel() * 2, 2, L.DTYPE_BF16
        return d

    cuda._prepare(A)
    da, db, dc = desc(A), desc(B), desc(C)
    L.call("chelis_cuda_bf16_gemm_f32_acc_row_major", ctypes.byref(da), ctypes.byref(db),
           ctypes.byref(dc), 70, 50, 90)
    torch.cuda.synchronize()
    ref = A.double() @ B.double()
    bound = A.double().abs() @ B.double().abs()
    assert bool(((C.double() - ref).abs() <= 2.0 ** -8 * ref.abs() + 92 * 2.0 ** -23 * bound).all())
