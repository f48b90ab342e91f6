"""matmul on host buffers (chelis_cuda_[sd]gemm_host): the pipelined
upload / GEMM-panel / read-back path against the oracle.

Tolerances as for the device GEMM: |C - C_ref|_ij <= rtol * (|A|.|B|)_ij with
rtol 1e-5 (f32, 3xTF32) and 1e-12 (f64); the exact-tree mode must match the
device-buffer exact-tree GEMM bit for bit.
"""
import numpy as np
import pytest

from chelis_b200 import lib as L
from chelis_b200 import workloads as W

pytestmark = pytest.mark.gpu


def _rel_err(c, ref, a, b):
    bound = np.abs(a.astype(np.float64)) @ np.abs(b.astype(np.float64))
    err = np.abs(c.astype(np.float64) - ref.astype(np.float64))
    return float((err / np.maximum(bound, 1e-300)).max())


@pytest.mark.parametrize("dtype,rtol", [(np.float32, 1e-5), (np.float64, 1e-12)])
@pytest.mark.parametrize("m,n,k", [(1, 1, 1), (37, 45, 33), (1000, 300, 257), (2100, 130, 96)])
@pytest.mark.parametrize("pinned", [True, False])
def test_host_gemm_matches_oracle(cuda, orc, dtype, rtol, m, n, k, pinned):
    import torch
    a, b = W.gemm_inputs(m, n, k, dtype, seed=m + 3 * n + k)
    ta, tb = torch.from_numpy(a), torch.from_numpy(b)
    if pinned:
        ta, tb = ta.pin_memory(), tb.pin_memory()
    c = cuda.matmul_host(ta, tb).numpy()
    cuda.device_status()
    assert _rel_err(c, orc.gemm(a, b), a, b) <= rtol


@pytest.mark.parametrize("dtype,rtol", [(np.float32, 1e-5), (np.float64, 1e-12)])
@pytest.mark.parametrize("tr_a,tr_b", [(True, False), (False, True), (True, True)])
def test_host_gemm_transposed(cuda, orc, dtype, rtol, tr_a, tr_b):
    import torch
    m, n, k = 700, 190, 310
    a, b = W.gemm_inputs(m, n, k, dtype, seed=7)
    at = a.T.copy() if tr_a else a
    bt = b.T.copy() if tr_b else b
    c = cuda.matmul_host(torch.from_numpy(at).pin_memory(), torch.from_numpy(bt).pin_memory(),
                         tr_a, tr_b).numpy()
    assert _rel_err(c, orc.gemm(a, b), a, b) <= rtol


def test_host_gemm_batched_and_padded_ldc(cuda, orc):
    """batch items `stride` apart and an output row stride wider than n."""
    import torch
    m, n, k, batch = 300, 70, 129, 3
    a, b = W.gemm_inputs(m, n, k, np.float32, seed=9, batch=batch)
    ldc = n + 5
    c = torch.full((batch, m, ldc), float("nan"), dtype=torch.float32).pin_memory()
    ha, hb = torch.from_numpy(a).pin_memory(), torch.from_numpy(b).pin_memory()
    cuda._prepare()
    L.call("chelis_cuda_sgemm_host", 0, 0, m, n, k, ha.data_ptr(), k, m * k, hb.data_ptr(), n,
           k * n, c.data_ptr(), ldc, m * ldc, batch)
    torch.cuda.synchronize()
    got = c.numpy()
    assert np.isnan(got[:, :, n:]).all()
    for i in range(batch):
        assert _rel_err(got[i, :, :n], orc.gemm(a[i], b[i]), a[i], b[i]) <= 1e-5


def test_host_gemm_exact_mode_bit_exact(cuda):
    import torch
    from chelis_b200.lib import GEMM_EXACT_TREE
    m, n, k = 333, 77, 500
    a, b = W.gemm_inputs(m, n, k, np.float32, seed=10)
    with cuda.gemm_mode(GEMM_EXACT_TREE):
        host = cuda.matmul_host(torch.from_numpy(a), torch.from_numpy(b)).numpy()
        dev = cuda.matmul(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()).cpu().numpy()
    assert np.array_equal(host.view(np.uint32), dev.view(np.uint32))


def test_host_gemm_empty_contraction_is_zero(cuda):
    import torch
    a = torch.empty((5, 0), dtype=torch.float64)
    b = torch.empty((0, 7), dtype=torch.float64)
    c = cuda.matmul_host(a, b)
    assert c.shape == (5, 7) and (c == 0).all()
