"""chelis_cuda_chain_bwd_noalloc: the fused-chain adjoint for callers that
cannot let the library allocate device memory (a host that fixed its whole
device arena in advance, or one that forbids driver allocation while it
runs).  Its scratch is a fixed device array inside the library, so it is
checked here against the allocating entry, chelis_cuda_chain_bwd, through the
C ABI, on two calls in a row (the second call finds the first call's
leftovers in the shared array and must not depend on them).

dx must equal the allocating entry's bit for bit.  dgamma / dbeta must too
when the allocating entry's grid (two CTAs per SM) fits the array's 296
CTAs, as on a 148-SM B200; otherwise they agree within f32 rel 1e-5.

This file is collected last on purpose: it must pass alone in a fresh
process and after every other test.
"""
import numpy as np
import pytest

from chelis_b200 import lib as L
from chelis_b200 import workloads as W

pytestmark = pytest.mark.gpu

RTOL = 1e-5  # f32 rel after reductions, as in tests/test_gpu_rows.py
MAX_GRID = 296  # CTAs the no-allocation entry's scratch array holds


def _normwise(got, ref):
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


def _noalloc(x, g, b, stats, eps, key, rate, base):
    import torch
    rows, hidden = x.shape
    dx = torch.full_like(x, float("nan"))
    dg = torch.full((hidden,), float("nan"), dtype=torch.float32, device=x.device)
    db = torch.full((hidden,), float("nan"), dtype=torch.float32, device=x.device)
    L.call("chelis_cuda_chain_bwd_noalloc", x.data_ptr(), g.data_ptr(), b.data_ptr(), eps, key,
           rate, rows, hidden, base, None if stats is None else stats.data_ptr(), dx.data_ptr(),
           dg.data_ptr(), db.data_ptr())
    return dx, dg, db


def _same_grid():
    import torch
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    return 2 * sms <= MAX_GRID


@pytest.mark.parametrize("rows,hidden,saved_stats", [
    (1000, 4096, True), (37, 1000, True), (200, 4096, True), (1000, 4096, False),
    (700, 257, False),
])
def test_noalloc_adjoint_matches_allocating_entry_twice(cuda, rows, hidden, saved_stats):
    import torch
    eps, key, rate = 1e-5, W.CHAIN_KEY, 0.1
    for call, seed in enumerate((rows + hidden, rows + hidden + 1)):
        x, g, b = (torch.from_numpy(v).cuda() for v in W.chain_inputs(rows, hidden, seed=seed))
        cuda._prepare(x, g, b)  # device init + torch's current stream
        base = 4096 * call
        stats = None
        if saved_stats:
            _, stats = cuda.chain_fwd(x, g, b, eps, key, rate, base, want_stats=True)
        ref = [t.cpu().numpy() for t in cuda.chain_bwd(x, g, b, eps, key, rate, base, stats)]
        cuda._prepare(x)
        got = [t.cpu().numpy() for t in _noalloc(x, g, b, stats, eps, key, rate, base)]
        torch.cuda.synchronize()
        cuda.device_status()
        assert np.array_equal(got[0].view(np.uint32), ref[0].view(np.uint32)), call
        if _same_grid():
            assert np.array_equal(got[1].view(np.uint32), ref[1].view(np.uint32)), call
            assert np.array_equal(got[2].view(np.uint32), ref[2].view(np.uint32)), call
        else:
            assert _normwise(got[1], ref[1]) <= RTOL, call
            assert _normwise(got[2], ref[2]) <= RTOL, call


def test_noalloc_zero_rows_gives_zero_parameter_gradients(cuda):
    import torch
    hidden = 512
    x = torch.empty((0, hidden), dtype=torch.float32, device="cuda")
    g = torch.ones(hidden, dtype=torch.float32, device="cuda")
    cuda._prepare(x, g)
    _, dg, db = _noalloc(x, g, g, None, 1e-5, 42, 0.1, 0)
    torch.cuda.synchronize()
    assert torch.count_nonzero(dg).item() == 0 and torch.count_nonzero(db).item() == 0
    assert not torch.signbit(dg).any().item() and not torch.signbit(db).any().item()


def test_noalloc_rejects_rows_beyond_its_limit(cuda):
    import torch
    x = torch.zeros((2, 4097), dtype=torch.float32, device="cuda")
    g = torch.ones(4097, dtype=torch.float32, device="cuda")
    cuda._prepare(x, g)
    with pytest.raises(L.ChelisCudaError, match="hidden <= 4096"):
        _noalloc(x, g, g, None, 1e-5, 42, 0.1, 0)
