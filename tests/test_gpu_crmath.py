"""Correctly rounded binary32 exp / log on the device against CORE-MATH (the
C lane's libm, linked into the oracle): every one of the 2^32 inputs, bit for
bit (any NaN matches any NaN)."""
import numpy as np
import pytest
import torch

from chelis_b200 import lib as L

pytestmark = pytest.mark.gpu

CHUNK = 1 << 28


@pytest.mark.parametrize("op,name", [(0, "exp"), (1, "log")])
def test_every_binary32_input_matches_core_math(cuda, orc, op, name):
    cuda._prepare(torch.empty(1, device="cuda"))
    out = torch.empty(CHUNK, dtype=torch.float32, device="cuda")
    host = torch.empty(CHUNK, dtype=torch.float32).pin_memory()
    for c in range((1 << 32) // CHUNK):
        start = c * CHUNK
        L.call("chelis_cuda_crmath_sweep_f32", op, start, CHUNK, out.data_ptr())
        host.copy_(out)
        bad, first = orc.crmath_check_f32(op, start, host.numpy())
        assert bad == 0, f"{name}: {bad} mismatches from bits {start:#010x}, first {start + first:#010x}"


def test_array_entry_and_specials(cuda, orc):
    x = np.array([0.0, -0.0, 1.0, -1.0, 88.72283, 88.7229, -103.97208, -103.9721, 1e-45, 2.0 ** -126,
                  np.inf, -np.inf, np.nan, 3.4e38, 0.5, 1.0000001, 0.99999994], dtype=np.float32)
    xs = torch.from_numpy(x).cuda()
    for op, ref in ((0, orc.expf), (1, orc.logf)):
        y = torch.empty_like(xs)
        L.call("chelis_cuda_crmath_f32", op, xs.data_ptr(), y.data_ptr(), x.size)
        got = y.cpu().numpy()
        want = np.array([ref(float(v)) for v in x], dtype=np.float32)
        same = (got.view(np.uint32) == want.view(np.uint32)) | (np.isnan(got) & np.isnan(want))
        assert same.all(), (op, x[~same], got[~same], want[~same])
