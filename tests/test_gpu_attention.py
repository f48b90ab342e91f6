"""Causal attention without materialised scores (chelis_cuda_attention_causal_fwd)
against a float64 evaluation of the reference graph:
softmax(where(causal, (q.k^T)*scale, -inf)).v per head.

Bound: each output element within max(2e-6, 3 x the error of a plain
float32 evaluation of the same graph) of the float64 value, normwise over
the tensor (|got - ref|max / |ref|max); the log-sum-exp within 1e-5 absolute
(it enters the adjoint as exp(s - lse)).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _reference(q, k, v, scale, dtype):
    import torch
    q, k, v = (torch.as_tensor(t, dtype=dtype) for t in (q, k, v))
    s = (q @ k.transpose(-1, -2)) * scale
    n = s.shape[-1]
    mask = torch.ones(n, n, dtype=torch.bool).tril()
    s = torch.where(mask, s, torch.tensor(-float("inf"), dtype=dtype))
    lse = torch.logsumexp(s, -1)
    return (torch.softmax(s, -1) @ v).numpy(), lse.numpy()


def _normwise(got, ref):
    """max |got - ref| / max |ref|; absolute when ref is identically zero
    (seq 1: the softmax is constant, dq = dk = 0)."""
    scale = np.abs(ref).max()
    return float(np.abs(got.astype(np.float64) - ref).max() / (scale if scale > 0 else 1.0))


@pytest.mark.parametrize("bh,seq,dh", [(1, 1, 64), (2, 64, 64), (3, 200, 64), (2, 384, 32),
                                       (4, 1000, 64), (1, 129, 32), (2, 2048, 64), (1, 2048, 32)])
def test_attention_causal_matches_float64(cuda, bh, seq, dh):
    import torch
    rng = np.random.default_rng(bh * 1000 + seq + dh)
    q, k, v = (rng.standard_normal((bh, seq, dh)).astype(np.float32) for _ in range(3))
    scale = np.float32(1.0 / np.sqrt(dh))
    o, lse = cuda.attention_causal(*(torch.from_numpy(t).cuda() for t in (q, k, v)), float(scale),
                                   with_lse=True)
    torch.cuda.synchronize()
    cuda.device_status()
    ref, ref_lse = _reference(q, k, v, float(scale), torch.float64)
    r32, _ = _reference(q, k, v, float(scale), torch.float32)
    bound = max(2e-6, 3.0 * _normwise(r32, ref))
    assert _normwise(o.cpu().numpy(), ref) <= bound
    assert np.abs(lse.cpu().numpy().astype(np.float64) - ref_lse).max() <= 1e-5


def test_attention_rejects_other_head_dims(cuda):
    import torch
    from chelis_b200 import lib as L
    x = torch.zeros((1, 8, 16), dtype=torch.float32, device="cuda")
    cuda._prepare(x)
    assert L.load().chelis_cuda_attention_causal_fwd(1, 8, 16, 1.0, x.data_ptr(), x.data_ptr(),
                                                      x.data_ptr(), x.data_ptr(), None) == 4


def _reference_grads(q, k, v, dout, scale, dtype):
    import torch
    Q, K, V = (torch.tensor(t, dtype=dtype, requires_grad=True) for t in (q, k, v))
    s = (Q @ K.transpose(-1, -2)) * scale
    n = s.shape[-1]
    mask = torch.ones(n, n, dtype=torch.bool).tril()
    s = torch.where(mask, s, torch.tensor(-float("inf"), dtype=dtype))
    o = torch.softmax(s, -1) @ V
    o.backward(torch.tensor(dout, dtype=dtype))
    return [t.grad.double().numpy() for t in (Q, K, V)]


@pytest.mark.parametrize("bh,seq,dh", [(1, 1, 64), (2, 64, 64), (3, 200, 64), (2, 384, 32),
                                       (2, 1000, 64), (1, 129, 32), (1, 300, 64), (2, 2048, 64),
                                       (1, 2048, 32)])
def test_attention_causal_bwd_matches_float64(cuda, bh, seq, dh):
    """dq, dk, dv from the blockwise recomputation against float64 autograd;
    each within max(1e-5, 3 x the float32 autograd error), normwise."""
    import torch
    rng = np.random.default_rng(7 * bh + seq + dh)
    q, k, v, do = (rng.standard_normal((bh, seq, dh)).astype(np.float32) for _ in range(4))
    scale = float(np.float32(1.0 / np.sqrt(dh)))
    tq, tk, tv, tdo = (torch.from_numpy(t).cuda() for t in (q, k, v, do))
    o, lse = cuda.attention_causal(tq, tk, tv, scale, with_lse=True)
    dq, dk, dv = cuda.attention_causal_bwd(tq, tk, tv, o, lse, tdo, scale)
    torch.cuda.synchronize()
    cuda.device_status()
    ref = _reference_grads(q, k, v, do, scale, torch.float64)
    r32 = _reference_grads(q, k, v, do, scale, torch.float32)
    for name, got, g64, g32 in zip(("dq", "dk", "dv"), (dq, dk, dv), ref, r32):
        bound = max(1e-5, 3.0 * _normwise(g32, g64))
        err = _normwise(got.cpu().numpy(), g64)
        assert err <= bound, (name, err, bound)


@pytest.mark.parametrize("bh,seq,dh", [(2, 2048, 64), (1, 777, 64)])
def test_attention_causal_matches_oracle(cuda, orc, bh, seq, dh):
    """Forward and reverse against the oracle's per-head restatement of the
    reference graph (scores materialised, canonical trees): o, dq, dk, dv
    within normwise f32 rel 1e-5."""
    import torch
    rng = np.random.default_rng(bh + seq)
    q, k, v, do = (rng.standard_normal((bh, seq, dh)).astype(np.float32) for _ in range(4))
    scale = float(np.float32(1.0 / np.sqrt(dh)))
    tq, tk, tv, tdo = (torch.from_numpy(t).cuda() for t in (q, k, v, do))
    o, lse = cuda.attention_causal(tq, tk, tv, scale, with_lse=True)
    dq, dk, dv = cuda.attention_causal_bwd(tq, tk, tv, o, lse, tdo, scale)
    torch.cuda.synchronize()
    cuda.device_status()
    o_ref, (dq_ref, dk_ref, dv_ref) = orc.attention_causal(q, k, v, scale, do)
    for name, got, ref in (("o", o, o_ref), ("dq", dq, dq_ref), ("dk", dk, dk_ref),
                           ("dv", dv, dv_ref)):
        err = _normwise(got.cpu().numpy(), ref.astype(np.float64))
        assert err <= 1e-5, (name, err)
