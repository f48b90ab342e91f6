"""Pins the parity oracle (oracle/) against the reference's own known-answer
tests and fixtures, and checks its adjoint graphs against autograd.  CPU only.
"""
import struct

import numpy as np
import pytest

from chelis_b200 import workloads as W


def f32_from_bits(b):
    return struct.unpack("<f", struct.pack("<I", b))[0]


def bits_f32(x):
    return struct.unpack("<I", struct.pack("<f", float(np.float32(x))))[0]


# ---------------------------------------------------------------- keyed RNG
# crates/chelis-numeric-core/src/dtype_semantics.rs:5340-5425

def test_rng_word_and_unit_known_answers(orc):
    k45 = orc.key_from_seed(45)
    assert orc.word(k45, 0) == 0x3CF6DC70D6515D83
    assert bits_f32(orc.unit(k45, 0)) == 0x3E73DB72
    k7 = orc.key_from_seed(7)
    assert orc.word(k7, 0) == 0x20654588FCD25740
    assert orc.unit(k7, 0) == 0.12654528231070938
    k44 = orc.key_from_seed(44)
    assert orc.unit(k44, 0) < 0.5 <= orc.unit(k44, 1)


def _spec_unit(key, index):
    # [05-RNG-2] word and [05-RNG-1] unit written out from the spec text
    M = (1 << 64) - 1

    def sm(x):
        z = (x + 0x9E3779B97F4A7C15) & M
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M
        return z ^ (z >> 31)

    s = sm(index)
    rot = ((s << 41) | (s >> 23)) & M
    return (sm(key ^ rot) >> 11) / float(1 << 53)


def test_rng_matches_spec_transcription(orc):
    M = (1 << 64) - 1
    for seed in [0, 42, -1, -(1 << 63), (1 << 63) - 1]:
        root = orc.key_from_seed(seed)
        keys = [root, orc.derive(root, 0), orc.derive(root, 1)]
        for key in keys:
            for index in [0, 1, 5, 1 << 40, M]:
                assert orc.unit(key, index) == _spec_unit(key, index)


# ---------------------------------------------------------------- dropout
# dtype_semantics.rs:5340-5408

def test_dropout_rounds_unit_then_compares_and_finalizes_division(orc):
    key = orc.key_from_seed(45)
    rate = np.float32(f32_from_bits(0x3E73DB72))
    y = orc.dropout(np.array([1.0], np.float32), key, rate)
    assert y[0] == np.float32(1.0) / (np.float32(1.0) - rate)
    x = np.array([f32_from_bits(0x3F800005)], np.float32)
    y = orc.dropout(x, key, np.float32(0.1))
    assert y.view(np.uint32)[0] == 0x3F8E38E9
    assert y.view(np.uint32)[0] != 0x3F8E38EA  # reciprocal-multiply mutant


def test_dropout_keeps_signed_zero_and_is_pure(orc):
    x = np.array([-0.0, -0.0], np.float32)
    a = orc.dropout(x, orc.key_from_seed(44), np.float32(0.5))
    b = orc.dropout(x, orc.key_from_seed(44), np.float32(0.5))
    assert a.view(np.uint32).tolist() == [0, 0x80000000]
    assert (a.view(np.uint32) == b.view(np.uint32)).all()
    assert orc.dropout(np.zeros(0, np.float32), orc.key_from_seed(-1), np.float32(0.5)).size == 0


def _threshold(rate):
    """Host rule of libchelis_cuda (rows.cu dropout_threshold): least 53-bit
    integer whose f32 rounding reaches rate * 2^53."""
    target = float(np.float32(rate)) * 2.0 ** 53
    lo, hi = 0, 1 << 53
    while lo < hi:
        mid = (lo + hi) // 2
        if float(np.float32(mid)) >= target:
            hi = mid
        else:
            lo = mid + 1
    return lo


@pytest.mark.parametrize("rate", [0.1, 0.5, 0.0, f32_from_bits(0x3E73DB72), 0.999])
def test_integer_threshold_equals_rounded_unit_compare(orc, rate):
    rate = np.float32(rate)
    thr = _threshold(rate)
    key = orc.key_from_seed(42)
    n = 20000
    keep = orc.dropout_mask(n, key, rate)
    words = np.array([orc.word(key, i) for i in range(n)], dtype=np.uint64)
    assert ((words >> np.uint64(11)) >= np.uint64(thr)).astype(np.uint8).tolist() == keep.tolist()
    # boundary integers around the threshold
    for u in [thr - 2, thr - 1, thr, thr + 1]:
        if u < 0:
            continue
        unit32 = np.float32(u / float(1 << 53))
        assert (float(unit32) >= float(rate)) == (u >= thr)


# ---------------------------------------------------------------- tree schedule
# crates/chelis-backend-c/tests/reduction_carry_tree.rs:757-806

def _pass_by_pass(count):
    level = [str(i) for i in range(count)]
    while len(level) > 1:
        level = [f"({level[i]}+{level[i + 1]})" if i + 1 < len(level) else level[i]
                 for i in range(0, len(level), 2)]
    return level[0] if level else None


def _carried(count):
    levels = [None] * 64
    for leaf in range(count):
        carry, depth, pending = str(leaf), 0, leaf
        while pending & 1:
            carry = f"({levels[depth]}+{carry})"
            levels[depth] = None
            pending >>= 1
            depth += 1
        levels[depth] = carry
    total, remaining = None, count
    for lv in levels:
        if remaining & 1:
            total = lv if total is None else f"({lv}+{total})"
        remaining >>= 1
    return total


def _split_pow2(lo, hi):
    # split at the largest power of two below the count (the form the CUDA
    # kernels use: aligned power-of-two blocks are subtrees)
    n = hi - lo
    if n == 0:
        return None
    if n == 1:
        return str(lo)
    p = 1
    while p * 2 < n:
        p *= 2
    return f"({_split_pow2(lo, lo + p)}+{_split_pow2(lo + p, hi)})"


@pytest.mark.parametrize("counts", [range(0, 1025), [2047, 2048, 2049, 4095, 4096, 4097]])
def test_carry_schedule_is_adjacent_pair_tree(counts):
    for c in counts:
        ref = _pass_by_pass(c)
        assert _carried(c) == ref, c
        assert _split_pow2(0, c) == ref, c


def _fold_f32(x):
    level = list(np.asarray(x, np.float32))
    while len(level) > 1:
        level = [np.float32(level[i] + level[i + 1]) if i + 1 < len(level) else level[i]
                 for i in range(0, len(level), 2)]
    return np.float32(level[0]) if level else np.float32(0)


def test_oracle_tree_sum_is_bit_exact_pass_by_pass(orc):
    rng = np.random.default_rng(7)
    for n in [0, 1, 2, 3, 5, 31, 32, 33, 100, 1023, 1024, 1025, 4097]:
        x = (rng.standard_normal(n) * 10 ** rng.uniform(-3, 3, n)).astype(np.float32)
        assert orc.tree_sum(x).view(np.uint32) == _fold_f32(x).view(np.uint32), n


def test_oracle_gemm_matches_tree_per_output(orc):
    rng = np.random.default_rng(3)
    a = rng.standard_normal((5, 37)).astype(np.float32)
    b = rng.standard_normal((37, 70)).astype(np.float32)
    c = orc.gemm(a, b)
    for i in range(5):
        for j in range(0, 70, 7):
            leaves = (a[i, :] * b[:, j]).astype(np.float32)
            assert c[i, j].view(np.uint32) == _fold_f32(leaves).view(np.uint32)
    ct = orc.gemm_t(a.T.copy(), b.T.copy(), True, True)
    assert (ct.view(np.uint32) == c.view(np.uint32)).all()


@pytest.mark.parametrize("k", [0, 1, 7, 8, 9, 64, 100, 263, 1024])
@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_oracle_gemm_grouped_leaves_equal_the_carry_tree(orc, k, dtype):
    """Full 64-column blocks take 8-leaf groups (each an aligned subtree) into
    the carry tree; the values must equal the leaf-by-leaf tree bit for bit,
    with specials among the operands, for plain and transposed operands."""
    rng = np.random.default_rng(k + 11)
    m, n = 3, 150  # two full 64-column blocks and a ragged one
    a = (rng.standard_normal((m, k)) * 10 ** rng.uniform(-4, 4, (m, k))).astype(dtype)
    b = (rng.standard_normal((k, n)) * 10 ** rng.uniform(-4, 4, (k, n))).astype(dtype)
    if k > 9:
        a[1, 5] = np.inf
        b[7, 3] = np.nan
        b[2, 70] = -np.inf
    c = orc.gemm(a, b)
    view = np.uint32 if dtype == np.float32 else np.uint64
    for i in range(m):
        for j in (0, 3, 63, 64, 70, 127, 128, 149):
            leaves = (a[i, :] * b[:, j]).astype(dtype)
            assert c[i, j].view(view) == np.asarray(orc.tree_sum(leaves), dtype).view(view), (i, j)
    ct = orc.gemm_t(a.T.copy(), b.T.copy(), True, True)
    assert (ct.view(view) == c.view(view)).all()


# ---------------------------------------------------------------- CORE-MATH and IEEE pins

def _golden(name):
    import os
    path = os.path.join(os.path.dirname(__file__), "golden", name)
    with open(path) as f:
        return [ln.split() for ln in f if ln.strip() and not ln.startswith("#")]


def test_oracle_transcendentals_match_reference_canary(orc):
    fns = {"exp": orc.lib().orc_expf, "log": orc.lib().orc_logf, "erfc": orc.lib().orc_erfcf}
    rows = _golden("crmath_f32.txt")
    assert len(rows) > 100
    for fn, xin, want in rows:
        got = bits_f32(fns[fn](f32_from_bits(int(xin, 16))))
        assert got == int(want, 16), (fn, xin, want, hex(got))


def test_oracle_arithmetic_matches_reference_obligations(orc):
    L = orc.lib()
    rows = _golden("ieee_f32.txt")
    assert len(rows) > 50
    for prim, want, *ops in rows:
        v = [f32_from_bits(int(o, 16)) for o in ops]
        if prim == "add":
            got = L.orc_add_f32(*v)
        elif prim == "mul":
            got = L.orc_mul_f32(*v)
        elif prim == "div":
            got = L.orc_div_f32(*v)
        else:
            got = L.orc_sqrt_f32(*v)
        assert bits_f32(got) == int(want, 16), (prim, ops, want, hex(bits_f32(got)))


# ---------------------------------------------------------------- adjoint graphs vs autograd

def test_chain_adjoint_matches_autograd(orc):
    torch = pytest.importorskip("torch")
    x, g, b = W.chain_inputs(rows=64, hidden=256, seed=11)
    eps, key, rate = W.CHAIN_EPS, W.CHAIN_KEY, W.CHAIN_RATE
    rs = orc.chain_fwd(x, g, b, eps, key, rate)
    dx, dg, db = orc.chain_bwd(x, g, b, eps, key, rate)
    keep = orc.dropout_mask(x.size, key, rate).reshape(x.shape).astype(np.float64)
    den = float(np.float32(1.0) - rate)
    X = torch.tensor(x, dtype=torch.float64, requires_grad=True)
    G = torch.tensor(g, dtype=torch.float64, requires_grad=True)
    B = torch.tensor(b, dtype=torch.float64, requires_grad=True)
    m = X.mean(1, keepdim=True)
    c = X - m
    v = (c * c).mean(1, keepdim=True)
    y = c / torch.sqrt(v + float(eps)) * G + B
    s = torch.softmax(y, 1)
    p = s * torch.tensor(keep) / den
    r = p.sum(1)
    r.sum().backward()
    np.testing.assert_allclose(rs, r.detach().numpy(), rtol=2e-5, atol=0)
    scale = np.abs(X.grad.numpy()).max()
    assert np.abs(dx - X.grad.numpy()).max() <= 1e-4 * scale
    assert np.abs(dg - G.grad.numpy()).max() <= 1e-4 * np.abs(G.grad.numpy()).max()
    assert np.abs(db - B.grad.numpy()).max() <= 1e-4 * np.abs(B.grad.numpy()).max()


def test_mlp_adjoint_matches_autograd(orc):
    torch = pytest.importorskip("torch")
    x, labels, w1, b1, w2, b2 = W.mlp_inputs(batch=16, din=40, dh=24, dout=10, seed=5)
    b1 = (np.random.default_rng(1).standard_normal(24) * 0.1).astype(np.float32)
    loss, dw1, db1, dw2, db2 = orc.mlp_step(x, labels, w1, b1, w2, b2)
    T = {k: torch.tensor(v, dtype=torch.float64, requires_grad=True)
         for k, v in dict(w1=w1, b1=b1, w2=w2, b2=b2).items()}
    h = torch.relu(torch.tensor(x, dtype=torch.float64) @ T["w1"] + T["b1"])
    z = h @ T["w2"] + T["b2"]
    L = torch.nn.functional.cross_entropy(z, torch.tensor(labels))
    L.backward()
    assert abs(loss - L.item()) <= 1e-5 * abs(L.item())
    for name, got in dict(w1=dw1, b1=db1, w2=dw2, b2=db2).items():
        want = T[name].grad.numpy()
        assert np.abs(got - want).max() <= 1e-4 * np.abs(want).max(), name


def test_portfolio_matches_numpy(orc):
    r, w = W.portfolio_inputs(count=8, t=252, a=64, seed=9)
    sigma, risk, cum = orc.portfolio(r, w)
    for p in range(8):
        c = r[p] - r[p].mean(0)
        s = c.T @ c / 251.0
        np.testing.assert_allclose(sigma[p], s, rtol=1e-12, atol=1e-18)
        np.testing.assert_allclose(risk[p], np.sqrt(w[p] @ s @ w[p]), rtol=1e-12)
        np.testing.assert_allclose(cum[p], np.cumsum(r[p] @ w[p]), rtol=1e-12, atol=1e-16)


def test_cumsum_first_prefix_is_first_input(orc):
    x = np.array([[-0.0, 1.0, 2.0]], np.float64)
    y = orc.cumsum(x)
    assert np.signbit(y[0, 0]) and y[0, 2] == 3.0
    yr = orc.cumsum(x, reverse=True)
    assert yr[0].tolist() == [3.0, 3.0, 2.0]


# ---------------------------------------------------------------- transformer block (config 4)

@pytest.mark.parametrize("shape", [
    dict(batch=2, seq=64, d_model=128, heads=2, d_ff=512),
    dict(batch=1, seq=200, d_model=128, heads=4, d_ff=384),
    dict(batch=3, seq=17, d_model=64, heads=2, d_ff=96),
])
def test_oracle_block_step_matches_float64_autograd(orc, shape):
    """orc_block_step (the reference graph restated: tree matmuls, masked
    softmax, Phi-graph GELU and the AD graphs) against torch float64 autograd
    of the same block: every output within normwise 2e-6 and no further
    from float64 than a plain float32 evaluation is."""
    import torch
    from _block_ref import normwise, reference
    from chelis_b200 import workloads as W
    x, dy, w = W.block_inputs(seed=5, **shape)
    y, g = orc.block_step(x, w, shape["heads"], 1e-5, dy)
    y64, g64 = reference(x, dy, w, shape["heads"], 1e-5)
    y32, g32 = reference(x, dy, w, shape["heads"], 1e-5, torch.float32)
    assert normwise(y, y64) <= max(2e-6, normwise(y32, y64))
    for k in g64:
        assert normwise(g[k], g64[k]) <= max(2e-6, normwise(g32[k], g64[k])), k
    y_only, none = orc.block_step(x, w, shape["heads"], 1e-5)
    assert none is None and np.array_equal(y_only, y)


def test_oracle_attention_matches_block_heads_and_float64(orc):
    import torch
    rng = np.random.default_rng(4)
    bh, seq, dh = 3, 150, 32
    q, k, v, do = (rng.standard_normal((bh, seq, dh)).astype(np.float32) for _ in range(4))
    scale = float(np.float32(1.0 / np.sqrt(dh)))
    o, (dq, dk, dv) = orc.attention_causal(q, k, v, scale, do)
    Q, K, V = (torch.tensor(t, dtype=torch.float64, requires_grad=True) for t in (q, k, v))
    s = (Q @ K.transpose(-1, -2)) * scale
    s = torch.where(torch.ones(seq, seq, dtype=torch.bool).tril(), s,
                    torch.tensor(-float("inf"), dtype=torch.float64))
    out = torch.softmax(s, -1) @ V
    out.backward(torch.tensor(do, dtype=torch.float64))
    for got, ref in ((o, out), (dq, Q.grad), (dk, K.grad), (dv, V.grad)):
        ref = ref.detach().numpy()
        assert np.abs(got - ref).max() / np.abs(ref).max() <= 2e-6


def test_oracle_gelu_adjoint_is_the_derivative(orc):
    """The reverse sweep through the Phi graph equals g * (Phi(x) + x phi(x))
    to a few f32 ulps; at the guard values it follows the graph's selects."""
    from math import erfc, exp, pi, sqrt
    rng = np.random.default_rng(8)
    x = np.concatenate([rng.standard_normal(4000) * 3, [0.0, -0.0, 1e-30, -9.0, 9.0, 63.9, -63.9,
                                                        70.0, -70.0]]).astype(np.float32)
    g = rng.standard_normal(x.size).astype(np.float32)
    dx = orc.gelu_adjoint(x, g)
    for xi, gi, di in zip(x.astype(np.float64), g.astype(np.float64), dx.astype(np.float64)):
        der = 0.5 * erfc(-xi / sqrt(2.0)) + xi * exp(-0.5 * xi * xi) / sqrt(2.0 * pi)
        ref = gi * der
        assert abs(di - ref) <= 4e-7 * max(abs(gi), 1e-30) + 1e-37, (xi, gi, di, ref)


def test_crmath_checker_counts_mismatches(orc):
    """The exhaustive CORE-MATH comparison itself: CORE-MATH's own results
    pass, a planted wrong bit is found at its offset, NaNs match any NaN."""
    start = 0x3f800000 - 500
    bits = (np.arange(1000, dtype=np.uint64) + start).astype(np.uint32)
    xs = bits.view(np.float32)
    for op, f in ((0, orc.expf), (1, orc.logf)):
        want = np.array([f(float(v)) for v in xs], dtype=np.float32)
        assert orc.crmath_check_f32(op, start, want) == (0, -1)
        bad = want.copy()
        bad.view(np.uint32)[617] ^= 1
        assert orc.crmath_check_f32(op, start, bad) == (1, 617)
    nan_start = 0x7fc00000
    got = np.full(4, np.float32("nan"))
    got.view(np.uint32)[:] = 0xffc01234
    assert orc.crmath_check_f32(0, nan_start, got) == (0, -1)
