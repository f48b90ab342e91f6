"""The N > 1 plumbing on CPU with two gloo ranks: batch sharding and the
single flat-buffer gradient all-reduce give the full-batch gradient, and
vmap shards tile the batch.  The per-shard computation here is a float64
torch stand-in for the device step (the sharding and collective logic is
what is under test)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from chelis_b200 import dp


def test_shards_tile_the_batch():
    for n in (0, 1, 7, 8, 65536):
        for world in (1, 2, 3, 4, 8):
            spans = [dp.shard(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1


def _loss_grads(x, w1, w2):
    w1 = w1.clone().requires_grad_(True)
    w2 = w2.clone().requires_grad_(True)
    y = torch.tanh(x @ w1) @ w2
    y.sum().backward()
    return w1.grad, w2.grad


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    g = torch.Generator().manual_seed(0)
    x = torch.randn(8, 16, generator=g, dtype=torch.float64)
    w1 = torch.randn(16, 32, generator=g, dtype=torch.float64)
    w2 = torch.randn(32, 4, generator=g, dtype=torch.float64)
    a, b = dp.shard(x.shape[0], world, rank)
    grads = dp.FlatGrads({"w1": (16, 32), "w2": (32, 4)}, "cpu", torch.float64)
    g1, g2 = _loss_grads(x[a:b], w1, w2)
    grads["w1"].copy_(g1)
    grads["w2"].copy_(g2)
    dp.allreduce_sum(grads.flat, world)
    if rank == 0:
        f1, f2 = _loss_grads(x, w1, w2)
        q.put((float((grads["w1"] - f1).abs().max()), float((grads["w2"] - f2).abs().max())))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_gradient_allreduce_equals_full_batch():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    e1, e2 = q.get(timeout=10)
    assert e1 < 1e-12 and e2 < 1e-12


def test_c_abi_shard_matches_host_rule():
    import ctypes
    from chelis_b200 import lib as L
    lib = L.load()
    a, b = ctypes.c_int64(), ctypes.c_int64()
    for n in (0, 1, 7, 65536, 1000003):
        for world in (1, 2, 3, 8):
            for r in range(world):
                assert lib.chelis_cuda_dp_shard(n, world, r, ctypes.byref(a), ctypes.byref(b)) == 0
                assert (a.value, b.value) == dp.shard(n, world, r)
    assert lib.chelis_cuda_dp_shard(5, 2, 2, ctypes.byref(a), ctypes.byref(b)) == 1
    # no communicator: the all-reduce refuses, the world is one rank
    w, r = ctypes.c_int32(), ctypes.c_int32()
    assert lib.chelis_cuda_dp_world(ctypes.byref(w), ctypes.byref(r)) == 0 and (w.value, r.value) == (1, 0)
    assert lib.chelis_cuda_dp_allreduce_sum(L.DTYPE_F32, None, 4) == 1
    assert "dp_init" in L.last_error()
    assert lib.chelis_cuda_dp_allreduce_sum(L.DTYPE_BOOL, None, 4) == 4
    assert lib.chelis_cuda_dp_finalize(0) == 0
