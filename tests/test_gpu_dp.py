"""The library's own NCCL communicator on two GPUs: every rank sums a buffer
whose values are exact in f32 / f64 / i64, through chelis_cuda_dp_*; the
data-parallel gradient of the sharded batch equals the full-batch one, also
for the transformer block with its gradients reduced during the reverse
pass (chelis_cuda_block_step_dp)."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _worker(rank, world, port, q):
    try:
        import torch
        import torch.distributed as dist
        from chelis_b200 import dp, ops
        torch.cuda.set_device(rank)
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        dp.native_init(world, rank)
        out = {}
        for dtype in (torch.float32, torch.float64, torch.int64):
            x = (torch.arange(1 << 20, device="cuda") % 1000 + rank * 7).to(dtype)
            dp.allreduce_sum(x, world)
            torch.cuda.synchronize()
            ref = sum((torch.arange(1 << 20, device="cuda") % 1000 + r * 7) for r in range(world)).to(dtype)
            out[str(dtype)] = bool(torch.equal(x, ref))
        # data-parallel gradient: sharded matmul adjoint summed over ranks
        g = torch.Generator(device="cpu").manual_seed(0)
        xb = torch.randn(64, 32, generator=g).cuda()
        dyb = torch.randn(64, 16, generator=g).cuda()
        a, b = dp.shard(64, world, rank)
        dw = ops.matmul(xb[a:b].contiguous(), dyb[a:b].contiguous(), trans_a=True)
        dp.allreduce_sum(dw, world)
        full = ops.matmul(xb, dyb, trans_a=True)
        torch.cuda.synchronize()
        out["grad"] = float((dw - full).abs().max() / full.abs().max())
        # transformer block: each rank steps its half of the batch with the
        # gradients reduced during the reverse pass; they must equal the
        # full-batch gradients (one GPU, same kernels) within f32 rel 1e-5
        from chelis_b200 import workloads as W
        shape = dict(batch=2, seq=128, d_model=128, heads=2, d_ff=256)
        xn, dyn, wn = W.block_inputs(seed=21, **shape)
        wt = {k: torch.from_numpy(v).cuda() for k, v in wn.items()}
        X, DY = torch.from_numpy(xn).cuda(), torch.from_numpy(dyn).cuda()
        a, b = dp.shard(2, world, rank)
        grads = dp.FlatGrads({"d" + k: tuple(wt[k].shape) for k in ops.BLOCK_WEIGHTS}, "cuda")
        res = {k: grads[k] for k in grads.views}
        part = ops.block_step(X[a:b].contiguous(), wt, 2, 1e-5, DY[a:b].contiguous(), out=res,
                              reduce_grads=True)
        ref = ops.block_step(X, wt, 2, 1e-5, DY)
        torch.cuda.synchronize()
        out["block"] = max(float((part[k] - ref[k]).abs().max() / ref[k].abs().max())
                           for k in grads.views)
        out["block_dx"] = float((part["dx"] - ref["dx"][a:b]).abs().max() / ref["dx"].abs().max())
        dp.native_finalize()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, out))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, repr(e)))


def test_two_rank_native_allreduce():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(2):
        rank, out = q.get(timeout=240)
        results[rank] = out
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    for rank in (0, 1):
        out = results[rank]
        assert isinstance(out, dict), out
        assert out["torch.float32"] and out["torch.float64"] and out["torch.int64"]
        assert out["grad"] <= 1e-5
        assert out["block"] <= 1e-5, out["block"]
        assert out["block_dx"] <= 1e-5, out["block_dx"]
