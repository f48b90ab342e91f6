"""Data-parallel and vmap sharding across the GPUs of one box.

One process per GPU (torch.distributed over NCCL for the plumbing).  Two
ways the hot path shards, both along the batch axis the reference's vmap /
data-parallel plan names (crates/chelis-ir-core/src/vmap.rs:9-56,
spec/design/chelis_project_plan.md:1188-1192):

* vmap'd programs (batched GEMM, covariance / risk): batch items are
  independent; every rank computes a contiguous shard, no collective.
* data-parallel training step (transformer block): every rank runs forward +
  reverse mode on its batch shard; the weight gradients, packed in one flat
  buffer, are summed across ranks with a single all-reduce.  The loss is a
  sum over samples, so the sum of the shard gradients is the full-batch
  gradient (no rescaling).
"""
from __future__ import annotations

import ctypes

import torch

from . import lib as L

_native = [False]


def shard(n: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [start, stop) of n items for `rank`; shard sizes differ by at
    most one and the shards tile [0, n) in rank order."""
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


class FlatGrads:
    """Gradient tensors that are views into one flat buffer, so a single
    collective reduces all of them."""

    def __init__(self, shapes: dict[str, tuple[int, ...]], device, dtype=torch.float32):
        total = 0
        self.offsets = {}
        for name, shp in shapes.items():
            n = 1
            for s in shp:
                n *= s
            # 64-element alignment keeps every view 256-byte aligned
            self.offsets[name] = (total, n, shp)
            total += (n + 63) // 64 * 64
        self.flat = torch.zeros(total, dtype=dtype, device=device)
        self.views = {name: self.flat[o:o + n].view(shp) for name, (o, n, shp) in self.offsets.items()}

    def __getitem__(self, name):
        return self.views[name]


def native_init(world: int, rank: int) -> None:
    """Open the library's own NCCL communicator (chelis_cuda_dp_init) over the
    ranks of the running torch.distributed group: rank 0 makes the id, the
    group's broadcast hands it to the others."""
    import torch.distributed as dist
    buf = (ctypes.c_uint8 * 128)()
    if rank == 0:
        L.call("chelis_cuda_dp_unique_id", buf)
    obj = [bytes(buf)]
    dist.broadcast_object_list(obj, src=0)
    ctypes.memmove(buf, obj[0], 128)
    L.call("chelis_cuda_dp_init", world, rank, buf)
    _native[0] = True


def native_finalize(abort: bool = False) -> None:
    if _native[0]:
        _native[0] = False
        L.call("chelis_cuda_dp_finalize", 1 if abort else 0)


def allreduce_sum(flat: torch.Tensor, world: int) -> None:
    """Sum `flat` over the ranks, in place, on the current stream.  Device
    tensors go through the library's communicator (native_init must have
    opened it; otherwise this raises: there is no library-free path for
    GPU data).  Host tensors, the CPU (gloo) form of the same host logic,
    go through torch.distributed."""
    if world <= 1:
        return
    if flat.is_cuda:
        if not _native[0]:
            raise RuntimeError("dp.allreduce_sum on a CUDA tensor needs native_init "
                               "(the library's NCCL communicator)")
        from . import ops
        ops._prepare(flat)
        dt = {torch.float32: L.DTYPE_F32, torch.float64: L.DTYPE_F64,
              torch.int64: L.DTYPE_I64, torch.int32: L.DTYPE_I32}[flat.dtype]
        L.call("chelis_cuda_dp_allreduce_sum", dt, flat.data_ptr(), flat.numel())
        return
    import torch.distributed as dist
    dist.all_reduce(flat, op=dist.ReduceOp.SUM)
