"""Multi-GPU plumbing: one process per GPU, torch.distributed for the
process group (NCCL over NVLink on GPUs, gloo on CPU).

The Lamp3 paths shard as follows:
* elementwise / fused chains and last-axis reductions: rows are independent,
  each rank owns a contiguous row block (no collective);
* leading-axis reductions: each rank reduces its row block, then one
  all-reduce (sum / max / min) of the small partial;
* data-parallel training: replicated parameters, per-rank batch slice,
  gradients summed with all-reduce (the loss is a sum, so no averaging).
"""
from __future__ import annotations

import os

import numpy as np

_OPS = {"sum": "SUM", "max": "MAX", "min": "MIN"}


def env():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def init(backend: str | None = None):
    """Initialises the default process group from the torchrun environment."""
    import torch
    import torch.distributed as dist

    rank, world, local = env()
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    if backend == "nccl":
        torch.cuda.set_device(local)
        from . import cuda

        cuda.set_device(local)
    if world > 1 and not dist.is_initialized():
        kw = {"device_id": torch.device("cuda", local)} if backend == "nccl" else {}
        dist.init_process_group(backend, **kw)
    return rank, world, local


def shard_rows(n: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous block of rows [r0, r1) owned by `rank`; blocks differ by at most one row."""
    base, extra = divmod(n, world)
    r0 = rank * base + min(rank, extra)
    return r0, r0 + base + (1 if rank < extra else 0)


def all_reduce_(x, op: str = "sum"):
    """In-place all-reduce of a backend tensor (rushlite_b200 _Tensor on CUDA,
    zero-copy through __cuda_array_interface__) or of a NumPy array (gloo)."""
    import torch
    import torch.distributed as dist

    if not dist.is_initialized() or dist.get_world_size() == 1:
        return x
    rop = getattr(dist.ReduceOp, _OPS[op])
    if isinstance(x, np.ndarray):
        dist.all_reduce(torch.from_numpy(x), op=rop)
    else:
        dist.all_reduce(torch.as_tensor(x, device="cuda"), op=rop)
    return x


def max_over_ranks(value: float) -> float:
    import torch
    import torch.distributed as dist

    if not dist.is_initialized() or dist.get_world_size() == 1:
        return value
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([value], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
