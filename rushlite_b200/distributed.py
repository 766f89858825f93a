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


def init_comm() -> bool:
    """Creates the library's own device communicator (lmpb_comm_init, NCCL)
    for the torch.distributed job this process belongs to: rank 0 makes the id,
    the process group broadcasts it.  Collectives through it run on the host
    layer's stream, so they order after the kernels that feed them and can be
    recorded into a CUDA graph with the step.  Returns False for one rank."""
    import torch.distributed as dist

    from . import capi

    if not dist.is_initialized() or dist.get_world_size() == 1:
        return False
    if capi.comm_size():
        return True
    box = [capi.comm_unique_id() if dist.get_rank() == 0 else None]
    dist.broadcast_object_list(box, src=0)
    capi.comm_init(box[0], dist.get_world_size(), dist.get_rank())
    return True


def init_peer() -> bool:
    """Maps every rank's exchange region into this process (CUDA IPC over
    NVLink; handles exchanged through the torch.distributed group) for the
    fused leading-axis reduce + all-reduce (reduce_allreduce).  One rank per
    GPU.  Returns False for one rank."""
    import torch.distributed as dist

    from . import capi

    if not dist.is_initialized() or dist.get_world_size() == 1 or os.environ.get("LMPB_PEER") == "0":
        return False  # LMPB_PEER=0: A/B switch, keep the NCCL route
    if capi.peer_size():
        return True
    mine = capi.peer_export()
    handles = [None] * dist.get_world_size()
    dist.all_gather_object(handles, mine)
    capi.peer_import(handles, dist.get_rank())
    dist.barrier()
    return True


def reduce_allreduce(x, op: str = "sum", out=None):
    """Sum / max / min / prod over axis 0 of a rank's row block of a 2-D
    Variable, combined over all ranks: the result of the whole row-partitioned
    tensor, identical on every rank.  With a peer context (init_peer) it is one
    kernel (lmpb_reduce_allreduce), written into `out` when given; otherwise,
    or for a shape outside that kernel, the local reduction followed by
    all_reduce_."""
    from . import _C, capi

    fn = {"sum": _C.sum, "max": _C.max, "min": _C.min, "prod": _C.prod}[op]
    if capi.peer_size() and len(x.shape) == 2:
        if out is None:  # `out`: a [1, cols] Variable of x's dtype to write into
            out = _C.zeros([1, x.shape[1]], False, _C.device.cuda, x.dtype)
        st = capi.reduce_allreduce(capi.REDUCE_OPS[op], int(x.dtype.value), x.data.data_ptr(), list(x.shape), 0,
                                   out.data.data_ptr(), _stream())
        if st == 0:
            return out
    r = fn(x, 0)
    all_reduce_(r.data, op)
    return r


def _stream():
    from . import _C

    return _C.cuda.current_stream()


def all_reduce_many(tensors, op: str = "sum", overlap: bool = False):
    """In-place all-reduce of backend CUDA tensors of one dtype through the
    library's communicator, as one grouped launch.  overlap=True runs it on
    the communication stream (ordered after the work queued so far), so the
    kernels that follow proceed; join() orders the host layer's stream after it."""
    from . import capi

    if not tensors:
        return
    dt = int(tensors[0].dtype.value)
    ptrs = [t.data_ptr() for t in tensors]
    counts = [int(np.prod(t.shape)) for t in tensors]
    capi.allreduce(dt, ptrs, counts, capi.REDUCE_OPS[op], overlap, _stream())


def join():
    """Makes the host layer's stream wait for every overlapped all-reduce."""
    from . import capi

    capi.comm_join(_stream())


def shard_rows(n: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous block of rows [r0, r1) owned by `rank`; blocks differ by at most one row."""
    base, extra = divmod(n, world)
    r0 = rank * base + min(rank, extra)
    return r0, r0 + base + (1 if rank < extra else 0)


def all_reduce_(x, op: str = "sum"):
    """In-place all-reduce of a backend tensor (rushlite_b200 _Tensor on CUDA)
    or of a NumPy array (gloo).  A CUDA tensor goes through the library's
    communicator when init_comm() created one, else through torch.distributed
    (zero-copy via __cuda_array_interface__)."""
    import torch
    import torch.distributed as dist

    if not dist.is_initialized() or dist.get_world_size() == 1:
        return x
    if not isinstance(x, np.ndarray):
        from . import capi

        if capi.comm_size():
            all_reduce_many([x], op)
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
