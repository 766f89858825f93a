"""The multi-rank paths on the product kernels: two ranks (processes), gloo
process group, both on GPU 0, calling rushlite_b200 and
rushlite_b200.distributed.all_reduce_ on CUDA backend tensors.

* C3 dim 0, row-sharded: each rank reduces its row block with the product's
  reduction kernel, then one all-reduce combines the [1, 4096] partials.  The
  result must equal the unsharded reduction: bit-exact for max, min and the
  int32 sum, within 1e-5 for the float sum (the partial order differs).
  Dim 1 needs no exchange: each rank's rows equal the unsharded rows exactly.
* Data-parallel MLP step (C5-shaped, narrower): each rank runs forward and
  backward on its half of the batch, gradients are summed by all-reduce, and
  the result must equal the single-rank full-batch gradients within 1e-5;
  the loss partials summed equal the full-batch loss within 1e-5.

gloo all-reduces CUDA tensors through host staging, so the two ranks never
wait on each other on the device; each rank's kernels finish before its
collective starts.
"""
from __future__ import annotations

import multiprocessing as mp
import os
import socket
import sys
import traceback

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DMAX = sys.float_info.max


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _mlp_grads(rsl, params, x, y):
    P = [rsl.Variable(p, requires_grad=True) for p in params]
    X, Y = rsl.Variable(x), rsl.Variable(y)
    with rsl.capture_on():
        h = X
        n = len(P) // 2
        for i in range(n):
            h = rsl.matmul(h, P[2 * i]) + P[2 * i + 1]
            if i < n - 1:
                h = rsl.clamp(h, 0, DMAX)
        m = rsl.max(h, 1)
        e = rsl.exp(h - m)
        p = e / rsl.sum(e, 1)
    loss = rsl.sum(rsl.sum(-Y * rsl.log(p + 1e-3), 1), 0)
    loss.backward()
    return loss, P


def _worker(rank, world, port, q, mode="gloo"):
    try:
        sys.path.insert(0, ROOT)
        dev = rank if mode == "lmpb" else 0
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                          WORLD_SIZE=str(world), LOCAL_RANK=str(dev))
        import torch
        import torch.distributed as dist

        torch.cuda.set_device(dev)
        import rushlite_b200 as rsl
        from rushlite_b200 import distributed as D

        rsl.cuda.set_device(dev)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        if mode == "lmpb":
            assert D.init_comm()  # the library's NCCL communicator carries all_reduce_
        out = {}
        # --- C3, row-sharded
        R, Cn = 4096, 4096
        rng = np.random.default_rng(3)
        xf = rng.standard_normal((R, Cn), dtype=np.float32)
        xi = rng.integers(-1000, 1001, (R, Cn)).astype(np.int32)
        r0, r1 = D.shard_rows(R, rank, world)
        for name, x, fn, op in [("sum", xf, rsl.sum, "sum"), ("max", xf, rsl.max, "max"),
                                ("min", xf, rsl.min, "min"), ("isum", xi, rsl.sum, "sum")]:
            dt = rsl.dtype.int32 if x.dtype == np.int32 else rsl.dtype.float32
            part = fn(rsl.Variable(np.ascontiguousarray(x[r0:r1]), dtype=dt), 0)
            D.all_reduce_(part.data, op)
            full = fn(rsl.Variable(x, dtype=dt), 0)
            out[name + "_dim0"] = (part.numpy(), full.numpy())
            loc = fn(rsl.Variable(np.ascontiguousarray(x[r0:r1]), dtype=dt), 1)
            out[name + "_dim1"] = (loc.numpy(), fn(rsl.Variable(x, dtype=dt), 1).numpy()[r0:r1])
        # --- DP step: half batch per rank, gradient all-reduce
        dims = [512, 512, 512, 512, 100]
        B = 1024
        prng = np.random.default_rng(5)
        params = []
        for i in range(len(dims) - 1):
            params.append((prng.standard_normal((dims[i], dims[i + 1])) / np.sqrt(dims[i])).astype(np.float32))
            params.append((prng.standard_normal((dims[i + 1],)) / np.sqrt(dims[i])).astype(np.float32))
        xb = prng.standard_normal((B, dims[0])).astype(np.float32)
        yb = np.zeros((B, dims[-1]), np.float32)
        yb[np.arange(B), prng.integers(0, dims[-1], B)] = 1
        b0, b1 = D.shard_rows(B, rank, world)
        loss, P = _mlp_grads(rsl, params, np.ascontiguousarray(xb[b0:b1]), np.ascontiguousarray(yb[b0:b1]))
        for p in P:
            D.all_reduce_(p.grad, "sum")
        D.all_reduce_(loss.data, "sum")
        loss1, P1 = _mlp_grads(rsl, params, xb, yb)
        out["dp_loss"] = (loss.numpy(), loss1.numpy())
        for i, (p, p1) in enumerate(zip(P, P1)):
            out[f"dp_grad{i}"] = (p.grad.numpy(), p1.grad.numpy())
        if mode == "lmpb":
            # the fused reduce + all-reduce over peer memory: one kernel, the
            # result over all ranks' rows, the same bits on every rank
            assert D.init_peer()
            from rushlite_b200 import capi as _capi

            for name, x, op in [("sum", xf, "sum"), ("max", xf, "max"), ("min", xf, "min"), ("isum", xi, "sum")]:
                dt = rsl.dtype.int32 if x.dtype == np.int32 else rsl.dtype.float32
                v = rsl.Variable(np.ascontiguousarray(x[r0:r1]), dtype=dt)
                o = rsl.Variable(np.zeros((1, x.shape[1]), x.dtype), dtype=dt)
                v.realize()
                o.realize()
                rsl.cuda.synchronize()
                n0 = _capi.kernel_launches()
                got = D.reduce_allreduce(v, op, out=o)
                launched = _capi.kernel_launches() - n0
                fn = {"sum": rsl.sum, "max": rsl.max, "min": rsl.min}[op]
                out["peer_" + name] = (got.numpy(), fn(rsl.Variable(x, dtype=dt), 0).numpy(), launched)
            _capi.device_error()
            _capi.peer_close()
            # overlapped all-reduce on the communication stream, then join
            g = [p.grad for p in P1]
            before = [x.numpy() for x in g]
            D.all_reduce_many(g, "sum", overlap=True)
            D.join()
            out["overlap"] = [(x.numpy(), 2 * b) for x, b in zip(g, before)]
            from rushlite_b200 import capi

            capi.comm_destroy()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, out, None))
    except Exception:
        q.put((rank, None, traceback.format_exc()))


@pytest.mark.parametrize("mode", ["gloo", "lmpb"])
def test_two_ranks_on_product_kernels(cuda, mode):
    """gloo: both ranks on GPU 0, all-reduce through torch's gloo group.
    lmpb: one rank per GPU (needs two), all-reduce through the library's own
    NCCL communicator (lmpb_allreduce), blocking and overlapped."""
    from tests.util import assert_bitexact, rel_err

    if mode == "lmpb" and cuda.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, mode)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(2):
            rank, out, err = q.get(timeout=600)
            assert err is None, f"rank {rank}:\n{err}"
            results[rank] = out
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for rank, out in results.items():
        for name in ("max", "min", "isum"):
            assert_bitexact(*out[name + "_dim0"], f"rank {rank} {name} dim0")
            assert_bitexact(*out[name + "_dim1"], f"rank {rank} {name} dim1")
        assert rel_err(*out["sum_dim0"]) <= 1e-5
        assert_bitexact(*out["sum_dim1"], f"rank {rank} sum dim1")
        assert rel_err(*out["dp_loss"]) <= 1e-5
        for k in [k for k in out if k.startswith("dp_grad")]:
            g, g1 = out[k]
            assert rel_err(g, g1) <= 1e-5, (rank, k, rel_err(g, g1))
        for got, want in out.get("overlap", []):
            assert_bitexact(got, want, f"rank {rank} overlapped all-reduce")
        for name in ("sum", "max", "min", "isum"):
            if "peer_" + name not in out:
                continue
            got, want, launched = out["peer_" + name]
            assert launched == 1, (name, launched)  # one fused kernel, no fallback
            if name == "sum":
                assert rel_err(got, want) <= 1e-5
            else:
                assert_bitexact(got, want, f"rank {rank} peer {name}")
    if mode == "lmpb":
        for name in ("sum", "max", "min", "isum"):
            assert_bitexact(results[0]["peer_" + name][0], results[1]["peer_" + name][0], f"peer {name} across ranks")
