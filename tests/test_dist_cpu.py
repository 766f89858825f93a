"""The multi-rank host logic on CPU: two gloo ranks shard a [rows, cols]
array by rows, reduce their blocks with the CPU restatement, and all-reduce
the leading-axis partials; the result must equal the single-process
reduction (bit-exact for max/min/int32, within tolerance for a float sum).
Also checks the row partition covers every row exactly once."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from rushlite_b200.distributed import shard_rows


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import torch.distributed as dist

    from oracle import port as oport
    from rushlite_b200 import distributed as D

    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(0)
        xf = rng.standard_normal((1001, 37)).astype(np.float32)
        xi = rng.integers(-1000, 1001, (1001, 37)).astype(np.int32)
        r0, r1 = D.shard_rows(1001, rank, world)
        out = {}
        for name, x, op, code in [("sum_f", xf, "sum", 0), ("max_f", xf, "max", 1), ("min_f", xf, "min", 2),
                                  ("sum_i", xi, "sum", 0)]:
            part = oport.reduce(code, np.ascontiguousarray(x[r0:r1]), 0)
            D.all_reduce_(part, op)
            out[name] = part
        # dim 1 needs no exchange: gather the row blocks for the check
        loc = oport.reduce(0, np.ascontiguousarray(xf[r0:r1]), 1)
        full = np.zeros((1001, 1), np.float32)
        full[r0:r1] = loc
        D.all_reduce_(full, "sum")
        out["sum_dim1"] = full
        out["t"] = D.max_over_ranks(float(rank + 1))
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_row_partition_covers_every_row():
    for n in (0, 1, 7, 1001, 8192):
        for w in (1, 2, 3, 8):
            seen = []
            for r in range(w):
                a, b = shard_rows(n, r, w)
                seen += list(range(a, b))
            assert seen == list(range(n))


def test_two_gloo_ranks_sharded_reductions():
    import multiprocessing as mp

    from oracle import port as oport

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    rng = np.random.default_rng(0)
    xf = rng.standard_normal((1001, 37)).astype(np.float32)
    xi = rng.integers(-1000, 1001, (1001, 37)).astype(np.int32)
    for r in (0, 1):
        o = res[r]
        np.testing.assert_array_equal(o["max_f"], oport.reduce(1, xf, 0))
        np.testing.assert_array_equal(o["min_f"], oport.reduce(2, xf, 0))
        np.testing.assert_array_equal(o["sum_i"], oport.reduce(0, xi, 0))
        want = oport.reduce(0, xf, 0).astype(np.float64)
        assert np.max(np.abs(o["sum_f"] - want)) / np.max(np.abs(want)) <= 1e-5
        np.testing.assert_array_equal(o["sum_dim1"], oport.reduce(0, xf, 1))
        assert o["t"] == 2.0
