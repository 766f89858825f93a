"""Run by tests/test_lamp3_front_gpu.py in a fresh interpreter (not a test
module itself): the README MLP trained through the reference's own pybind11
module (rushlite._C, built by rushlite_b200/lamp3_cuda on the lmpb-served
core) on device=cuda and on device=cpu, from the same injected weights.
Prints one JSON line with the per-step losses, the parameters' relative
differences and how many lmpb kernels ran."""
from __future__ import annotations

import ctypes
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "rushlite_b200", "lamp3_cuda", "_build", "py"))
from rushlite import _C as R  # noqa: E402  (the reference's module)

DMAX = sys.float_info.max


def step(device, params, x, y, lr):
    """Linear-ReLU-Linear-Softmax under capture, loss
    (-y*log(p+1e-3)).sum(1).sum(0), backward, SGD on the host."""
    P = [R.Variable(p.tolist(), True, device, R.dtype.float32) for p in params]
    X = R.Variable(x.tolist(), False, device, R.dtype.float32)
    Y = R.Variable(y.tolist(), False, device, R.dtype.float32)
    R.set_capture_enabled(True)
    try:
        h = R.clamp(X @ P[0] + P[1], 0.0, DMAX)
        h = h @ P[2] + P[3]
        e = R.exp(h - R.max(h, 1))
        p = e / R.sum(e, 1)
    finally:
        R.set_capture_enabled(False)
    loss = R.sum(R.sum(-Y * R.log(p + 1e-3), 1), 0)
    loss.backward()
    new = []
    for q, p0 in zip(P, params):
        g = np.array(q.grad.tolist(), np.float64).reshape(p0.shape).astype(np.float32)
        new.append((p0 - np.float32(lr) * g).astype(np.float32))
    return new, loss.tolist()[0]


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-300))


def main():
    lmpb = ctypes.CDLL(os.path.join(ROOT, "rushlite_b200", "liblmpb.so"))
    lmpb.lmpb_kernel_launches.restype = ctypes.c_uint64
    rng = np.random.default_rng(0)
    x = rng.random((32, 256), dtype=np.float32)
    y = rng.random((32, 10), dtype=np.float32)
    prng = np.random.default_rng(5)
    params = []
    for i, o in ((256, 64), (64, 10)):
        params += [(prng.standard_normal((i, o)) / np.sqrt(i)).astype(np.float32),
                   (prng.standard_normal((o,)) / np.sqrt(i)).astype(np.float32)]
    pc = ph = params
    n0 = lmpb.lmpb_kernel_launches()
    steps = []
    for _ in range(3):
        pc, lc = step(R.device.cuda, pc, x, y, 1e-3)
        ph, lh = step(R.device.cpu, ph, x, y, 1e-3)
        steps.append({"loss_cuda": lc, "loss_cpu": lh})
    print(json.dumps({"cuda_available": bool(R.cuda.is_available()),
                      "lmpb_launches": int(lmpb.lmpb_kernel_launches() - n0), "steps": steps,
                      "param_rel_err": [rel(a, b) for a, b in zip(pc, ph)]}))


if __name__ == "__main__":
    main()
