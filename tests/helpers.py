"""Shared helpers for the test-suite: seeded inputs, error metrics, oracle wrappers."""
import os

import numpy as np
import torch

from oracle import swvr_oracle as orc
from tests.conftest import GOLDEN

f64 = torch.float64
CDT = {torch.bfloat16: "bf16", torch.float16: "fp16", torch.float32: "fp32", torch.float64: "fp64"}


def load_golden(name):
    z = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    return {k: z[k] for k in z.files}


def rel_err(a, r):
    """Norm-wise relative error (the reference's test_cuda.py:33-35)."""
    a = a.detach().double().cpu() if isinstance(a, torch.Tensor) else torch.as_tensor(np.asarray(a, np.float64))
    r = r.detach().double().cpu() if isinstance(r, torch.Tensor) else torch.as_tensor(np.asarray(r, np.float64))
    return ((a - r).norm() / r.norm().clamp_min(1e-30)).item()


def npy(t):
    return t.detach().to(torch.float64).cpu().numpy() if t.dtype != f64 else t.detach().cpu().numpy()


def make_cpu(N=6, K=12, V=41, D=5, dtype=f64, bias=True, lead=None, seed=0, device="cuda"):
    """The reference's CPU-suite inputs (tests/test_cpu.py:10-19), placed on ``device``."""
    g = torch.Generator().manual_seed(seed)
    shape = (*(lead or (N,)), K)
    t = lambda *s: torch.randn(*s, generator=g, dtype=f64).to(device=device, dtype=dtype)
    h, W, E = t(*shape), t(V, K), t(V, D)
    b = t(V) if bias else None
    for x in (h, W, E, b):
        if x is not None:
            x.requires_grad_(True)
    return h, W, E, b


def make_gpu(N, K, V, D, dtype, bias=True, seed=0):
    """The reference's GPU-suite inputs (tests/test_cuda.py:17-23): W scale 3/sqrt(K), b 0.5.

    Generated on CPU with a seeded generator so the oracle sees identical values."""
    g = torch.Generator().manual_seed(seed)
    t = lambda *s, scale=1.0: (scale * torch.randn(*s, generator=g)).to(dtype)
    h, W, E = t(N, K), t(V, K, scale=3 / K ** 0.5), t(V, D)
    b = t(V, scale=0.5) if bias else None
    return [x.cuda().requires_grad_(True) if x is not None else None for x in (h, W, E, b)]


def functional_grads(fn, inputs, seed=1):
    """Gradients of a seeded random linear functional of fn's outputs (test_cpu.py:22-28)."""
    outs = fn(*inputs)
    g = torch.Generator().manual_seed(seed)
    ws = [torch.randn(o.shape, generator=g, dtype=f64).to(o) for o in outs]
    loss = sum((o * w).sum() for o, w in zip(outs, ws))
    xs = []
    for x in inputs:
        if x is not None and x.requires_grad and all(x is not y for y in xs):
            xs.append(x)
    return outs, ws, torch.autograd.grad(loss, xs, allow_unused=True)


def oracle_eager(h, W, E, b, scale, gO, glse):
    """fp64 eager oracle outputs and grads (swvr/reference.py:5-14 and its gradient)."""
    args = [npy(h), npy(W), npy(E), None if b is None else npy(b)]
    O, lse = orc.softmax_readout_reference(*args, logit_scale=scale)
    grads = orc.readout_grads(*args, npy(gO), npy(glse), logit_scale=scale)
    return O, lse, grads
