"""Generate the golden vectors in this folder by running the reference library itself.

    python tests/golden/make_golden.py --ref <reference checkout>   (or SWVR_REFERENCE=<checkout>)

The reference (pengzhangzhi/swvr, pure Python on torch) is imported from ``--ref`` and run on
CPU. Each case stores its seeded inputs and the reference's outputs and gradients as a
compressed ``.npz``; bf16 tensors are stored as their exact fp32 values with a ``cdt`` tag.
These fixtures pin the numpy oracle (``oracle/swvr_oracle.py``) in
``tests/test_oracle_golden.py``; the GPU parity tests then compare the CUDA path with that
oracle. The reference is needed only to regenerate the fixtures, never at test time.

Case inputs follow the reference's own tests (tests/test_cpu.py:10-19 ``make``, seeds 0/1)
and BASELINE configs[0] (N=256, K=64, V=1000, D=16, fp32).
"""
import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
f64 = torch.float64


def _np(x):
    if x is None:
        return None
    return x.detach().to(torch.float64 if x.dtype == f64 else torch.float32).cpu().numpy()


def save(name, cdt, **arrays):
    out = {"cdt": np.array(cdt)}
    for k, v in arrays.items():
        if v is None:
            continue
        if isinstance(v, torch.Tensor):
            v = _np(v)
        out[k] = np.asarray(v)
    path = os.path.join(HERE, f"{name}.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({os.path.getsize(path) / 1024:.1f} KiB)")


def make(N=6, K=12, V=41, D=5, dtype=f64, bias=True, lead=None, seed=0):
    """tests/test_cpu.py:10-19."""
    g = torch.Generator().manual_seed(seed)
    shape = (*(lead or (N,)), K)
    t = lambda *s: torch.randn(*s, generator=g, dtype=f64).to(dtype=dtype)
    h, W, E = t(*shape), t(V, K), t(V, D)
    b = t(V) if bias else None
    for x in (h, W, E, b):
        if x is not None:
            x.requires_grad_(True)
    return h, W, E, b


def functional_grads(swvr, h, W, E, b, scale, chunk, seed=1):
    """tests/test_cpu.py:22-28: gradients of a seeded random linear functional of (O, LSE)."""
    O, lse = swvr.softmax_readout(h, W, E, b, logit_scale=scale, chunk_size=chunk)
    g = torch.Generator().manual_seed(seed)
    gO = torch.randn(O.shape, generator=g, dtype=f64).to(O)
    glse = torch.randn(lse.shape, generator=g, dtype=f64).to(lse)
    loss = (O * gO).sum() + (lse * glse).sum()
    xs = [x for x in (h, W, E, b) if x is not None]
    grads = torch.autograd.grad(loss, xs)
    out = dict(O=O, lse=lse, gO=gO, glse=glse)
    for name, gr in zip(["gh", "gW", "gE", "gb"], grads):
        out[name] = gr
    return out


def case_f64(swvr, name, h, W, E, b, scale, chunk):
    r = functional_grads(swvr, h, W, E, b, scale, chunk)
    save(name, "fp64", h=h, W=W, E=E, b=b, scale=scale, chunk=chunk, **r)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("SWVR_REFERENCE"),
                    help="checkout of the reference project (the directory holding swvr/); or SWVR_REFERENCE")
    args = ap.parse_args()
    if not args.ref:
        ap.error("pass --ref <reference checkout> or set SWVR_REFERENCE")
    sys.path.insert(0, args.ref)
    import swvr  # the reference library
    if not os.path.abspath(swvr.__file__).startswith(os.path.abspath(args.ref)):
        raise SystemExit(f"imported {swvr.__file__}, not the reference under {args.ref}")
    torch.manual_seed(0)

    # fp64 cases from the reference's CPU test-suite (test_cpu.py)
    h, W, E, b = make()
    case_f64(swvr, "f64_basic", h, W, E, b, 0.5, 8)
    h, W, E, b = make()
    case_f64(swvr, "f64_chunk1_nobias", h, W, E, None, 2.5, 1)
    h, W, E, b = make()
    with torch.no_grad():
        b[3] = 1e4
        b[7] = -1e4
    case_f64(swvr, "f64_large_logits", h, W, E, b, 1.0, 8)
    h, W, E, b = make(V=40)
    with torch.no_grad():
        b[:16] = float("-inf")
        b[30:] = float("-inf")
    case_f64(swvr, "f64_neginf_bias", h, W, E, b, 1.0, 8)
    h, W, E, b = make(N=1, V=2)
    case_f64(swvr, "f64_tiny_vocab", h, W, E, b, 1.0, 1)

    # MSE epilogue with weight, z-loss and every reduction (test_cpu.py:170-182)
    for reduction in ("mean", "sum", "none"):
        h, W, E, b = make(lead=(2, 3))
        g = torch.Generator().manual_seed(7)
        target = torch.randn(2, 3, 5, generator=g, dtype=f64).requires_grad_(True)
        weight = torch.tensor([[1., 0., 2.], [1., 1., 0.]], dtype=f64).requires_grad_(True)
        loss = swvr.softmax_readout_mse(h, W, E, target, b, weight=weight, reduction=reduction,
                                        z_loss_weight=0.1, logit_scale=0.5, chunk_size=8)
        gl = torch.ones_like(loss) if reduction != "none" else \
            torch.randn(loss.shape, generator=g, dtype=f64)
        grads = torch.autograd.grad(loss, (h, W, E, b, target, weight), gl)
        O, lse = swvr.softmax_readout(h, W, E, b, logit_scale=0.5, chunk_size=8)
        save(f"f64_mse_{reduction}", "fp64", h=h.reshape(6, 12), W=W, E=E, b=b, scale=0.5, chunk=8,
             target=target.reshape(6, 5), weight=weight.reshape(6), z=0.1, loss=loss,
             grad_loss=gl.reshape(-1), O=O.reshape(6, 5), lse=lse.reshape(6),
             gh=grads[0].reshape(6, 12), gW=grads[1], gE=grads[2], gb=grads[3],
             gtarget=grads[4].reshape(6, 5), gweight=grads[5].reshape(6))

    # fp32, N=256, K=64, V=1000, D=16; MSE fwd+bwd, no weight, z=0.
    g = torch.Generator().manual_seed(0)
    N, K, V, D = 256, 64, 1000, 16
    h = torch.randn(N, K, generator=g).requires_grad_(True)
    W = (torch.randn(V, K, generator=g) * K ** -0.5).requires_grad_(True)
    b = (torch.randn(V, generator=g) * 0.02).requires_grad_(True)
    E = (torch.randn(V, D, generator=g) * 0.02).requires_grad_(True)
    target = torch.randn(N, D, generator=g) * 0.02
    for chunk in (8192, 128):
        loss = swvr.softmax_readout_mse(h, W, E, target, b, chunk_size=chunk)
        grads = torch.autograd.grad(loss, (h, W, E, b))
        O, lse = swvr.softmax_readout(h, W, E, b, chunk_size=chunk)
        save(f"c0_fp32_chunk{chunk}", "fp32", h=h, W=W, E=E, b=b, scale=1.0, chunk=chunk,
             target=target, z=0.0, loss=loss, O=O, lse=lse,
             gh=grads[0], gW=grads[1], gE=grads[2], gb=grads[3])

    # bf16 through the reference's chunked CPU path (test_cpu.py:141-147 shapes)
    h, W, E, b = make(dtype=torch.bfloat16, K=32, V=300)
    r = functional_grads(swvr, h, W, E, b, 1.0, 64)
    save("bf16_small", "bf16", h=h, W=W, E=E, b=b, scale=1.0, chunk=64, **r)

    # bf16 with the GPU test-suite's scales (test_cuda.py:17-23), several chunks
    g = torch.Generator().manual_seed(0)
    N, K, V, D = 64, 128, 2000, 16
    t = lambda *s, sc=1.0: (sc * torch.randn(*s, generator=g)).to(torch.bfloat16)
    h, W, E, b = t(N, K), t(V, K, sc=3 / K ** 0.5), t(V, D), t(V, sc=0.5)
    for x in (h, W, E, b):
        x.requires_grad_(True)
    r = functional_grads(swvr, h, W, E, b, 0.8, 512)
    save("bf16_medium", "bf16", h=h, W=W, E=E, b=b, scale=0.8, chunk=512, **r)


if __name__ == "__main__":
    main()
