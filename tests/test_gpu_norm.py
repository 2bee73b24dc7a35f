"""GPU parity of the fused RMSNorm producer of h (``rmsnorm_softmax_readout[_mse]``).

Checkers: the fp64 oracle chain (``rmsnorm_forward`` -> the eager readout oracle -> its
gradients -> ``rmsnorm_backward``), at 1e-10 for fp64, 1e-4 for fp32 and 2e-2 (LSE 1e-2
absolute) for bf16; and the unfused composition ``torch.nn.functional.rms_norm`` ->
``softmax_readout`` on the same inputs.  Also: no weight, leading dims, a hidden size that
is not a multiple of 8, an empty batch, autocast over fp32 parameters, the module with
``norm=nn.RMSNorm``, ``torch.compile(fullgraph=True)``, activation checkpointing and
bit-identical repeat runs.
"""
import numpy as np
import pytest
import torch

import swvr_b200 as swvr
from oracle import swvr_oracle as orc
from tests.helpers import npy, rel_err

pytestmark = pytest.mark.gpu


def _inputs(N, K, V, D, dtype, seed=0, affine=True, lead=None):
    g = torch.Generator().manual_seed(seed)
    t = lambda *s, scale=1.0: (scale * torch.randn(*s, generator=g)).to(dtype)
    x = t(*(lead or (N,)), K, scale=2.0)
    w = (1.0 + 0.3 * torch.randn(K, generator=g)).to(dtype) if affine else None
    W, E, b = t(V, K, scale=3 / K ** 0.5), t(V, D), t(V, scale=0.5)
    return [None if v is None else v.cuda().requires_grad_(True) for v in (x, w, W, E, b)]


def _oracle(x, w, W, E, b, eps, scale, gO, glse):
    """Outputs and gradients of the fused op from the fp64 oracle chain."""
    K = x.shape[-1]
    x2 = npy(x).reshape(-1, K)
    wn = None if w is None else npy(w)
    h, _ = orc.rmsnorm_forward(x2, wn, eps)
    O, lse = orc.softmax_readout_reference(h, npy(W), npy(E), npy(b), logit_scale=scale)
    gh, gW, gE, gb = orc.readout_grads(h, npy(W), npy(E), npy(b), npy(gO).reshape(O.shape), npy(glse).reshape(-1),
                                       logit_scale=scale)
    gx, gw = orc.rmsnorm_backward(gh, x2, wn, eps)
    return O, lse, [gx.reshape(x.shape), gw, gW, gE, gb]


def _run(x, w, W, E, b, eps, scale, gO, glse, chunk=1000):
    O, lse = swvr.rmsnorm_softmax_readout(x, w, W, E, b, eps=eps, logit_scale=scale, chunk_size=chunk)
    leaves = [v for v in (x, w, W, E, b) if v is not None]
    grads = torch.autograd.grad((O * gO).sum() + (lse * glse).sum(), leaves)
    it = iter(grads)
    return O, lse, [next(it) if v is not None else None for v in (x, w, W, E, b)]


@pytest.mark.parametrize("dtype,tol", [(torch.float64, 1e-10), (torch.float32, 1e-4), (torch.bfloat16, 2e-2)])
@pytest.mark.parametrize("affine", [True, False])
def test_fused_norm_matches_the_oracle(dtype, tol, affine):
    N, K, V, D, eps, scale = 300, 256, 3001, 48, 1e-5, 0.7
    x, w, W, E, b = _inputs(N, K, V, D, dtype, affine=affine)
    g = torch.Generator().manual_seed(5)
    gO, glse = torch.randn(N, D, generator=g).cuda(), torch.randn(N, generator=g).cuda()
    O, lse, grads = _run(x, w, W, E, b, eps, scale, gO, glse)
    Or, lr, gr = _oracle(x, w, W, E, b, eps, scale, gO, glse)
    assert rel_err(O, Or) < tol and rel_err(lse, lr) < tol
    # LSE near 10: 1e-4 absolute is the fp32 contract's 1e-5 relative (test_cuda.py:65)
    assert np.max(np.abs(npy(lse) - lr)) < {torch.bfloat16: 1e-2, torch.float32: 1e-4, torch.float64: 1e-9}[dtype]
    for name, a, r in zip(["gx", "gw", "gW", "gE", "gb"], grads, gr):
        if r is None:
            assert a is None, name
            continue
        assert a.dtype == dtype and torch.isfinite(a).all(), name
        assert rel_err(a, r) < tol, (name, rel_err(a, r))


def test_fused_norm_agrees_with_the_unfused_composition():
    """bf16: rms_norm then softmax_readout (torch's norm, the library's readout) on the same
    inputs; the fused path rounds h once and feeds the norm's backward the fp32 dh."""
    N, K, V, D, eps = 1000, 512, 20011, 64, 1e-6
    x, w, W, E, b = _inputs(N, K, V, D, torch.bfloat16, seed=2)
    g = torch.Generator().manual_seed(6)
    gO, glse = torch.randn(N, D, generator=g).cuda(), torch.randn(N, generator=g).cuda()
    O, lse, grads = _run(x, w, W, E, b, eps, 1.0, gO, glse, chunk=8192)
    xs = [v.detach().clone().requires_grad_(True) for v in (x, w, W, E, b)]
    h = torch.nn.functional.rms_norm(xs[0], (K,), xs[1], eps)
    O2, lse2 = swvr.softmax_readout(h, xs[2], xs[3], xs[4])
    grads2 = torch.autograd.grad((O2 * gO).sum() + (lse2 * glse).sum(), xs)
    assert rel_err(O, O2) < 2e-2 and float((lse - lse2).abs().max()) < 1e-2
    for name, a, r in zip(["gx", "gw", "gW", "gE", "gb"], grads, grads2):
        assert rel_err(a, r) < 2e-2, (name, rel_err(a, r))


@pytest.mark.parametrize("K,lead", [(100, (3, 7)), (64, (0,))])
def test_fused_norm_leading_dims_odd_hidden_and_empty_batch(K, lead):
    """h [..., K] with leading dims, a hidden size that is not a multiple of 8 (the readout
    pads its operand copy), and an empty batch (zero gradients for W, E, b, the weight)."""
    V, D, eps = 777, 16, 1e-6
    x, w, W, E, b = _inputs(None, K, V, D, torch.bfloat16, seed=3, lead=lead)
    g = torch.Generator().manual_seed(7)
    gO = torch.randn(*lead, D, generator=g).cuda()
    glse = torch.randn(*lead, generator=g).cuda()
    O, lse, grads = _run(x, w, W, E, b, eps, 1.0, gO, glse)
    assert O.shape == (*lead, D) and lse.shape == lead
    if lead == (0,):
        for a in grads[1:]:
            assert torch.count_nonzero(a) == 0
        return
    Or, lr, gr = _oracle(x, w, W, E, b, eps, 1.0, gO, glse)
    assert rel_err(O.reshape(-1, D), Or) < 2e-2
    for name, a, r in zip(["gx", "gw", "gW", "gE", "gb"], grads, gr):
        assert rel_err(a, r) < 2e-2, (name, rel_err(a, r))


def test_fused_norm_under_autocast_with_fp32_params():
    N, K, V, D, eps = 256, 256, 4000, 16, 1e-6
    x, w, W, E, b = _inputs(N, K, V, D, torch.float32, seed=4)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        O, lse = swvr.rmsnorm_softmax_readout(x, w, W, E, b, eps=eps)
    assert O.dtype == torch.float32
    (O.sum() + lse.sum()).backward()
    assert x.grad.dtype == torch.float32 and w.grad.dtype == torch.float32 and W.grad.dtype == torch.float32
    Or, _, gr = _oracle(x, w, W, E, b, eps, 1.0, torch.ones_like(O), torch.ones_like(lse))
    assert rel_err(O, Or) < 2e-2
    for name, a, r in zip(["gx", "gw", "gW", "gE", "gb"], [x.grad, w.grad, W.grad, E.grad, b.grad], gr):
        assert rel_err(a, r) < 2e-2, (name, rel_err(a, r))


def test_module_with_norm_equals_the_unfused_module():
    """SoftmaxReadoutMSE(head, embedding, norm=nn.RMSNorm) on the trunk output against the
    reference-style module on rms_norm of it: loss and every gradient (x, norm weight, head
    weight and bias, embedding)."""
    torch.manual_seed(0)
    N, K, V, D = 512, 256, 5003, 32
    head = torch.nn.Linear(K, V).cuda().to(torch.bfloat16)
    emb = torch.nn.Embedding(V, D).cuda().to(torch.bfloat16)
    norm = torch.nn.RMSNorm(K, eps=1e-5).cuda().to(torch.bfloat16)
    with torch.no_grad():
        norm.weight.uniform_(0.5, 1.5)
    x = (2 * torch.randn(N, K, device="cuda")).to(torch.bfloat16).requires_grad_(True)
    t = 0.02 * torch.randn(N, D, device="cuda")
    fused = swvr.SoftmaxReadoutMSE(head, emb, norm=norm, z_loss_weight=1e-4)
    plain = swvr.SoftmaxReadoutMSE(head, emb, z_loss_weight=1e-4)
    params = [x, norm.weight, head.weight, head.bias, emb.weight]
    l1 = fused(x, t)
    g1 = torch.autograd.grad(l1, params)
    l2 = plain(norm(x), t)
    g2 = torch.autograd.grad(l2, params)
    assert abs(l1.item() - l2.item()) <= 2e-2 * abs(l2.item())
    for name, a, r in zip(["x", "norm", "W", "b", "E"], g1, g2):
        assert rel_err(a, r) < 2e-2, (name, rel_err(a, r))


def test_fused_norm_compiles_checkpoints_and_repeats_bit_exactly():
    N, K, V, D, eps = 384, 256, 3001, 32, 1e-6
    x, w, W, E, b = _inputs(N, K, V, D, torch.bfloat16, seed=8)
    g = torch.Generator().manual_seed(9)
    gO, glse = torch.randn(N, D, generator=g).cuda(), torch.randn(N, generator=g).cuda()

    def f(x_, w_, W_, E_, b_):
        O, lse = swvr.rmsnorm_softmax_readout(x_, w_, W_, E_, b_, eps=eps)
        return (O * gO).sum() + (lse * glse).sum()

    leaves = [x, w, W, E, b]
    ref = torch.autograd.grad(f(*leaves), leaves)
    again = torch.autograd.grad(f(*leaves), leaves)
    for a, r in zip(again, ref):
        assert torch.equal(a, r)
    ckpt = torch.autograd.grad(torch.utils.checkpoint.checkpoint(f, *leaves, use_reentrant=False), leaves)
    for a, r in zip(ckpt, ref):
        assert torch.equal(a, r)
    compiled = torch.compile(f, fullgraph=True)
    comp = torch.autograd.grad(compiled(*leaves), leaves)
    for a, r in zip(comp, ref):
        assert torch.equal(a, r)
