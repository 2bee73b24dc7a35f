"""Parity at BASELINE's full sizes, on exactly the workloads bench.py measures.

c1 (N=16384 as h [8, 2048, 1024], V=152064, D=16, no bias), c2 (the headline: N=16384,
K=2560, V=152064, D=64, bias, Bernoulli(0.9) per-token weight, z-loss 1e-4), c3 (N=8192,
K=4096, V=128256, D=128, the raw ``softmax_readout`` with a torch MSE on top against
``E[randint] + N(0, 0.01)``) and c4 (N=131072 as h [32, 4096, 4096], V=152064, D=64, bias,
under ``torch.utils.checkpoint``, on one GPU), built by bench.py's own ``make_inputs`` /
``make_step``.

Two checkers, each within the north star's bf16 tolerance (2e-2 norm-wise relative, the
reference's test_cuda.py:33-35,54; LSE 1e-2 absolute):

* the reference library itself, unmodified, from its offline install under baseline/_ref
  (its public API: cuBLAS GEMMs plus its Triton kernels, swvr/chunked.py:82-151) on the same
  GPU inputs: loss, O, LSE and every gradient (h, W, E, bias, and target / weight where they
  take one) over the whole tensors.  Skipped where the install is absent.
* for c2, an independent restatement of the math in torch with fp32 scores
  (swvr/reference.py:5-14 evaluated in vocabulary chunks): the full LSE and O vectors, dh on
  512 token rows and dW / dE / db on 512 vocabulary rows (first, last and random rows), with
  the backward's delta built from the restatement's own O.
"""
import pytest
import torch

import swvr_b200 as swvr
from bench import CONFIGS, load_reference, make_inputs, make_step

pytestmark = pytest.mark.gpu


def rel(a, r):
    """Norm-wise relative error on the GPU (the tensors are too large to move to the host)."""
    a, r = a.detach().float(), r.detach().float()
    return ((a - r).norm() / r.norm().clamp_min(1e-30)).item()


def _leaves(c, target_grad):
    h, W, E, b, t, w, _ = make_inputs(c, torch.device("cuda", 0), 0, 1)
    if target_grad:
        t = t.clone().requires_grad_(True)
        w = w.clone().requires_grad_(True) if w is not None else None
    return h, W, E, b, t, w


def _run(api, c, leaves):
    h, W, E, b, t, w = leaves
    for x in leaves:
        if x is not None:
            x.grad = None
    loss = make_step(c, api, W, E, b, None)(h, t, w)
    grads = {k: x.grad.detach().clone() for k, x in zip(("h", "W", "E", "b", "t", "w"), leaves)
             if x is not None and x.grad is not None}
    with torch.no_grad():
        O, lse = api.softmax_readout(h, W, E, b)
    return loss.detach(), O, lse, grads


@pytest.mark.parametrize("config", ["c1", "c2", "c3", "c4"])
def test_full_size_matches_the_reference_library(config):
    ref = load_reference()
    if ref is None:
        pytest.skip("the reference library is not installed under baseline/_ref")
    c = CONFIGS[config]
    leaves = _leaves(c, target_grad=True)
    loss, O, lse, grads = _run(swvr, c, leaves)
    loss_r, O_r, lse_r, grads_r = _run(ref, c, leaves)
    torch.cuda.synchronize()
    assert torch.isfinite(loss) and abs(loss.item() - loss_r.item()) <= 2e-2 * abs(loss_r.item()), \
        (loss.item(), loss_r.item())
    assert O.shape == O_r.shape and lse.shape == lse_r.shape
    assert (lse - lse_r).abs().max().item() < 1e-2
    assert rel(O, O_r) < 2e-2, rel(O, O_r)
    assert set(grads) == set(grads_r), (sorted(grads), sorted(grads_r))
    for k in grads:
        assert torch.isfinite(grads[k]).all(), k
        assert rel(grads[k], grads_r[k]) < 2e-2, (k, rel(grads[k], grads_r[k]))


# ------------------------------------------------------------------ independent fp32 restatement (c2)

def _pick(n, k, seed):
    g = torch.Generator().manual_seed(seed)
    edge = torch.tensor([0, 1, 127, 128, 255, 256, n - 257, n - 256, n - 129, n - 128, n - 2, n - 1])
    rest = torch.randperm(n, generator=g)[:k - edge.numel()]
    return torch.unique(torch.cat([edge, rest])).cuda()


def _scores(h, W, b, rows=None, cols=None):
    hh = h if rows is None else h[rows]
    WW = W if cols is None else W[cols]
    bb = b if cols is None else b[cols]
    return torch.mm(hh, WW.t(), out_dtype=torch.float32) + bb.float()


@torch.no_grad()
def _restated_forward(h, W, E, b, step=8192):
    """O and LSE in fp32 from fp32 scores, the vocabulary in chunks (two passes)."""
    N, V = h.shape[0], W.shape[0]
    lse = torch.full((N,), -float("inf"), device="cuda")
    for v0 in range(0, V, step):
        lse = torch.logaddexp(lse, torch.logsumexp(_scores(h, W[v0:v0 + step], b[v0:v0 + step]), dim=1))
    O = torch.zeros(N, E.shape[1], device="cuda")
    for v0 in range(0, V, step):
        P = torch.exp(_scores(h, W[v0:v0 + step], b[v0:v0 + step]) - lse[:, None])
        O += P @ E[v0:v0 + step].float()
    return O, lse


def test_headline_matches_an_fp32_restatement():
    c = CONFIGS["c2"]
    h, W, E, b, t, w = _leaves(c, target_grad=False)
    loss, O, lse, grads = _run(swvr, c, (h, W, E, b, t, w))
    torch.cuda.synchronize()
    with torch.no_grad():
        hd, Wd, Ed, bd = h.detach(), W.detach(), E.detach(), b.detach()
        O_ref, lse_ref = _restated_forward(hd, Wd, Ed, bd)
        assert (lse - lse_ref).abs().max().item() < 1e-2
        assert rel(O, O_ref) < 2e-2
        # the loss of swvr/api.py:54-66 on the restated O, LSE
        per_tok = ((O_ref - t) ** 2).mean(1) + c["z"] * lse_ref ** 2
        loss_ref = (per_tok * w).sum() / w.sum()
        assert abs(loss.item() - loss_ref.item()) <= 2e-2 * abs(loss_ref.item())
        # upstream gradients of that loss: dL/dO and dL/dLSE
        gO = (2.0 / c["D"]) * (O_ref - t) * (w / w.sum())[:, None]
        glse = 2.0 * c["z"] * lse_ref * (w / w.sum())
        delta = (O_ref * gO).sum(1) - glse

        tr = _pick(c["N"], 512, 1)  # token rows: dh needs every vocabulary row of those tokens
        P = torch.exp(_scores(hd, Wd, bd, rows=tr) - lse_ref[tr, None])
        dS = P * (gO[tr] @ Ed.float().t() - delta[tr, None])
        assert rel(grads["h"][tr], dS @ Wd.float()) < 2e-2
        del P, dS

        vr = _pick(c["V"], 512, 2)  # vocabulary rows: dW, dE, db need every token of those rows
        P = torch.exp(_scores(hd, Wd, bd, cols=vr) - lse_ref[:, None])
        dS = P * (gO @ Ed[vr].float().t() - delta[:, None])
        assert rel(grads["W"][vr], dS.t() @ hd.float()) < 2e-2
        assert rel(grads["E"][vr], P.t() @ gO) < 2e-2
        assert rel(grads["b"][vr], dS.sum(0)) < 2e-2
        for k in ("h", "W", "E", "b"):
            assert torch.isfinite(grads[k]).all(), k
