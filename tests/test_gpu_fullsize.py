"""Parity at the headline size (c2: N=16384, K=2560, V=152064, D=64, bf16, bias).

The numpy oracle cannot finish this size in a test, so the reference here is the same
algorithm in torch on the GPU with fp32 scores (swvr/reference.py:5-14 evaluated in vocab
chunks, as swvr/chunked.py:82-151 does): the full LSE vector, O and dh on a subset of token
rows, and dW, dE, db on a subset of vocabulary rows, each against that reference with the
bf16 tolerance of the reference's GPU suite (2e-2 norm-wise, test_cuda.py:54; LSE 1e-2
absolute).  The subsets span the first, last and random rows, so tile and chunk tails are
included.
"""
import pytest
import torch

import swvr_b200 as swvr
from tests.helpers import rel_err

pytestmark = pytest.mark.gpu

N, K, V, D = 16384, 2560, 152064, 64
SCALE = 1.0


def _inputs():
    g = torch.Generator(device="cuda").manual_seed(2024)
    h = torch.randn(N, K, generator=g, device="cuda").to(torch.bfloat16)
    W = (K ** -0.5 * torch.randn(V, K, generator=g, device="cuda")).to(torch.bfloat16)
    E = (0.02 * torch.randn(V, D, generator=g, device="cuda")).to(torch.bfloat16)
    b = (0.02 * torch.randn(V, generator=g, device="cuda")).to(torch.bfloat16)
    gO = 0.02 * torch.randn(N, D, generator=g, device="cuda")
    glse = 0.01 * torch.randn(N, generator=g, device="cuda")
    return h, W, E, b, gO, glse


def _rows(n, k, seed):
    g = torch.Generator().manual_seed(seed)
    edge = torch.tensor([0, 1, 127, 128, 255, 256, n - 257, n - 256, n - 129, n - 128, n - 2, n - 1])
    rest = torch.randperm(n, generator=g)[:k - edge.numel()]
    return torch.unique(torch.cat([edge, rest])).cuda()


def _scores(h, W, b, rows=None, cols=None):
    hh = h if rows is None else h[rows]
    WW = W if cols is None else W[cols]
    bb = b if cols is None else b[cols]
    return torch.mm(hh, WW.t(), out_dtype=torch.float32) * SCALE + bb.float()


@torch.no_grad()
def _reference_lse(h, W, b, step=8192):
    lse = torch.full((N,), -float("inf"), device="cuda")
    for v0 in range(0, V, step):
        s = torch.mm(h, W[v0:v0 + step].t(), out_dtype=torch.float32) * SCALE + b[v0:v0 + step].float()
        lse = torch.logaddexp(lse, torch.logsumexp(s, dim=1))
        del s
    return lse


def test_headline_size_matches_fp32_reference():
    h, W, E, b, gO, glse = _inputs()
    hq, Wq, Eq, bq = (x.detach().clone().requires_grad_(True) for x in (h, W, E, b))
    O, lse = swvr.softmax_readout(hq, Wq, Eq, bq, logit_scale=SCALE)
    torch.autograd.backward([O, lse], [gO, glse])
    torch.cuda.synchronize()

    with torch.no_grad():
        ref_lse = _reference_lse(h, W, b)
        assert (lse - ref_lse).abs().max().item() < 1e-2

        # token rows: O and dh need every vocabulary row of those tokens
        tr = _rows(N, 512, 1)
        P = torch.exp(_scores(h, W, b, rows=tr) - ref_lse[tr, None])           # [t, V]
        O_ref = P @ E.float()
        assert rel_err(O[tr], O_ref) < 2e-2
        delta = (O_ref * gO[tr]).sum(1) - glse[tr]
        dS = P * (gO[tr] @ E.float().t() - delta[:, None])
        dh_ref = SCALE * (dS @ W.float())
        assert rel_err(hq.grad[tr], dh_ref) < 2e-2
        del P, dS

        # vocabulary rows: dW, dE, db need every token of those rows
        vr = _rows(V, 512, 2)
        P = torch.exp(_scores(h, W, b, cols=vr) - ref_lse[:, None])            # [N, v]
        O_full = O.float()
        delta = (O_full * gO).sum(1) - glse
        dS = P * (gO @ E[vr].float().t() - delta[:, None])
        assert rel_err(Wq.grad[vr], SCALE * (dS.t() @ h.float())) < 2e-2
        assert rel_err(Eq.grad[vr], P.t() @ gO) < 2e-2
        assert rel_err(bq.grad[vr], dS.sum(0)) < 2e-2
        # every gradient is finite at full size
        for x in (hq, Wq, Eq, bq):
            assert torch.isfinite(x.grad).all()
