"""CUDA-graph capture of a whole fwd+bwd step through the public API.

The C ABI allocates nothing and never synchronises; all work goes on the caller's current
stream, so a training step that calls softmax_readout_mse can be captured once and
replayed.  Replay removes the host-side launch cost of the chunk loop, which dominates the
small shapes (the reference's chunk loop, swvr/chunked.py:96-105 and 120-151, launches per
chunk from Python).
"""
import pytest
import torch

import swvr_b200 as swvr
from tests.helpers import rel_err

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("N,K,V,D,chunk", [(256, 64, 1000, 16, 8192), (1000, 256, 9000, 64, 1024),
                                           (512, 512, 20000, 128, 4096)])
def test_captured_step_matches_eager(N, K, V, D, chunk):
    g = torch.Generator(device="cuda").manual_seed(7)
    W = (K ** -0.5 * torch.randn(V, K, generator=g, device="cuda")).to(torch.bfloat16).requires_grad_(True)
    E = (0.02 * torch.randn(V, D, generator=g, device="cuda")).to(torch.bfloat16).requires_grad_(True)
    b = (0.02 * torch.randn(V, generator=g, device="cuda")).to(torch.bfloat16).requires_grad_(True)
    h_static = torch.randn(N, K, generator=g, device="cuda").to(torch.bfloat16)
    t_static = 0.02 * torch.randn(N, D, generator=g, device="cuda")
    w_static = (torch.rand(N, generator=g, device="cuda") < 0.9).float()

    def step():
        hh = h_static.detach().requires_grad_(True)
        loss = swvr.softmax_readout_mse(hh, W, E, t_static, b, weight=w_static, z_loss_weight=1e-4,
                                        chunk_size=chunk)
        loss.backward()
        return loss, hh

    # warm up on a side stream (as torch.cuda.graphs requires), then capture
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            for p in (W, E, b):
                p.grad = None
            step()
    torch.cuda.current_stream().wait_stream(s)
    for p in (W, E, b):
        p.grad = None
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        loss_g, h_g = step()
    grads_g = [h_g.grad, W.grad, E.grad, b.grad]  # the graph's static gradient buffers

    # new inputs into the static buffers, replay, and compare with an eager step
    for seed in (11, 12):
        gg = torch.Generator(device="cuda").manual_seed(seed)
        h_static.copy_(torch.randn(N, K, generator=gg, device="cuda").to(torch.bfloat16))
        t_static.copy_(0.02 * torch.randn(N, D, generator=gg, device="cuda"))
        graph.replay()
        torch.cuda.synchronize()
        got = [loss_g.detach().clone()] + [x.clone() for x in grads_g]
        for p in (W, E, b):
            p.grad = None
        loss_e, h_e = step()
        torch.cuda.synchronize()
        want = [loss_e.detach(), h_e.grad, W.grad, E.grad, b.grad]
        for a, r in zip(got, want):
            assert rel_err(a, r) == 0.0, rel_err(a, r)  # same kernels, same order: bit-identical
        for p in (W, E, b):
            p.grad = None
    del graph


def test_captured_step_matches_oracle():
    """A captured fwd+bwd step replayed on new inputs against the fp64 numpy oracle (loss and
    every gradient, bf16 tolerance), not only against eager."""

    from oracle import swvr_oracle as orc
    from tests.helpers import npy

    N, K, V, D = 300, 128, 3001, 16
    g = torch.Generator(device="cuda").manual_seed(9)
    W = (K ** -0.5 * torch.randn(V, K, generator=g, device="cuda")).to(torch.bfloat16).requires_grad_(True)
    E = (0.5 * torch.randn(V, D, generator=g, device="cuda")).to(torch.bfloat16).requires_grad_(True)
    b = (0.5 * torch.randn(V, generator=g, device="cuda")).to(torch.bfloat16).requires_grad_(True)
    h_static = torch.zeros(N, K, device="cuda", dtype=torch.bfloat16)
    t_static = torch.zeros(N, D, device="cuda")

    def step():
        hh = h_static.detach().requires_grad_(True)
        loss = swvr.softmax_readout_mse(hh, W, E, t_static, b, z_loss_weight=1e-3, chunk_size=1024)
        loss.backward()
        return loss, hh

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            for p in (W, E, b):
                p.grad = None
            step()
    torch.cuda.current_stream().wait_stream(s)
    for p in (W, E, b):
        p.grad = None
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        loss_g, h_g = step()
    gg = torch.Generator(device="cuda").manual_seed(10)
    h_static.copy_(torch.randn(N, K, generator=gg, device="cuda").to(torch.bfloat16))
    t_static.copy_(0.1 * torch.randn(N, D, generator=gg, device="cuda"))
    graph.replay()
    torch.cuda.synchronize()
    args = [npy(h_static), npy(W), npy(E), npy(b)]
    O, lse = orc.softmax_readout_reference(*args)
    t = npy(t_static)
    loss_ref = orc.mse_forward(O, lse, t, None, "mean", 1e-3)
    gO, glse, _, _ = orc.mse_backward(O, lse, t, None, "mean", 1e-3)
    ref = orc.readout_grads(*args, gO, glse)
    assert abs(loss_g.item() - loss_ref) <= 2e-2 * abs(loss_ref)
    for name, got, want in zip("hWEb", (h_g.grad, W.grad, E.grad, b.grad), ref):
        assert rel_err(got, want) < 2e-2, (name, rel_err(got, want))
    del graph
