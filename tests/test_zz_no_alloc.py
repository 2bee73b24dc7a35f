"""swvr_fwd_noalloc: the forward for callers that cannot allocate device memory.

Hosts that plan all device memory up front, or FFI hosts that forbid their plugins
cudaMalloc, call this entry point with only the problem, the outputs and a stream; its
scratch is a static device array inside the library.  This file runs last (pytest collects
it last by name) so that a failure here leaves every other test already run.  It checks the
entry point through the C ABI against swvr_fwd on two calls in a row, and that a problem
too large for the static scratch is rejected with a message.
"""
import ctypes

import numpy as np
import pytest
import torch

from tests.helpers import make_gpu, rel_err

pytestmark = pytest.mark.gpu


def _fwd_with_workspace(nat, p, N, D, dev):
    O = torch.empty(N, D, dtype=torch.float32, device=dev)
    lse = torch.empty(N, dtype=torch.float32, device=dev)
    nbytes = ctypes.c_size_t(0)
    nat.check(nat.lib().swvr_fwd_workspace_size(p, ctypes.byref(nbytes)), "swvr_fwd_workspace_size")
    ws = torch.empty(max(nbytes.value, 1), dtype=torch.uint8, device=dev)
    nat.check(nat.lib().swvr_fwd(p, O.data_ptr(), lse.data_ptr(), ws.data_ptr(), ws.numel(), nat.stream_ptr(dev)),
              "swvr_fwd")
    return O, lse


def test_fwd_noalloc_matches_fwd_on_two_calls():
    from swvr_b200 import _native as nat
    from swvr_b200.ops import _prepare, _problem

    N, K, V, D = 1000, 512, 20011, 64
    h, W, E, b = make_gpu(N, K, V, D, torch.bfloat16)
    dev = h.device
    hc, Wc, Ec, bc = _prepare(h.detach(), W.detach(), E.detach(), b.detach(), torch.bfloat16)
    p = _problem(hc, Wc, Ec, bc, 0.8, 8192, torch.bfloat16)
    O_ref, lse_ref = _fwd_with_workspace(nat, p, N, D, dev)
    for call in range(2):
        O = torch.full((N, D), float("nan"), dtype=torch.float32, device=dev)
        lse = torch.full((N,), float("nan"), dtype=torch.float32, device=dev)
        nat.check(nat.lib().swvr_fwd_noalloc(p, O.data_ptr(), lse.data_ptr(), nat.stream_ptr(dev)),
                  "swvr_fwd_noalloc")
        torch.cuda.synchronize()
        nat.check_device_error()
        assert torch.isfinite(O).all() and torch.isfinite(lse).all(), call
        assert rel_err(O, O_ref) < 2e-2, (call, rel_err(O, O_ref))
        assert float((lse - lse_ref).abs().max()) < 1e-2, call


def test_fwd_noalloc_rejects_problems_beyond_its_scratch():
    from swvr_b200 import _native as nat

    p = nat.Problem()
    p.n_tokens, p.hidden, p.vocab, p.embed_dim = 1 << 20, 64, 1000, 128   # ~0.5 GB of state
    p.compute_dtype, p.bias_dtype = nat.BF16, nat.F32
    buf = torch.empty(1 << 16, dtype=torch.bfloat16, device="cuda")
    p.h = p.W = p.E = buf.data_ptr()
    p.ldh = p.ldw = 64
    p.lde = 128
    p.logit_scale, p.chunk = 1.0, 8192
    rc = nat.lib().swvr_fwd_noalloc(p, buf.data_ptr(), buf.data_ptr(), nat.stream_ptr(buf.device))
    assert rc == nat.ERR_UNSUPPORTED
    assert "static scratch" in nat.last_error()
