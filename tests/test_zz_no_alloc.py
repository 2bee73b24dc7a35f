"""swvr_fwd_noalloc: the forward for callers that cannot allocate device memory.

Hosts that plan all device memory up front, or FFI hosts that forbid their plugins
cudaMalloc, call this entry point with only the problem, the outputs and a stream; its
scratch is a static device array inside the library.  This file runs last (pytest collects
it last by name) so that a failure here leaves every other test already run.  It checks the
entry point through the C ABI, on two calls in a row, against swvr_fwd and against the
numpy oracle; at sizes where the planner must lower the vocabulary splits to fit the array
and where a single split nearly fills it; that the calls leave the device's free memory
unchanged; and that a problem too large for the static scratch is rejected with a message.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import swvr_oracle as orc
from tests.helpers import make_gpu, npy, rel_err

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


def _problem(N, K, V, D, scale, seed=0):
    from swvr_b200.ops import _prepare, _problem as make_problem

    h, W, E, b = make_gpu(N, K, V, D, torch.bfloat16, seed=seed)
    ops_in = _prepare(h.detach(), W.detach(), E.detach(), b.detach(), torch.bfloat16)
    return make_problem(*ops_in, scale, 8192, torch.bfloat16), ops_in, (h, W, E, b)


def _noalloc_twice(nat, p, N, D, dev):
    """Two calls in a row into fresh NaN-filled outputs (nothing of a call may leak into the next)."""
    outs = []
    for _ in range(2):
        O = torch.full((N, D), float("nan"), dtype=torch.float32, device=dev)
        lse = torch.full((N,), float("nan"), dtype=torch.float32, device=dev)
        nat.check(nat.lib().swvr_fwd_noalloc(p, O.data_ptr(), lse.data_ptr(), nat.stream_ptr(dev)), "swvr_fwd_noalloc")
        torch.cuda.synchronize()
        nat.check_device_error()
        outs.append((O, lse))
    return outs


def test_fwd_noalloc_matches_fwd_and_oracle_on_two_calls():
    from swvr_b200 import _native as nat

    N, K, V, D, scale = 1000, 512, 20011, 64, 0.8
    p, _keep, (h, W, E, b) = _problem(N, K, V, D, scale)
    dev = h.device
    O_ref, lse_ref = _fwd_with_workspace(nat, p, N, D, dev)
    O_orc, lse_orc = orc.chunked_forward(npy(h), npy(W), npy(E), npy(b), scale, 8192, "bf16")
    for call, (O, lse) in enumerate(_noalloc_twice(nat, p, N, D, dev)):
        assert torch.isfinite(O).all() and torch.isfinite(lse).all(), call
        assert rel_err(O, O_ref) < 2e-2, (call, rel_err(O, O_ref))
        assert float((lse - lse_ref).abs().max()) < 1e-2, call
        assert rel_err(O, O_orc) < 2e-2, (call, rel_err(O, O_orc))
        assert float(np.abs(npy(lse) - lse_orc).max()) < 1e-2, call


@pytest.mark.parametrize("N,K,V,D", [
    (4096, 256, 30011, 256),   # 16 token tiles at D = 256: 59 vocabulary splits lowered to 3
    (16000, 256, 20011, 256),  # 63 tiles at D = 256: lowered to one split, the array nearly full
    (16384, 256, 30011, 64),   # 64 tiles at D = 64: 53 splits lowered to 1
])
def test_fwd_noalloc_at_the_limits_of_its_scratch(N, K, V, D):
    from swvr_b200 import _native as nat

    p, _keep, (h, _, _, _) = _problem(N, K, V, D, 1.0, seed=3)
    dev = h.device
    O_ref, lse_ref = _fwd_with_workspace(nat, p, N, D, dev)
    for call, (O, lse) in enumerate(_noalloc_twice(nat, p, N, D, dev)):
        assert torch.isfinite(O).all() and torch.isfinite(lse).all(), call
        assert rel_err(O, O_ref) < 2e-2, (call, rel_err(O, O_ref))
        assert float((lse - lse_ref).abs().max()) < 1e-2, call


def test_fwd_noalloc_leaves_free_device_memory_unchanged():
    from swvr_b200 import _native as nat

    N, K, V, D = 1000, 512, 20011, 64
    p, _keep, (h, _, _, _) = _problem(N, K, V, D, 1.0, seed=5)
    dev = h.device
    O = torch.empty(N, D, dtype=torch.float32, device=dev)
    lse = torch.empty(N, dtype=torch.float32, device=dev)
    call = lambda: nat.check(nat.lib().swvr_fwd_noalloc(p, O.data_ptr(), lse.data_ptr(), nat.stream_ptr(dev)),
                             "swvr_fwd_noalloc")
    call()  # loads the kernels' code on first launch
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info(dev)
    for _ in range(2):
        call()
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info(dev)
    nat.check_device_error()
    assert free1 == free0, (free0, free1)


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
