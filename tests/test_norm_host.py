"""CPU tests of the fused RMSNorm producer of h: the oracle it is checked against, its
argument validation (before any device work), the C ABI's host-side checks and the custom
ops' fake impls."""
import ctypes

import numpy as np
import pytest
import torch

import swvr_b200 as swvr
from oracle import swvr_oracle as orc
from swvr_b200 import _native as nat


@pytest.mark.parametrize("affine", [True, False])
def test_oracle_rmsnorm_matches_torch_rms_norm(affine):
    """The oracle's norm and its gradient against torch.nn.functional.rms_norm (fp64 autograd)."""
    g = torch.Generator().manual_seed(0)
    x = torch.randn(3, 5, 24, generator=g, dtype=torch.float64, requires_grad=True)
    w = torch.randn(24, generator=g, dtype=torch.float64, requires_grad=True) if affine else None
    dh = torch.randn(3, 5, 24, generator=g, dtype=torch.float64)
    eps = 1e-3
    y = torch.nn.functional.rms_norm(x, (24,), w, eps)
    grads = torch.autograd.grad(y, [x] + ([w] if affine else []), dh)
    h, rstd = orc.rmsnorm_forward(x.detach().numpy(), None if w is None else w.detach().numpy(), eps)
    np.testing.assert_allclose(h, y.detach().numpy(), rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(rstd, 1 / np.sqrt((x.detach().numpy() ** 2).mean(-1) + eps), rtol=1e-13)
    dx, dw = orc.rmsnorm_backward(dh.numpy(), x.detach().numpy(), None if w is None else w.detach().numpy(), eps)
    np.testing.assert_allclose(dx, grads[0].numpy(), rtol=1e-10, atol=1e-12)
    if affine:
        np.testing.assert_allclose(dw, grads[1].numpy(), rtol=1e-10, atol=1e-12)
    else:
        assert dw is None


def test_oracle_rmsnorm_backward_matches_finite_differences():
    rng = np.random.default_rng(1)
    x, w, dh, eps = rng.standard_normal((4, 9)), rng.standard_normal(9), rng.standard_normal((4, 9)), 1e-2
    dx, dw = orc.rmsnorm_backward(dh, x, w, eps)
    f = lambda x_, w_: (orc.rmsnorm_forward(x_, w_, eps)[0] * dh).sum()
    e = 1e-6
    num_x = np.array([[(f(x + e * np.eye(36)[i * 9 + j].reshape(4, 9), w) - f(x - e * np.eye(36)[i * 9 + j].reshape(4, 9), w))
                       / (2 * e) for j in range(9)] for i in range(4)])
    num_w = np.array([(f(x, w + e * np.eye(9)[j]) - f(x, w - e * np.eye(9)[j])) / (2 * e) for j in range(9)])
    np.testing.assert_allclose(dx, num_x, atol=1e-7)
    np.testing.assert_allclose(dw, num_w, atol=1e-7)


def test_fused_norm_validates_before_any_device_work():
    x, W, E, b = torch.randn(6, 12), torch.randn(41, 12), torch.randn(41, 5), torch.randn(41)
    g = torch.randn(12)
    with pytest.raises(ValueError, match="norm_weight"):
        swvr.rmsnorm_softmax_readout(x, g[:-1], W, E)
    with pytest.raises(ValueError, match="eps"):
        swvr.rmsnorm_softmax_readout(x, g, W, E, eps=-1.0)
    with pytest.raises(ValueError):
        swvr.rmsnorm_softmax_readout(x, g, W[:, :-1], E)
    with pytest.raises(ValueError):
        swvr.rmsnorm_softmax_readout(x, g, W, E, b[:-1])
    with pytest.raises(ValueError):
        swvr.rmsnorm_softmax_readout_mse(x, g, W, E, torch.randn(6, 5), reduction="max")
    with pytest.raises(RuntimeError, match="CUDA devices only"):  # no CPU fallback
        swvr.rmsnorm_softmax_readout(x, g, W, E)
    with pytest.raises(ValueError, match="RMSNorm"):
        swvr.SoftmaxReadoutMSE(torch.nn.Linear(12, 41), torch.nn.Embedding(41, 5), norm=torch.nn.LayerNorm(12))
    with pytest.raises(ValueError, match="last dimension"):
        swvr.SoftmaxReadoutMSE(torch.nn.Linear(12, 41), torch.nn.Embedding(41, 5), norm=torch.nn.RMSNorm((3, 12)))
    norm = torch.nn.RMSNorm(12)
    m = swvr.SoftmaxReadoutMSE(torch.nn.Linear(12, 41), torch.nn.Embedding(41, 5), norm=norm)
    assert m.norm is norm


def test_norm_abi_rejects_bad_arguments_on_the_host():
    lib = nat.lib()
    buf = 1 << 20
    assert lib.swvr_rmsnorm_fwd(-1, 8, buf, nat.BF16, 8, None, 0, 1e-6, buf, nat.BF16, 8, buf, None) == \
        nat.ERR_INVALID_ARGUMENT
    assert lib.swvr_rmsnorm_fwd(4, 8, buf, 9, 8, None, 0, 1e-6, buf, nat.BF16, 8, buf, None) == nat.ERR_INVALID_ARGUMENT
    assert lib.swvr_rmsnorm_fwd(4, 8, buf, nat.BF16, 4, None, 0, 1e-6, buf, nat.BF16, 8, buf, None) == \
        nat.ERR_INVALID_ARGUMENT  # row pitch below hidden
    assert lib.swvr_rmsnorm_fwd(4, 8, None, nat.BF16, 8, None, 0, 1e-6, buf, nat.BF16, 8, buf, None) == \
        nat.ERR_INVALID_ARGUMENT
    assert lib.swvr_rmsnorm_fwd(4, 8, buf, nat.BF16, 8, None, 0, -1.0, buf, nat.BF16, 8, buf, None) == \
        nat.ERR_INVALID_ARGUMENT
    n = ctypes.c_size_t(0)
    assert lib.swvr_rmsnorm_bwd_workspace_size(16384, 2560, nat.F32, 1, ctypes.byref(n)) == nat.OK
    assert 0 < n.value <= 296 * 2560 * 4
    assert lib.swvr_rmsnorm_bwd_workspace_size(16384, 2560, nat.F32, 0, ctypes.byref(n)) == nat.OK and n.value == 0
    assert lib.swvr_rmsnorm_bwd_workspace_size(16, 8, nat.BF16, 1, ctypes.byref(n)) == nat.ERR_INVALID_ARGUMENT
    args = lambda ws_bytes, K=8, gw=buf, w=buf: (16, K, buf, nat.F32, buf, nat.BF16, K, w, nat.F32, buf, buf, nat.BF16,
                                                 gw, nat.F32, buf, ws_bytes, None)
    assert lib.swvr_rmsnorm_bwd(*args(0)) == nat.ERR_WORKSPACE
    assert lib.swvr_rmsnorm_bwd(*args(1 << 30, w=None)) == nat.ERR_INVALID_ARGUMENT  # grad_weight without weight
    assert lib.swvr_rmsnorm_bwd(*args(1 << 30, K=100000)) == nat.ERR_UNSUPPORTED
    assert "too wide" in nat.last_error()


@pytest.mark.parametrize("dtype,adt", [(torch.bfloat16, torch.float32), (torch.float64, torch.float64)])
def test_norm_fake_impls_give_shapes(dtype, adt):
    x = torch.empty(6, 16, dtype=dtype, device="meta")
    g = torch.empty(16, dtype=torch.float32, device="meta")
    W = torch.empty(100, 16, dtype=dtype, device="meta")
    E = torch.empty(100, 5, dtype=dtype, device="meta")
    O, lse, h, rstd = torch.ops.swvr_b200.norm_fwd(x, g, W, E, None, 1e-6, 1.0, 8192, dtype)
    assert O.shape == (6, 5) and lse.shape == (6,) and O.dtype == adt
    assert h.shape == (6, 16) and h.dtype == dtype and rstd.shape == (6,) and rstd.dtype == adt
    grads = torch.ops.swvr_b200.norm_bwd(O, lse, x, g, W, E, None, O, lse, h, rstd, 1.0, 8192, dtype,
                                         True, True, False, True, True)
    assert [tuple(t.shape) for t in grads] == [(6, 16), (16,), (0,), (100, 5), (0,)]
