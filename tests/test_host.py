"""CPU tests of the host side: the C ABI loads and exports every declared symbol, argument
validation and planning entry points behave, the Python API validates like the reference's
and refuses CPU tensors (no fallback), and the custom ops' fake impls give the shapes."""
import ctypes

import pytest
import torch

import swvr_b200 as swvr
from swvr_b200 import _native as nat
from swvr_b200.ops import acc_dtype, default_chunk_size


def test_library_exports_every_declared_symbol():
    lib = nat.lib()
    names = nat.header_functions()
    assert len(names) >= 11
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) == set(nat._SIGNATURES), "binding table out of sync with the header"
    assert lib.swvr_abi_version() == 2


def test_swvr_import_name_is_this_library():
    """``import swvr`` (the reference's package name) reaches this implementation."""
    import swvr as alias
    for name in ("softmax_readout", "softmax_readout_mse", "SoftmaxReadoutMSE", "softmax_readout_reference"):
        assert getattr(alias, name) is getattr(swvr, name), name
    assert sorted(alias.__all__) == sorted(swvr.__all__)
    assert alias.__version__ == swvr.__version__


def _problem(N=256, K=64, V=1000, D=16, dt=nat.BF16, ptr=1 << 20, chunk=8192, ld=None):
    p = nat.Problem()
    p.n_tokens, p.hidden, p.vocab, p.embed_dim = N, K, V, D
    p.compute_dtype, p.bias_dtype = dt, nat.F32
    p.h = p.W = p.E = ptr
    p.ldh = p.ldw = ld or K
    p.lde = (max(D, 8) + 7) // 8 * 8 if dt in (nat.BF16, nat.F16) else D  # pitch as ops._operand pads it
    p.logit_scale, p.chunk = 1.0, chunk
    return p


def test_workspace_planning_without_a_gpu():
    lib = nat.lib()
    nbytes = ctypes.c_size_t(0)
    assert lib.swvr_fwd_workspace_size(_problem(), ctypes.byref(nbytes)) == nat.OK and nbytes.value > 0
    g = nat.Grads()
    g.grad_h, g.grad_W, g.grad_E = 1 << 20, 1 << 20, 1 << 20
    # headline shape: the backward workspace (dS chunk, dh accumulator, partials) stays far below 3 GiB
    p = _problem(N=16384, K=2560, V=152064, D=64)
    assert lib.swvr_bwd_workspace_size(p, g, ctypes.byref(nbytes)) == nat.OK
    assert 16384 * 8192 * 2 < nbytes.value < 1.2 * 2 ** 30
    assert lib.swvr_fwd_workspace_size(_problem(dt=nat.F64, D=5, K=12), ctypes.byref(nbytes)) == nat.OK


@pytest.mark.parametrize("bad,code", [
    (dict(N=-1), nat.ERR_INVALID_ARGUMENT),
    (dict(chunk=0), nat.ERR_INVALID_ARGUMENT),
    (dict(dt=7), nat.ERR_INVALID_ARGUMENT),
    (dict(D=300), nat.ERR_UNSUPPORTED),          # tensor-core path: D <= 256
    (dict(K=12), nat.ERR_UNSUPPORTED),           # tensor-core path: K multiple of 8
    (dict(ptr=(1 << 20) + 2), nat.ERR_UNSUPPORTED),  # 16-byte alignment
    (dict(ld=32), nat.ERR_INVALID_ARGUMENT),     # row stride shorter than the row
])
def test_abi_argument_validation(bad, code):
    nbytes = ctypes.c_size_t(0)
    rc = nat.lib().swvr_fwd_workspace_size(_problem(**bad), ctypes.byref(nbytes))
    assert rc == code
    assert nat.last_error()
    with pytest.raises(ValueError if code == nat.ERR_INVALID_ARGUMENT else RuntimeError):
        nat.check(rc, "swvr_fwd_workspace_size")


def test_combine_and_mse_argument_validation():
    lib = nat.lib()
    assert lib.swvr_combine(0, 4, 4, nat.F32, None, None, None, None, None, None) == nat.ERR_INVALID_ARGUMENT
    assert lib.swvr_combine(2, 4, 4, nat.BF16, 1, 1, 1, 1, 1, None) == nat.ERR_INVALID_ARGUMENT
    assert lib.swvr_mse_fwd(4, 4, nat.F32, 1, 1, 1, None, 0.0, 9, 1, None, None) == nat.ERR_INVALID_ARGUMENT
    assert lib.swvr_mse_bwd(4, 4, nat.F32, 1, 1, 1, None, 0.0, nat.REDUCE_MEAN, 1, None, 1, 1, None, None,
                            None) == nat.ERR_INVALID_ARGUMENT


def test_cpu_tensors_raise_instead_of_falling_back():
    h, W, E = torch.randn(4, 8), torch.randn(10, 8), torch.randn(10, 3)
    with pytest.raises(RuntimeError, match="CUDA devices only"):
        swvr.softmax_readout(h, W, E)
    with pytest.raises(RuntimeError, match="CUDA devices only"):
        swvr.softmax_readout_mse(h, W, E, torch.randn(4, 3))


def test_input_validation_matches_reference():
    """swvr/api.py:14-22 and 37-38: ValueErrors before any device work."""
    h, W, E, b = torch.randn(6, 12), torch.randn(41, 12), torch.randn(41, 5), torch.randn(41)
    with pytest.raises(ValueError):
        swvr.softmax_readout(h, W[:, :-1], E)
    with pytest.raises(ValueError):
        swvr.softmax_readout(h, W, E[:-1])
    with pytest.raises(ValueError):
        swvr.softmax_readout(h, W, E, b[:-1])
    with pytest.raises(ValueError):
        swvr.softmax_readout(h, W, E, chunk_size=-1)
    with pytest.raises(ValueError):
        swvr.softmax_readout(h, W[None], E)
    with pytest.raises(ValueError):
        swvr.softmax_readout_mse(h, W, E, torch.randn(6, 5), reduction="max")


def test_chunk_and_dtype_resolution(monkeypatch):
    assert default_chunk_size() == 8192
    monkeypatch.setenv("SWVR_CHUNK", "1234")
    assert default_chunk_size() == 1234
    assert acc_dtype(torch.bfloat16) == torch.float32 and acc_dtype(torch.float64) == torch.float64


@pytest.mark.parametrize("dtype,adt", [(torch.bfloat16, torch.float32), (torch.float64, torch.float64)])
def test_fake_impls_give_shapes(dtype, adt):
    """The opaque custom ops' fake impls (what torch.compile traces) on meta tensors."""
    h = torch.empty(6, 16, dtype=dtype, device="meta")
    W = torch.empty(100, 16, dtype=dtype, device="meta")
    E = torch.empty(100, 5, dtype=dtype, device="meta")
    b = torch.empty(100, dtype=dtype, device="meta")
    O, lse = torch.ops.swvr_b200.fwd(h, W, E, b, 1.0, 8192, dtype)
    assert O.shape == (6, 5) and lse.shape == (6,) and O.dtype == adt
    grads = torch.ops.swvr_b200.bwd(O, lse, h, W, E, b, O, lse, 1.0, 8192, dtype, True, False, True, True)
    assert [tuple(g.shape) for g in grads] == [(6, 16), (0,), (100, 5), (100,)]
    loss, stats = torch.ops.swvr_b200.mse(O, lse, O, None, 0.0, 2)
    assert loss.shape == () and stats.shape == (nat.MSE_STATS_LEN,)


def test_module_holds_references():
    head, emb = torch.nn.Linear(12, 41), torch.nn.Embedding(41, 5)
    m = swvr.SoftmaxReadoutMSE(head, emb, z_loss_weight=1e-2)
    assert m.head is head and m.embedding is emb
    assert swvr.__version__ == "0.1.0"
    assert set(swvr.__all__) == {"softmax_readout", "softmax_readout_mse", "SoftmaxReadoutMSE",
                                 "softmax_readout_reference", "rmsnorm_softmax_readout",
                                 "rmsnorm_softmax_readout_mse"}


def test_wide_embedding_and_chunk_planning():
    """D up to 256 plans on the tensor-core path (257 is rejected); backward chunks are balanced:
    19008 rows (one shard of c2 on 8 GPUs) at chunk_size 8192 are two chunks of 9728, not
    16384 + 2624, so the dS buffer is sized for 9728 rows."""
    lib = nat.lib()
    nbytes = ctypes.c_size_t(0)
    for D in (129, 200, 256):
        assert lib.swvr_fwd_workspace_size(_problem(N=1000, K=512, V=5000, D=D), ctypes.byref(nbytes)) == nat.OK
    assert lib.swvr_fwd_workspace_size(_problem(D=257), ctypes.byref(nbytes)) == nat.ERR_UNSUPPORTED
    g = nat.Grads()
    g.grad_h, g.grad_W, g.grad_E = 1 << 20, 1 << 20, 1 << 20
    N = 16384
    assert lib.swvr_bwd_workspace_size(_problem(N=N, K=2560, V=19008, D=64), g, ctypes.byref(nbytes)) == nat.OK
    dh = N * 2560 * 4                       # the fp32 dh accumulator shares the workspace
    assert 9728 * N * 2 + dh < nbytes.value < 16384 * N * 2 + dh


def test_selftest_limits_are_checked_on_the_host():
    lib = nat.lib()
    assert lib.swvr_selftest_wait_timeout(10, None) == nat.ERR_INVALID_ARGUMENT
    assert lib.swvr_selftest_wait_timeout(20_000_000_000, None) == nat.ERR_INVALID_ARGUMENT
    assert "limit_ns" in nat.last_error()


def test_backward_token_tile_choice_and_override(monkeypatch):
    """The score kernel's token tile sets dS's token pitch and so the backward workspace:
    192-token tiles by default for D <= 64 with hidden >= 1024, 128 otherwise;
    SWVR_BWD_TOKEN_TILE=128|192 overrides where that tile exists (192 needs D <= 64)."""
    lib = nat.lib()
    g = nat.Grads()
    g.grad_h, g.grad_W, g.grad_E = 1 << 20, 1 << 20, 1 << 20

    def ws(tile, **kw):
        if tile is None:
            monkeypatch.delenv("SWVR_BWD_TOKEN_TILE", raising=False)
        else:
            monkeypatch.setenv("SWVR_BWD_TOKEN_TILE", tile)
        n = ctypes.c_size_t(0)
        assert lib.swvr_bwd_workspace_size(_problem(**kw), g, ctypes.byref(n)) == nat.OK
        return n.value

    long_k = dict(N=16384, K=2560, V=19008, D=64)
    # dS is [chunk rows, 86 x 192 = 16512 tokens] against 128 x 128 = 16384, and the dE / db
    # partial slots follow the token splits of each plan
    assert ws(None, **long_k) == ws("192", **long_k) != ws("128", **long_k)
    short_k = dict(N=16384, K=512, V=19008, D=64)
    assert ws(None, **short_k) == ws("128", **short_k) != ws("192", **short_k)
    wide_d = dict(N=16384, K=2560, V=19008, D=128)
    assert ws(None, **wide_d) == ws("128", **wide_d) == ws("192", **wide_d)


def test_forward_and_backward_reject_bad_arguments_before_any_launch():
    """swvr_fwd / swvr_bwd check their arguments on the host before touching the device (this
    container has none): NULL grads or backward inputs, a workspace smaller than the size
    query's, a grad_W dtype other than the compute dtype or fp32, a misaligned grad_W."""
    lib = nat.lib()
    p = _problem()
    buf, big = 1 << 20, 1 << 40
    assert lib.swvr_fwd(p, buf, buf, buf, 16, None) == nat.ERR_WORKSPACE
    assert lib.swvr_bwd(p, None, None, 0, None) == nat.ERR_INVALID_ARGUMENT
    g = nat.Grads()
    assert lib.swvr_bwd(p, g, None, 0, None) == nat.ERR_INVALID_ARGUMENT  # NULL O / lse / grad_O / grad_lse
    g.O = g.lse = g.grad_O = g.grad_lse = buf
    g.grad_W, g.grad_W_dtype, g.ld_grad_W = buf, nat.BF16, p.hidden
    assert lib.swvr_bwd(p, g, buf, 16, None) == nat.ERR_WORKSPACE
    g.grad_W_dtype = nat.F16
    assert lib.swvr_bwd(p, g, buf, big, None) == nat.ERR_UNSUPPORTED
    assert "grad_W" in nat.last_error()
    g.grad_W_dtype, g.grad_W = nat.BF16, buf + 8
    assert lib.swvr_bwd(p, g, buf, big, None) == nat.ERR_UNSUPPORTED
    assert "aligned" in nat.last_error()
    with pytest.raises(RuntimeError):
        nat.check(nat.ERR_UNSUPPORTED, "swvr_bwd")
