"""GPU parity: the CUDA path against the numpy oracle and the reference's golden vectors.

Ports the reference's GPU contracts (tests/test_cuda.py) and CPU contracts (tests/test_cpu.py,
here run on the GPU in fp64 through the exact SIMT kernels) with the oracle as the checker.
Tolerances: fp64 1e-10; fp32 1e-4 relative (north star) / 1e-5 (test_cuda.py:65);
bf16 / fp16 2e-2 relative norm-wise, LSE 1e-2 absolute.
"""
import numpy as np
import pytest
import torch
from torch import nn

from oracle import swvr_oracle as orc
from tests.helpers import (CDT, f64, functional_grads, load_golden, make_cpu, make_gpu, npy, oracle_eager,
                           rel_err)

pytestmark = pytest.mark.gpu

swvr = pytest.importorskip("swvr_b200")


def cuda(x, dtype=None):
    t = torch.as_tensor(np.asarray(x))
    t = t.to(dtype) if dtype is not None else t
    return t.cuda()


# ------------------------------------------------------------------------------ golden vectors
@pytest.mark.parametrize("name", ["f64_basic", "f64_chunk1_nobias", "f64_large_logits", "f64_neginf_bias",
                                  "f64_tiny_vocab"])
def test_golden_fp64(name):
    c = load_golden(name)
    h, W, E = (cuda(c[k]).requires_grad_(True) for k in ("h", "W", "E"))
    b = cuda(c["b"]).requires_grad_(True) if "b" in c else None
    O, lse = swvr.softmax_readout(h, W, E, b, logit_scale=float(c["scale"]), chunk_size=int(c["chunk"]))
    np.testing.assert_allclose(npy(O), c["O"], rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(npy(lse), c["lse"], rtol=1e-10, atol=1e-12)
    xs = [x for x in (h, W, E, b) if x is not None]
    grads = torch.autograd.grad((O * cuda(c["gO"])).sum() + (lse * cuda(c["glse"])).sum(), xs)
    for name_, g in zip(["gh", "gW", "gE", "gb"], grads):
        np.testing.assert_allclose(npy(g), c[name_], rtol=1e-9, atol=1e-12, err_msg=name_)


@pytest.mark.parametrize("reduction", ["mean", "sum", "none"])
def test_golden_mse(reduction):
    c = load_golden(f"f64_mse_{reduction}")
    h, W, E, b, t, w = (cuda(c[k]).requires_grad_(True) for k in ("h", "W", "E", "b", "target", "weight"))
    loss = swvr.softmax_readout_mse(h, W, E, t, b, weight=w, reduction=reduction, z_loss_weight=float(c["z"]),
                                    logit_scale=0.5, chunk_size=8)
    np.testing.assert_allclose(npy(loss), c["loss"].reshape(loss.shape), rtol=1e-10)
    gl = cuda(c["grad_loss"]).reshape(loss.shape)
    grads = torch.autograd.grad(loss, (h, W, E, b, t, w), gl)
    for k, g in zip(["gh", "gW", "gE", "gb", "gtarget", "gweight"], grads):
        np.testing.assert_allclose(npy(g), c[k], rtol=1e-9, atol=1e-13, err_msg=k)


@pytest.mark.parametrize("chunk", [8192, 128])
def test_golden_c0_fp32(chunk):
    """fp32 MSE fwd+bwd against the reference's outputs (1e-4 relative)."""
    c = load_golden(f"c0_fp32_chunk{chunk}")
    h, W, E, b = (cuda(c[k]).requires_grad_(True) for k in ("h", "W", "E", "b"))
    t = cuda(c["target"])
    O, lse = swvr.softmax_readout(h, W, E, b, chunk_size=chunk)
    assert O.dtype == torch.float32
    assert rel_err(O, c["O"]) < 1e-5 and rel_err(lse, c["lse"]) < 1e-5
    loss = swvr.softmax_readout_mse(h, W, E, t, b, chunk_size=chunk)
    assert abs(loss.item() - float(c["loss"])) <= 1e-4 * abs(float(c["loss"]))
    grads = torch.autograd.grad(loss, (h, W, E, b))
    for k, g in zip(["gh", "gW", "gE", "gb"], grads):
        assert rel_err(g, c[k]) < 1e-4, (k, rel_err(g, c[k]))


@pytest.mark.parametrize("name", ["bf16_small", "bf16_medium"])
def test_golden_bf16(name):
    """Tensor-core path against the reference's own bf16 chunked outputs and the oracle."""
    c = load_golden(name)
    h, W, E, b = (cuda(c[k], torch.bfloat16).requires_grad_(True) for k in ("h", "W", "E", "b"))
    s, C = float(c["scale"]), int(c["chunk"])
    O, lse = swvr.softmax_readout(h, W, E, b, logit_scale=s, chunk_size=C)
    assert O.dtype == torch.float32 and lse.dtype == torch.float32
    assert rel_err(O, c["O"]) < 2e-2
    assert np.max(np.abs(npy(lse) - c["lse"])) < 1e-2
    grads = torch.autograd.grad((O * cuda(c["gO"])).sum() + (lse * cuda(c["glse"])).sum(), (h, W, E, b))
    for k, g in zip(["gh", "gW", "gE", "gb"], grads):
        assert g.dtype == torch.bfloat16
        assert rel_err(g, c[k]) < 2e-2, (k, rel_err(g, c[k]))
    # the bf16-emulating chunked oracle restates the same rounding points: a tighter bound
    Oo, lo = orc.chunked_forward(c["h"], c["W"], c["E"], c["b"], s, C, "bf16")
    assert rel_err(O, Oo) < 5e-3 and np.max(np.abs(npy(lse) - lo)) < 2e-3


# ------------------------------------------------------------------------------ test_cuda.py contracts
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("chunk", [1024, 3000])
@pytest.mark.parametrize("D", [5, 16, 128, 200, 256])
def test_low_precision_matches_fp64(dtype, chunk, D):
    """test_cuda.py:37-54 with the fp64 numpy oracle as the checker (D = 200 and 256 run the
    tensor-core variant for D <= 256: single-buffered scores in the backward)."""
    N, K, V = 517, 512, 10007
    inputs = make_gpu(N, K, V, D, dtype)
    g = torch.Generator().manual_seed(3)
    gO = torch.randn(N, D, generator=g).cuda()
    glse = (0.1 * torch.randn(N, generator=g)).cuda()
    O, lse = swvr.softmax_readout(*inputs, chunk_size=chunk, logit_scale=0.8)
    grads = torch.autograd.grad((O * gO).sum() + (lse * glse).sum(), inputs)
    Or, lr, gr = oracle_eager(*inputs, 0.8, gO, glse)
    errs = {"O": rel_err(O, Or), "lse": rel_err(lse, lr)}
    errs.update({n: rel_err(a, r) for n, a, r in zip(["gh", "gW", "gE", "gb"], grads, gr)})
    print(dtype, chunk, D, {k: f"{v:.1e}" for k, v in errs.items()})
    for n, e in errs.items():
        assert e < 2e-2, (n, e)
    assert np.max(np.abs(npy(lse) - lr)) < 1e-2


def test_fp32_no_tf32_is_exact():
    """test_cuda.py:57-65: fp32 inputs without TF32 are exact to 1e-5."""
    N, K, V, D = 256, 128, 5000, 8
    inputs = make_gpu(N, K, V, D, torch.float32)
    g = torch.Generator().manual_seed(4)
    gO, glse = torch.randn(N, D, generator=g).cuda(), torch.randn(N, generator=g).cuda()
    O, lse = swvr.softmax_readout(*inputs, chunk_size=777)
    grads = torch.autograd.grad((O * gO).sum() + (lse * glse).sum(), inputs)
    Or, lr, gr = oracle_eager(*inputs, 1.0, gO, glse)
    for a, r in zip([O, lse, *grads], [Or, lr, *gr]):
        assert rel_err(a, r) < 1e-5, rel_err(a, r)


@pytest.mark.parametrize("N,K,V,D,chunk", [
    (2048, 256, 4096, 64, 1024),   # aligned: every GEMM on the split-TF32 kernel, dE and P.E split in K
    (1000, 200, 3000, 36, 1000),   # ragged tiles and K splits with a short last range
    (513, 130, 2001, 10, 700),     # unaligned rows: the CUDA-core kernel for some GEMMs
])
def test_fp32_split_tf32_gemms_are_exact(N, K, V, D, chunk):
    """The fp32 path's GEMMs (three-term split-TF32 tensor-core products, split in K where the
    output is narrow, the score bias in the GEMM's epilogue; CUDA-core fallback where the
    operands cannot be staged 16 bytes at a time) against the fp64 oracle at the fp32
    contract's 1e-5 (test_cuda.py:57-65)."""
    inputs = make_gpu(N, K, V, D, torch.float32, seed=9)
    g = torch.Generator().manual_seed(10)
    gO, glse = torch.randn(N, D, generator=g).cuda(), torch.randn(N, generator=g).cuda()
    O, lse = swvr.softmax_readout(*inputs, chunk_size=chunk, logit_scale=0.9)
    grads = torch.autograd.grad((O * gO).sum() + (lse * glse).sum(), inputs)
    Or, lr, gr = oracle_eager(*inputs, 0.9, gO, glse)
    for name, a, r in zip(["O", "lse", "gh", "gW", "gE", "gb"], [O, lse, *grads], [Or, lr, *gr]):
        assert rel_err(a, r) < 1e-5, (name, rel_err(a, r))


def test_autocast_with_fp32_params():
    """test_cuda.py:68-77: autocast bf16 with fp32 parameters keeps fp32 grads."""
    N, K, V, D = 256, 256, 4000, 16
    h, W, E, b = make_gpu(N, K, V, D, torch.float32)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        O, lse = swvr.softmax_readout(h, W, E, b, chunk_size=1024)
    assert O.dtype == torch.float32
    (O.sum() + lse.sum()).backward()
    assert W.grad.dtype == torch.float32 and h.grad.dtype == torch.float32
    Or, _ = orc.softmax_readout_reference(npy(h), npy(W), npy(E), npy(b))
    assert rel_err(O, Or) < 2e-2
    _, _, gr = oracle_eager(h, W, E, b, 1.0, torch.ones_like(O), torch.ones_like(lse))
    for a, r in zip([h.grad, W.grad, E.grad, b.grad], gr):
        assert rel_err(a, r) < 2e-2


def test_autocast_fp32_params_cast_per_chunk():
    """fp32 parameters under bf16 autocast: W and E are cast to bf16 one vocabulary chunk at a time
    (the reference's W[v0:v1].to(cdt), chunked.py:90-95), so no whole bf16 copy of W is held."""
    N, K, V, D, C = 1024, 1024, 131072, 16, 4096
    h, W, E, b = make_gpu(N, K, V, D, torch.float32)
    torch.cuda.synchronize()
    base = torch.cuda.memory_allocated()
    torch.cuda.reset_peak_memory_stats()
    with torch.autocast("cuda", dtype=torch.bfloat16):
        O, lse = swvr.softmax_readout(h, W, E, b, chunk_size=C)
    (O.sum() + lse.sum()).backward()
    torch.cuda.synchronize()
    extra = torch.cuda.max_memory_allocated() - base
    grads = sum(x.numel() * x.element_size() for x in (h, W, E, b))
    whole_copy = V * K * 2
    print(f"extra {extra / 2**20:.0f} MiB, grads {grads / 2**20:.0f} MiB, a whole bf16 W {whole_copy / 2**20:.0f} MiB")
    assert extra < grads + whole_copy // 2
    assert W.grad.dtype == torch.float32 and torch.isfinite(W.grad).all()


def test_autocast_fp32_params_odd_shapes():
    """The per-chunk parameter cast with K not a multiple of 8 (zero-padded per chunk), D = 5,
    fp16 autocast, an fp32 bias and a vocabulary that leaves a ragged last chunk."""
    N, K, V, D = 300, 100, 5003, 5
    h, W, E, b = make_gpu(N, K, V, D, torch.float32)
    g = torch.Generator().manual_seed(9)
    gO = torch.randn(N, D, generator=g).cuda()
    glse = (0.1 * torch.randn(N, generator=g)).cuda()
    with torch.autocast("cuda", dtype=torch.float16):
        O, lse = swvr.softmax_readout(h, W, E, b, chunk_size=1000, logit_scale=0.7)
    grads = torch.autograd.grad((O * gO).sum() + (lse * glse).sum(), (h, W, E, b))
    assert all(x.dtype == torch.float32 for x in grads)
    Or, lr, gr = oracle_eager(h, W, E, b, 0.7, gO, glse)
    assert rel_err(O, Or) < 2e-2 and np.max(np.abs(npy(lse) - lr)) < 1e-2
    for name, a_, r in zip(["gh", "gW", "gE", "gb"], grads, gr):
        assert rel_err(a_, r) < 2e-2, (name, rel_err(a_, r))


def test_wide_embedding_runs_simt():
    """D > 256 in bf16: the tensor-core kernels stop at 256, so the exact fp32 SIMT kernels run on
    fp32 copies of the operands; results still match the oracle within the 16-bit tolerance."""
    N, K, V, D = 200, 128, 2000, 300
    inputs = make_gpu(N, K, V, D, torch.bfloat16)
    g = torch.Generator().manual_seed(4)
    gO = torch.randn(N, D, generator=g).cuda()
    glse = (0.1 * torch.randn(N, generator=g)).cuda()
    O, lse = swvr.softmax_readout(*inputs, chunk_size=700)
    grads = torch.autograd.grad((O * gO).sum() + (lse * glse).sum(), inputs)
    Or, lr, gr = oracle_eager(*inputs, 1.0, gO, glse)
    assert rel_err(O, Or) < 2e-2 and np.max(np.abs(npy(lse) - lr)) < 1e-2
    for name, a_, r in zip(["gh", "gW", "gE", "gb"], grads, gr):
        assert rel_err(a_, r) < 2e-2, (name, rel_err(a_, r))
    assert all(x.dtype == torch.bfloat16 for x in grads)


def test_bf16_chunk_invariance():
    """test_cuda.py:80-86."""
    inputs = make_gpu(300, 256, 9000, 16, torch.bfloat16)
    g = torch.Generator().manual_seed(5)
    gO, glse = torch.randn(300, 16, generator=g).cuda(), torch.randn(300, generator=g).cuda()
    outs = []
    for C in (512, 9000):
        O, lse = swvr.softmax_readout(*inputs, chunk_size=C)
        grads = torch.autograd.grad((O * gO).sum() + (lse * glse).sum(), inputs)
        outs.append([O, lse, *grads])
    for x, y in zip(*outs):
        assert rel_err(x, y) < 1e-2


def test_peak_memory_is_chunk_bounded():
    """test_cuda.py:89-106: extra memory stays within grads + a few [N, C] fp32 tiles."""
    N, K, V, D, C = 4096, 1024, 65536, 16, 4096
    inputs = make_gpu(N, K, V, D, torch.bfloat16)
    target = torch.randn(N, D, device="cuda")
    torch.cuda.synchronize()
    base = torch.cuda.memory_allocated()
    torch.cuda.reset_peak_memory_stats()
    loss = swvr.softmax_readout_mse(*inputs[:3], target, inputs[3], chunk_size=C)
    loss.backward()
    torch.cuda.synchronize()
    extra = torch.cuda.max_memory_allocated() - base
    grads = sum(x.numel() * x.element_size() for x in inputs) + N * K * 4
    tiles = 6 * N * C * 4
    print(f"extra {extra / 2**20:.0f} MiB, budget {(grads + tiles) / 2**20:.0f} MiB")
    assert extra < grads + tiles


def test_masked_vocab_and_frozen_codebook():
    """test_cuda.py:109-121: -inf bias over whole vocabulary tiles with a frozen E."""
    N, K, V, D = 300, 256, 5000, 16
    h, W, E, b = make_gpu(N, K, V, D, torch.bfloat16)
    E.requires_grad_(False)
    with torch.no_grad():
        b[:2048] = float("-inf")
    g = torch.Generator().manual_seed(6)
    gO, glse = torch.randn(N, D, generator=g).cuda(), torch.randn(N, generator=g).cuda()
    O, lse = swvr.softmax_readout(h, W, E, b, chunk_size=1024)
    grads = torch.autograd.grad((O * gO).sum() + (lse * glse).sum(), (h, W, b))
    Or, lr, (gh, gW, _, gb) = oracle_eager(h, W, E, b, 1.0, gO, glse)
    for a, r in zip([O, lse, *grads], [Or, lr, gh, gW, gb]):
        assert torch.isfinite(a).all()
        assert rel_err(a, r) < 2e-2
    assert (grads[2][:2048] == 0).all()


def test_torch_compile_matches_eager_and_stays_chunked():
    """test_cuda.py:124-146."""
    N, K, V, D, C = 2048, 512, 32768, 16, 2048
    h, W, E, b = make_gpu(N, K, V, D, torch.bfloat16)
    target = torch.randn(N, D, device="cuda")
    fn = lambda h: swvr.softmax_readout_mse(h, W, E, target, b, chunk_size=C)
    torch._dynamo.reset()
    cfn = torch.compile(fn, fullgraph=True)
    for _ in range(2):
        torch.cuda.synchronize()
        base = torch.cuda.memory_allocated()
        torch.cuda.reset_peak_memory_stats()
        loss_c = cfn(h)
        g_c = torch.autograd.grad(loss_c, (h, W))
        torch.cuda.synchronize()
        extra = torch.cuda.max_memory_allocated() - base
    loss_e = fn(h)
    g_e = torch.autograd.grad(loss_e, (h, W))
    assert rel_err(loss_c, loss_e) < 1e-3
    for a, r in zip(g_c, g_e):
        assert rel_err(a, r) < 1e-2
    assert extra < N * V * 2


# ------------------------------------------------------------------------------ test_cpu.py contracts on GPU
def assert_matches_oracle(h, W, E, b, scale=1.0, chunk=8, rtol=1e-10, atol=1e-12):
    fast = lambda *a: swvr.softmax_readout(*a, logit_scale=scale, chunk_size=chunk)
    (O, lse), (gO, glse), grads = functional_grads(fast, (h, W, E, b))
    Or, lr, gr = oracle_eager(h, W, E, b, scale, gO, glse)
    np.testing.assert_allclose(npy(O), Or, rtol=rtol, atol=atol)
    np.testing.assert_allclose(npy(lse), lr, rtol=rtol, atol=atol)
    # the same tensor passed twice (tied W = E) receives the sum of both gradients
    ref = {}
    for x, r in zip((h, W, E, b), gr):
        if x is not None and r is not None:
            ref[id(x)] = ref.get(id(x), 0) + r
    xs = []
    for x in (h, W, E, b):
        if x is not None and x.requires_grad and all(x is not y for y in xs):
            xs.append(x)
    for x, g in zip(xs, grads):
        np.testing.assert_allclose(npy(g), ref[id(x)], rtol=rtol, atol=atol)


@pytest.mark.parametrize("chunk", [1, 3, 8, 40, 41, 42, 1000])
def test_chunk_sizes_match_oracle(chunk):
    assert_matches_oracle(*make_cpu(), chunk=chunk)


@pytest.mark.parametrize("bias", [True, False])
@pytest.mark.parametrize("scale", [1.0, 0.3, 2.5])
def test_gradcheck(bias, scale):
    h, W, E, b = make_cpu(N=4, K=6, V=13, D=3, bias=bias)
    fn = lambda *a: swvr.softmax_readout(*a, logit_scale=scale, chunk_size=5)
    assert torch.autograd.gradcheck(fn, (h, W, E, b))


def test_leading_dims_and_non_contiguous():
    h, W, E, b = make_cpu(lead=(2, 3, 4))
    O, lse = swvr.softmax_readout(h, W, E, b, chunk_size=7)
    assert O.shape == (2, 3, 4, 5) and lse.shape == (2, 3, 4)
    Or, lr = orc.softmax_readout_reference(npy(h).reshape(-1, 12), npy(W), npy(E), npy(b))
    np.testing.assert_allclose(npy(O).reshape(-1, 5), Or, rtol=1e-10)
    h, W, E, b = make_cpu(N=8)
    h_t = h.detach().t().contiguous().t()[::2].requires_grad_(True)
    assert not h_t.is_contiguous()
    assert_matches_oracle(h_t, W, E, b)


@pytest.mark.parametrize("dtype", [f64, torch.bfloat16])
def test_empty_batch(dtype):
    h, W, E, b = make_cpu(N=0, K=16, D=8, dtype=dtype)
    O, lse = swvr.softmax_readout(h, W, E, b, chunk_size=8)
    assert O.shape == (0, 8) and lse.shape == (0,)
    (O.sum() + lse.sum()).backward()
    assert W.grad.abs().sum() == 0 and E.grad.abs().sum() == 0 and b.grad.abs().sum() == 0


def test_single_token_and_tiny_vocab():
    assert_matches_oracle(*make_cpu(N=1, V=1), chunk=8)
    assert_matches_oracle(*make_cpu(N=1, V=2), chunk=1)


@pytest.mark.parametrize("dtype", [f64, torch.bfloat16])
def test_large_logits_no_overflow(dtype):
    """test_cpu.py:81-88: a dominant token's bias of 1e4 gives O == E[3] exactly."""
    h, W, E, b = make_cpu(K=16, V=300, D=8, dtype=dtype)
    with torch.no_grad():
        b[3] = 1e4
        b[7] = -1e4
    O, lse = swvr.softmax_readout(h, W, E, b, chunk_size=8)
    torch.testing.assert_close(O, E[3].to(O.dtype).expand_as(O).detach())
    if dtype == f64:
        assert_matches_oracle(h, W, E, b)


@pytest.mark.parametrize("dtype", [f64, torch.bfloat16])
def test_masked_vocab_with_neg_inf_bias(dtype):
    """test_cpu.py:91-105, and whole tensor-core vocabulary tiles masked for bf16."""
    V = 40 if dtype == f64 else 1000
    h, W, E, b = make_cpu(K=16, V=V, D=8, dtype=dtype)
    with torch.no_grad():
        b[: V * 2 // 5] = float("-inf")
        b[V * 3 // 4:] = float("-inf")
    fast = lambda *a: swvr.softmax_readout(*a, chunk_size=8)
    (O, lse), (gO, glse), grads = functional_grads(fast, (h, W, E, b))
    Or, lr, gr = oracle_eager(h, W, E, b, 1.0, gO, glse)
    tol = dict(rtol=1e-10, atol=1e-12) if dtype == f64 else dict(rtol=3e-2, atol=3e-2)
    np.testing.assert_allclose(npy(O), Or, **tol)
    np.testing.assert_allclose(npy(lse), lr, **tol)
    assert (grads[3][: V * 2 // 5] == 0).all() and (grads[3][V * 3 // 4:] == 0).all()
    if dtype == f64:
        for a, r in zip(grads, gr):
            np.testing.assert_allclose(npy(a), r, rtol=1e-9, atol=1e-12)
    else:
        for a, r in zip(grads, gr):
            assert rel_err(a, r) < 2e-2


@pytest.mark.parametrize("frozen", ["h", "W", "E", "b", "WE", "hW"])
@pytest.mark.parametrize("dtype,tile", [(f64, None), (torch.bfloat16, "128"), (torch.bfloat16, "192")])
def test_frozen_inputs(monkeypatch, frozen, dtype, tile):
    """Frozen inputs skip their work (no dE / db partials, no dS when neither h nor W needs a
    gradient); bf16 runs both score-tile widths."""
    if tile is not None:
        monkeypatch.setenv("SWVR_BWD_TOKEN_TILE", tile)
    h, W, E, b = make_cpu(K=16, V=300, D=8, dtype=dtype)
    names = dict(h=h, W=W, E=E, b=b)
    for k in frozen:
        names[k].requires_grad_(False)
    if dtype == f64:
        assert_matches_oracle(h, W, E, b)
        return
    fast = lambda *a: swvr.softmax_readout(*a, chunk_size=128)
    (O, lse), (gO, glse), grads = functional_grads(fast, (h, W, E, b))
    _, _, gr = oracle_eager(h, W, E, b, 1.0, gO, glse)
    ref = dict(zip("hWEb", gr))
    live = [k for k in "hWEb" if names[k].requires_grad]
    for k, g in zip(live, grads):
        assert rel_err(g, ref[k]) < 2e-2, k


def test_tied_W_and_E():
    h, W, _, b = make_cpu(K=7, D=7)
    assert_matches_oracle(h, W, W, b)
    h, W, _, b = make_cpu(K=16, D=16, V=500, dtype=torch.bfloat16)
    O, lse = swvr.softmax_readout(h, W, W, b, chunk_size=256)
    (O.sum() + lse.sum()).backward()
    _, _, gr = oracle_eager(h, W, W, b, 1.0, torch.ones_like(O), torch.ones_like(lse))
    assert rel_err(W.grad, gr[1] + gr[2]) < 2e-2


def test_only_lse_or_only_O_used():
    h, W, E, b = make_cpu()
    for pick in (0, 1):
        out = swvr.softmax_readout(h, W, E, b, chunk_size=8)[pick].sum()
        g = torch.autograd.grad(out, (h, W, E, b), allow_unused=True)
        O, lse = swvr.softmax_readout(h, W, E, b)
        gO = torch.ones_like(O) if pick == 0 else torch.zeros_like(O)
        glse = torch.ones_like(lse) if pick == 1 else torch.zeros_like(lse)
        _, _, gr = oracle_eager(h, W, E, b, 1.0, gO, glse)
        for a, r in zip(g, gr):
            if a is None:
                assert np.abs(r).max() == 0
            else:
                np.testing.assert_allclose(npy(a), r, rtol=1e-9, atol=1e-12)


def test_fp32_inputs():
    h, W, E, b = make_cpu(dtype=torch.float32)
    assert_matches_oracle(h, W, E, b, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("reduction", ["mean", "sum", "none"])
@pytest.mark.parametrize("dtype", [f64, torch.bfloat16])
def test_mse_matches_oracle(reduction, dtype):
    h, W, E, b = make_cpu(lead=(2, 3), K=16, V=200, D=8, dtype=dtype)
    g = torch.Generator().manual_seed(9)
    target = torch.randn(2, 3, 8, generator=g, dtype=f64).cuda().requires_grad_(True)
    weight = torch.tensor([[1., 0., 2.], [1., 1., 0.]], dtype=f64).cuda().requires_grad_(True)
    kw = dict(weight=weight, reduction=reduction, z_loss_weight=0.1, logit_scale=0.5)
    loss = swvr.softmax_readout_mse(h, W, E, target, b, chunk_size=8, **kw)
    O, lse = orc.softmax_readout_reference(npy(h).reshape(6, 16), npy(W), npy(E), npy(b), logit_scale=0.5)
    ref = orc.mse_forward(O, lse, npy(target).reshape(6, 8), npy(weight).reshape(6), reduction, 0.1)
    tol = dict(rtol=1e-9) if dtype == f64 else dict(rtol=2e-2, atol=1e-3)
    np.testing.assert_allclose(npy(loss).reshape(-1), np.reshape(ref, -1), **tol)
    gl = torch.ones_like(loss)
    grads = torch.autograd.grad(loss, (h, W, E, b, target, weight), gl)
    gO, glse, gt, gw = orc.mse_backward(O, lse, npy(target).reshape(6, 8), npy(weight).reshape(6), reduction, 0.1,
                                        1.0 if reduction != "none" else np.ones(6))
    gr = orc.readout_grads(npy(h).reshape(6, 16), npy(W), npy(E), npy(b), gO, glse, logit_scale=0.5)
    refs = [gr[0].reshape(2, 3, 16), gr[1], gr[2], gr[3], gt.reshape(2, 3, 8), gw.reshape(2, 3)]
    for a, r in zip(grads, refs):
        if dtype == f64:
            np.testing.assert_allclose(npy(a), r, rtol=1e-8, atol=1e-12)
        else:
            assert rel_err(a, r) < 3e-2


def test_module_wraps_linear_and_embedding():
    torch.manual_seed(0)
    head, emb = nn.Linear(12, 41).double().cuda(), nn.Embedding(41, 5).double().cuda()
    h, target = torch.randn(7, 12, dtype=f64).cuda(), torch.randn(7, 5, dtype=f64).cuda()
    loss_fn = swvr.SoftmaxReadoutMSE(head, emb, z_loss_weight=1e-2, chunk_size=8)
    loss = loss_fn(h, target)
    O, lse = orc.softmax_readout_reference(npy(h), npy(head.weight), npy(emb.weight), npy(head.bias))
    ref = orc.mse_forward(O, lse, npy(target), None, "mean", 1e-2)
    np.testing.assert_allclose(loss.item(), ref, rtol=1e-10)
    loss.backward()
    assert head.weight.grad is not None and head.bias.grad is not None and emb.weight.grad is not None


@pytest.mark.parametrize("dtype", [f64, torch.bfloat16])
def test_activation_checkpointing(dtype):
    from torch.utils.checkpoint import checkpoint
    h, W, E, b = make_cpu(K=16, V=300, D=8, dtype=dtype)
    fn = lambda h: swvr.softmax_readout(h, W, E, b, chunk_size=128)[0].pow(2).sum()
    g1 = torch.autograd.grad(checkpoint(fn, h, use_reentrant=False), h)[0]
    g2 = torch.autograd.grad(fn(h), h)[0]
    torch.testing.assert_close(g1, g2)


def test_input_validation():
    h, W, E, b = make_cpu()
    with pytest.raises(ValueError):
        swvr.softmax_readout(h, W[:, :-1], E)
    with pytest.raises(ValueError):
        swvr.softmax_readout(h, W, E[:-1])
    with pytest.raises(ValueError):
        swvr.softmax_readout(h, W, E, b[:-1])
    with pytest.raises(ValueError):
        swvr.softmax_readout(h, W, E, chunk_size=-1)
    with pytest.raises(ValueError):
        swvr.softmax_readout_mse(h, W, E, torch.zeros(6, 5, dtype=f64, device="cuda"), reduction="max")


# ------------------------------------------------------------------------------ tensor-core edge shapes
@pytest.mark.parametrize("N,K,V,D", [(1, 8, 1, 1), (129, 64, 193, 8), (255, 136, 385, 64), (130, 200, 160, 72),
                                     (64, 1000, 4097, 128)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_tensor_core_tails(N, K, V, D, dtype):
    """Token, vocabulary, hidden and embedding tails that do not fill a tile."""
    inputs = make_gpu(N, K, V, D, dtype)
    g = torch.Generator().manual_seed(11)
    gO, glse = torch.randn(N, D, generator=g).cuda(), torch.randn(N, generator=g).cuda()
    O, lse = swvr.softmax_readout(*inputs, chunk_size=256, logit_scale=0.7)
    grads = torch.autograd.grad((O * gO).sum() + (lse * glse).sum(), inputs)
    Or, lr, gr = oracle_eager(*inputs, 0.7, gO, glse)
    assert rel_err(O, Or) < 2e-2 and np.max(np.abs(npy(lse) - lr)) < 1e-2
    for n, a, r in zip(["gh", "gW", "gE", "gb"], grads, gr):
        assert rel_err(a, r) < 2e-2, (n, rel_err(a, r))


# ------------------------------------------------------------------------------ backward score tiles
@pytest.mark.parametrize("N,K,V,D", [(1, 64, 300, 64), (191, 136, 385, 16), (193, 256, 1000, 64),
                                     (1000, 1024, 5003, 40)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_backward_192_token_tiles(monkeypatch, N, K, V, D, dtype):
    """192-token score tiles (dP^T in three 64-token chunks), forced on small shapes: a single
    token, ragged last token tiles, vocabulary tails, D below 64."""
    monkeypatch.setenv("SWVR_BWD_TOKEN_TILE", "192")
    inputs = make_gpu(N, K, V, D, dtype)
    g = torch.Generator().manual_seed(12)
    gO, glse = torch.randn(N, D, generator=g).cuda(), torch.randn(N, generator=g).cuda()
    O, lse = swvr.softmax_readout(*inputs, chunk_size=512, logit_scale=0.7)
    grads = torch.autograd.grad((O * gO).sum() + (lse * glse).sum(), inputs)
    Or, lr, gr = oracle_eager(*inputs, 0.7, gO, glse)
    assert rel_err(O, Or) < 2e-2 and np.max(np.abs(npy(lse) - lr)) < 1e-2
    for n, a, r in zip(["gh", "gW", "gE", "gb"], grads, gr):
        assert rel_err(a, r) < 2e-2, (n, rel_err(a, r))


@pytest.mark.parametrize("N,K,V,D,chunk", [(8192, 1024, 8192, 64, 4096), (3000, 2048, 3001, 40, 8192)])
def test_backward_token_tiles_agree(monkeypatch, N, K, V, D, chunk):
    """128- and 192-token score tiles on units of many token tiles (a tile's later dP^T chunks
    are issued during the next tile's S K-loop).  Both compute the same S, P and dS, and the
    GEMMs only add zero token blocks, so dh and dW agree bit for bit; dE and db sum the same
    terms grouped by different token tiles."""
    inputs = make_gpu(N, K, V, D, torch.bfloat16)
    g = torch.Generator().manual_seed(13)
    gO, glse = torch.randn(N, D, generator=g).cuda(), torch.randn(N, generator=g).cuda()
    res = {}
    for tile in ("128", "192"):
        monkeypatch.setenv("SWVR_BWD_TOKEN_TILE", tile)
        xs = [x.detach().clone().requires_grad_(True) for x in inputs]
        O, lse = swvr.softmax_readout(*xs, chunk_size=chunk)
        torch.autograd.backward([O, lse], [gO, glse])
        res[tile] = [x.grad for x in xs]
    a, b = res["128"], res["192"]
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
    assert rel_err(b[2], a[2]) < 1e-3 and rel_err(b[3], a[3]) < 1e-3


@pytest.mark.parametrize("tile", ["128", "192"])
def test_backward_unit_order_is_bit_exact(monkeypatch, tile):
    """The score kernel's unit order (SWVR_BWD_GROUP: vocabulary tiles per group walking the
    token splits) changes which pair computes which (vocabulary tile, token split) and when,
    never what a unit computes or where its partial dE / db lands: every gradient is
    bit-identical for groups of 1 (splits of a tile in a row), 3 and 7 (short last groups) and
    one group for the whole chunk.  Checked against the oracle too."""
    N, K, V, D = 3000, 1024, 12011, 64
    monkeypatch.setenv("SWVR_BWD_TOKEN_TILE", tile)
    inputs = make_gpu(N, K, V, D, torch.bfloat16, seed=17)
    g = torch.Generator().manual_seed(14)
    gO, glse = torch.randn(N, D, generator=g).cuda(), torch.randn(N, generator=g).cuda()
    res = {}
    for grp in ("1", "3", "7", "1000"):
        monkeypatch.setenv("SWVR_BWD_GROUP", grp)
        xs = [x.detach().clone().requires_grad_(True) for x in inputs]
        O, lse = swvr.softmax_readout(*xs, chunk_size=4096)
        torch.autograd.backward([O, lse], [gO, glse])
        res[grp] = [x.grad for x in xs]
    for grp in ("3", "7", "1000"):
        for n, a, b in zip(["gh", "gW", "gE", "gb"], res["1"], res[grp]):
            assert torch.equal(a, b), (grp, n)
    _, _, gr = oracle_eager(*inputs, 1.0, gO, glse)
    for n, a, r in zip(["gh", "gW", "gE", "gb"], res["7"], gr):
        assert rel_err(a, r) < 2e-2, (n, rel_err(a, r))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_reference_rise_inside_a_tile(dtype):
    """Scores that climb past the forward's emergency margin (64 octaves for bf16, 8 for fp16)
    inside a 192-column tile while the values just under the margin stay significant: the
    kernel's first pass over the tile raises the running reference to the tile's max before
    any P of the tile is written, so no 16-bit P is rescaled.  Checked against the fp64
    oracle."""
    m = 64.0 if dtype == torch.bfloat16 else 8.0
    N, K, V, D = 130, 64, 1000, 16
    g = torch.Generator().manual_seed(21)
    # log2-unit pattern of each 192-column tile, per 32-column block: ~0 (sets the reference),
    # just under the margin, just over it (first rise), under the next margin, over it, near it
    base = torch.tensor([-0.3, m - 0.3, m + 0.4, 2 * m + 0.2, 2 * m + 1.5, 2 * m + 1.8], dtype=f64)
    col = torch.arange(V)
    t = base[(col % 192) // 32] + 0.1 * torch.rand(V, generator=g, dtype=f64)
    b = (t * np.log(2.0)).to(torch.float32)                        # fp32 bias: no 16-bit rounding of t
    h = torch.randn(N, K, generator=g).to(dtype)
    W = (0.05 * K ** -0.5 * torch.randn(V, K, generator=g)).to(dtype)  # rows differ by a few hundredths
    E = torch.randn(V, D, generator=g).to(dtype)
    O, lse = swvr.softmax_readout(h.cuda(), W.cuda(), E.cuda(), b.cuda())
    Or, lr = orc.softmax_readout_reference(npy(h), npy(W), npy(E), npy(b))
    assert torch.isfinite(O).all() and torch.isfinite(lse).all()
    assert rel_err(O, Or) < 2e-2, rel_err(O, Or)
    assert np.abs(npy(lse) - lr).max() < 1e-2


@pytest.mark.parametrize("at", [3, 100, 250, 299])
def test_dominant_token_anywhere_is_exact_in_bf16(at):
    """test_cpu.py:81-88 with the dominant token (bias 1e4) in any 32-column block of any tile:
    its P is exactly 1 and every other P is 0, so O == E[at] exactly."""
    h, W, E, b = make_cpu(K=16, V=300, D=8, dtype=torch.bfloat16)
    with torch.no_grad():
        b[at] = 1e4
    O, _ = swvr.softmax_readout(h, W, E, b)
    torch.testing.assert_close(O, E[at].to(O.dtype).expand_as(O).detach(), rtol=0, atol=0)
