"""Pin the numpy oracle against golden vectors produced by the reference library itself.

The fixtures in tests/golden/ come from running pengzhangzhi/swvr (tests/golden/make_golden.py).
Every oracle function used by the GPU parity tests is checked here on CPU.
"""
import glob
import os

import numpy as np
import pytest

from oracle import swvr_oracle as orc
from tests.conftest import GOLDEN


def load(name):
    z = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    return {k: z[k] for k in z.files}


def rel(a, r):
    a = np.asarray(a, np.float64)
    r = np.asarray(r, np.float64)
    return float(np.linalg.norm(a - r) / max(np.linalg.norm(r), 1e-30))


F64_CASES = ["f64_basic", "f64_chunk1_nobias", "f64_large_logits", "f64_neginf_bias",
             "f64_tiny_vocab"]


def test_all_fixtures_present():
    names = {os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, "*.npz"))}
    expected = set(F64_CASES) | {"f64_mse_mean", "f64_mse_sum", "f64_mse_none",
                                 "c0_fp32_chunk8192", "c0_fp32_chunk128", "bf16_small",
                                 "bf16_medium"}
    assert expected <= names


@pytest.mark.parametrize("name", F64_CASES)
def test_chunked_oracle_matches_reference_fp64(name):
    c = load(name)
    b = c.get("b")
    O, lse = orc.chunked_forward(c["h"], c["W"], c["E"], b, float(c["scale"]), int(c["chunk"]), "fp64")
    np.testing.assert_allclose(O, c["O"], rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(lse, c["lse"], rtol=1e-10, atol=1e-12)
    gh, gW, gE, gb = orc.chunked_backward(c["gO"], c["glse"], c["h"], c["W"], c["E"], b, O, lse,
                                          float(c["scale"]), int(c["chunk"]), "fp64")
    np.testing.assert_allclose(gh, c["gh"], rtol=1e-9, atol=1e-12)
    np.testing.assert_allclose(gW, c["gW"], rtol=1e-9, atol=1e-12)
    np.testing.assert_allclose(gE, c["gE"], rtol=1e-9, atol=1e-12)
    if b is not None:
        np.testing.assert_allclose(gb, c["gb"], rtol=1e-9, atol=1e-12)


@pytest.mark.parametrize("name", F64_CASES)
def test_eager_oracle_and_analytic_grads_match_reference(name):
    c = load(name)
    b = c.get("b")
    O, lse = orc.softmax_readout_reference(c["h"], c["W"], c["E"], b, float(c["scale"]))
    np.testing.assert_allclose(O, c["O"], rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(lse, c["lse"], rtol=1e-10, atol=1e-12)
    gh, gW, gE, gb = orc.readout_grads(c["h"], c["W"], c["E"], b, c["gO"], c["glse"], float(c["scale"]))
    np.testing.assert_allclose(gh, c["gh"], rtol=1e-9, atol=1e-12)
    np.testing.assert_allclose(gW, c["gW"], rtol=1e-9, atol=1e-12)
    np.testing.assert_allclose(gE, c["gE"], rtol=1e-9, atol=1e-12)
    if b is not None:
        np.testing.assert_allclose(gb, c["gb"], rtol=1e-9, atol=1e-12)


def test_known_answer_dominant_logit():
    """test_cpu.py:81-88: with b[3] = 1e4, O equals E[3] exactly."""
    c = load("f64_large_logits")
    np.testing.assert_allclose(c["O"], np.broadcast_to(c["E"][3], c["O"].shape), rtol=0, atol=1e-12)


def test_known_answer_neginf_bias_has_zero_bias_grad():
    """test_cpu.py:91-105: the bias gradient at -inf entries is 0."""
    c = load("f64_neginf_bias")
    assert np.all(c["gb"][:16] == 0) and np.all(c["gb"][30:] == 0)


@pytest.mark.parametrize("reduction", ["mean", "sum", "none"])
def test_mse_oracle_matches_reference(reduction):
    c = load(f"f64_mse_{reduction}")
    O, lse = orc.chunked_forward(c["h"], c["W"], c["E"], c["b"], 0.5, 8, "fp64")
    np.testing.assert_allclose(O, c["O"], rtol=1e-10)
    loss = orc.mse_forward(O, lse, c["target"], c["weight"], reduction, float(c["z"]))
    np.testing.assert_allclose(loss, c["loss"].reshape(np.shape(loss)), rtol=1e-10)
    grad = c["grad_loss"] if reduction == "none" else float(c["grad_loss"][0])
    gO, glse, gt, gw = orc.mse_backward(O, lse, c["target"], c["weight"], reduction, float(c["z"]), grad)
    np.testing.assert_allclose(gt, c["gtarget"], rtol=1e-9, atol=1e-14)
    np.testing.assert_allclose(gw, c["gweight"], rtol=1e-9, atol=1e-14)
    gh, gW, gE, gb = orc.chunked_backward(gO, glse, c["h"], c["W"], c["E"], c["b"], O, lse, 0.5, 8, "fp64")
    np.testing.assert_allclose(gh, c["gh"], rtol=1e-9, atol=1e-14)
    np.testing.assert_allclose(gW, c["gW"], rtol=1e-9, atol=1e-14)
    np.testing.assert_allclose(gE, c["gE"], rtol=1e-9, atol=1e-14)
    np.testing.assert_allclose(gb, c["gb"], rtol=1e-9, atol=1e-14)


@pytest.mark.parametrize("chunk", [8192, 128])
def test_c0_fp32_oracle_matches_reference(chunk):
    """BASELINE configs[0] (fp32) MSE fwd+bwd."""
    c = load(f"c0_fp32_chunk{chunk}")
    O, lse = orc.chunked_forward(c["h"], c["W"], c["E"], c["b"], 1.0, chunk, "fp32")
    assert rel(O, c["O"]) < 1e-6 and rel(lse, c["lse"]) < 1e-6
    loss = orc.mse_forward(O, lse, c["target"])
    assert abs(float(loss) - float(c["loss"])) <= 1e-5 * abs(float(c["loss"]))
    gO, glse, _, _ = orc.mse_backward(O, lse, c["target"])
    gh, gW, gE, gb = orc.chunked_backward(gO, glse, c["h"], c["W"], c["E"], c["b"], O, lse, 1.0, chunk, "fp32")
    for a, r in ((gh, c["gh"]), (gW, c["gW"]), (gE, c["gE"]), (gb, c["gb"])):
        assert rel(a, r) < 1e-5


@pytest.mark.parametrize("name", ["bf16_small", "bf16_medium"])
def test_bf16_oracle_matches_reference_chunked_cpu(name):
    """The bf16 rounding points of the oracle reproduce the reference's chunked bf16 path."""
    c = load(name)
    s, C = float(c["scale"]), int(c["chunk"])
    O, lse = orc.chunked_forward(c["h"], c["W"], c["E"], c["b"], s, C, "bf16")
    assert rel(O, c["O"]) < 1e-5, rel(O, c["O"])
    assert np.max(np.abs(lse - c["lse"])) < 1e-4
    gh, gW, gE, gb = orc.chunked_backward(c["gO"], c["glse"], c["h"], c["W"], c["E"], c["b"], O, lse, s, C, "bf16")
    # the reference returns grads in the parameter dtype (bf16): compare after rounding
    for a, r in ((gh, c["gh"]), (gW, c["gW"]), (gE, c["gE"]), (gb, c["gb"])):
        assert rel(orc.round_bf16(a), r) < 3e-3, rel(orc.round_bf16(a), r)


def test_bf16_rounding_is_round_to_nearest_even():
    x = np.array([1.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, 1.0 + 2 ** -9, -2.5, np.inf, -np.inf, 0.0],
                 dtype=np.float32)
    y = orc.round_bf16(x)
    np.testing.assert_array_equal(y, np.array([1.0, 1.0, 1.0 + 2 ** -6, 1.0, -2.5, np.inf, -np.inf, 0.0],
                                              dtype=np.float32))
    assert np.isnan(orc.round_bf16(np.array([np.nan], np.float32)))[0]


def test_shard_combine_matches_eager():
    """Merging per-shard online-softmax states reproduces the unsharded result."""
    c = load("f64_basic")
    O_ref, lse_ref = orc.softmax_readout_reference(c["h"], c["W"], c["E"], c["b"], 0.5)
    for G in (1, 2, 3, 8):
        m2, l, acc = orc.shard_partials(c["h"], c["W"], c["E"], c["b"], 0.5, G)
        O, lse = orc.combine_partials(m2, l, acc)
        np.testing.assert_allclose(O, O_ref, rtol=1e-12)
        np.testing.assert_allclose(lse, lse_ref, rtol=1e-12)
