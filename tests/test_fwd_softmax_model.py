"""A model of the forward kernel's online softmax for one token row (swvr_b200/csrc/tc_fwd.cu,
softmax warps), checked against the exact softmax on adversarial logits (CPU only).

The kernel works in base-2 units, t = S*s*log2(e) + b*log2(e).  Per 192-column vocabulary
tile it makes two passes over S: the first finds the tile's max tm; if tm exceeds the running
reference ``ref`` by more than kEmergency octaves (64 for bf16, 8 for fp16), ``ref`` becomes
tm and l (now) and O (after the previous P.E) are multiplied by 2^(old - new) in fp32; the
second pass writes P = 2^(t - ref), summed unrounded into l (fp32) and rounded to 16 bits for
O += P.E (fp32 accumulation).  No P value is rescaled after it was rounded.  O = acc / l and
LSE = (ref + log2 l) ln 2.  The model restates those steps in numpy with the same roundings
and checks finiteness and the 16-bit error bound where the reference's own algorithm would
also be finite, that every P value carries one rounding, and that a dominant token gives
O == E exactly.
"""
import numpy as np
import pytest

from oracle import swvr_oracle as orc

LN2 = np.log(2.0)


def kernel_row(t, E, cdt="bf16", tile=192, block=32, trace=None):
    """O [D] and LSE of one row as fwd_kernel computes them (float32 state, 16-bit P).  With a
    list ``trace``, each tile's (t, P, ref) is appended to it."""
    f32 = np.float32
    k_emergency = f32(64.0 if cdt == "bf16" else 8.0)
    rnd = (lambda x: orc.round_bf16(x)) if cdt == "bf16" else (lambda x: orc.round_fp16(x))
    Eq = rnd(E.astype(np.float64)).astype(f32)
    ref, l = f32(-np.inf), f32(0.0)
    acc = np.zeros(E.shape[1], dtype=f32)
    for v0 in range(0, len(t), tile):
        tt = t[v0:v0 + tile].astype(f32)
        ref_start, alpha = ref, f32(1.0)
        tm = tt.max()                                  # pass 1
        if tm > ref + k_emergency:
            alpha = f32(0.0) if ref == -np.inf else f32(np.exp2(f32(ref - tm)))
            ref, l = tm, f32(l * alpha)
        refe = f32(0.0) if ref == -np.inf else ref
        p = np.exp2(tt - refe).astype(f32)             # pass 2
        lsum = f32(0.0)
        for c0 in range(0, len(tt), block):            # the kernel sums block by block
            lsum = f32(lsum + p[c0:c0 + block].sum(dtype=f32))
        P = rnd(p.astype(np.float64)).astype(f32)
        l = f32(l + lsum)
        if v0 > 0 and ref != ref_start:
            acc = (acc * alpha).astype(f32)
        acc = (acc + P @ Eq[v0:v0 + tile]).astype(f32)
        if trace is not None:
            trace.append((tt, P.copy(), ref))
    O = acc / l
    lse = (np.float64(ref) + np.log2(np.float64(l))) * LN2
    return O, lse


def exact_row(t, E):
    x = t.astype(np.float64) * LN2
    m = x.max()
    w = np.exp(x - m)
    return (w @ E) / w.sum(), m + np.log(w.sum())


def _logit_rows(V, rng):
    ramp = np.linspace(-30.0, 300.0, V)  # rising logits: a new reference in nearly every block
    return {
        "gaussian": rng.normal(0, 3, V),
        "wide": rng.normal(0, 80, V),
        "rising": ramp + rng.normal(0, 0.5, V),
        "falling": ramp[::-1].copy(),
        "one_dominant": np.where(np.arange(V) == V // 3, 1e4, rng.normal(0, 1, V)),
        "masked_tail": np.where(np.arange(V) < V // 2, rng.normal(0, 2, V), -np.inf),
        "masked_head": np.where(np.arange(V) < 400, -np.inf, rng.normal(0, 2, V)),
        "large_offset": 5000.0 + rng.normal(0, 4, V),
    }


@pytest.mark.parametrize("cdt", ["bf16", "fp16"])
@pytest.mark.parametrize("kind", ["gaussian", "wide", "rising", "falling", "one_dominant", "masked_tail",
                                  "masked_head", "large_offset"])
def test_online_softmax_row_matches_exact(cdt, kind):
    rng = np.random.default_rng(7)
    V, D = 1000, 16
    t = _logit_rows(V, rng)[kind]
    E = rng.normal(0, 1, (V, D))
    O, lse = kernel_row(t, E, cdt)
    O_ref, lse_ref = exact_row(t, orc.round_to(E, cdt))
    assert np.isfinite(O).all() and np.isfinite(lse)
    # 16-bit P (one rounding each, also where the reference moved within a tile) against exact weights
    assert np.linalg.norm(O - O_ref) <= 2e-2 * max(np.linalg.norm(O_ref), 1e-30) + 1e-6
    assert abs(lse - lse_ref) <= 1e-5 * max(1.0, abs(lse_ref))


def test_rising_logits_exercise_the_rescale():
    """The rising row moves the reference in several tiles, so the rescale path is what the
    comparison above checks."""
    t = np.linspace(-30.0, 300.0, 1000)
    moves, ref = 0, -np.inf
    for v0 in range(0, 1000, 192):
        tm = t[v0:v0 + 192].max()
        if tm > ref + 64:
            moves, ref = moves + 1, tm
    assert moves >= 3


@pytest.mark.parametrize("kind", ["rising", "staircase"])
def test_probabilities_carry_one_rounding(kind):
    """Each bf16 P value is within one rounding (2^-8 relative: half the spacing of 7 stored
    fraction bits) of the exact 2^(t - ref) for its tile's reference, also where the reference
    moved inside a tile's columns -- rescaling an already-rounded P by a factor that is not a
    power of two could reach about 2^-7.  The staircase puts values just under the margin next
    to values just over it."""
    rng = np.random.default_rng(3)
    V = 960
    if kind == "rising":
        t = np.linspace(-30.0, 300.0, V) + rng.normal(0, 0.5, V)
    else:
        base = np.array([-0.3, 63.7, 64.4, 128.2, 129.5, 129.8])
        t = base[(np.arange(V) % 192) // 32] + 0.1 * rng.random(V)
    trace = []
    kernel_row(t, rng.normal(0, 1, (V, 8)), "bf16", trace=trace)
    checked = 0
    for tt, P, ref in trace:
        exact = np.exp2(tt.astype(np.float64) - np.float64(ref))
        normal = exact > 2.0 ** -120
        err = np.abs(P[normal] - exact[normal]) / exact[normal]
        assert err.max() <= 2.0 ** -8 + 1e-6, err.max()
        checked += int(normal.sum())
    assert checked > V // 4


@pytest.mark.parametrize("at", [3, 100, 500])
@pytest.mark.parametrize("cdt", ["bf16", "fp16"])
def test_dominant_token_is_exact(at, cdt):
    """A token 1e4 nats above the rest gives P = 1 exactly for it and 0 elsewhere, so O equals
    its E row exactly (the reference's test_cpu.py:81-88), wherever the token sits."""
    rng = np.random.default_rng(1)
    t = rng.normal(0, 1, 700) / LN2
    t[at] = 1e4 / LN2
    E = rng.normal(0, 1, (700, 8))
    O, _ = kernel_row(t, E, cdt)
    Eq = orc.round_to(E, cdt).astype(np.float32)
    np.testing.assert_array_equal(O, Eq[at])
