"""A model of the forward kernel's online softmax for one token row (swvr_b200/csrc/tc_fwd.cu,
softmax warps), checked against the exact softmax on adversarial logits (CPU only).

The kernel works in base-2 units, t = S*s*log2(e) + b*log2(e).  Per 192-column vocabulary
tile it reads 32-column blocks; the running reference ``ref`` is a whole number.  A block
whose max cm exceeds ``ref`` by more than kEmergency octaves (64 for bf16, 8 for fp16) raises
``ref`` by ceil(cm - ref) octaves (to ceil(cm) from -inf), and the tile's P values already
written (16-bit), l and the running sum are multiplied by 2^(old - new), an exact power of two,
so the rescaled P values keep a single 16-bit rounding.  P = 2^(t - ref) is summed unrounded
into l (fp32) and rounded to 16 bits for O += P.E (fp32 accumulation); once per tile O is
rescaled by the same kind of factor if ``ref`` moved.  O = acc / l and
LSE = (ref + log2 l) ln 2.  The model restates those steps in numpy with the same roundings
and checks finiteness and the 16-bit error bound where the reference's own algorithm would
also be finite, and that every P value of a tile carries one rounding after its rescales.
"""
import numpy as np
import pytest

from oracle import swvr_oracle as orc

LN2 = np.log(2.0)


def _exp2_neg_int(k):
    """2^-k for a whole number k >= 0 (0 below the smallest normal float), as the kernel builds it."""
    return np.float32(0.0) if k >= 127 else np.float32(2.0 ** -int(k))


def kernel_row(t, E, cdt="bf16", tile=192, block=32, trace=None):
    """O [D] and LSE of one row as fwd_kernel computes them (float32 state, 16-bit P).  With a
    list ``trace``, each tile's final (t, P, ref) is appended to it."""
    f32 = np.float32
    k_emergency = f32(64.0 if cdt == "bf16" else 8.0)
    rnd = (lambda x: orc.round_bf16(x)) if cdt == "bf16" else (lambda x: orc.round_fp16(x))
    Eq = rnd(E.astype(np.float64)).astype(f32)
    ref, l = f32(-np.inf), f32(0.0)
    acc = np.zeros(E.shape[1], dtype=f32)
    for v0 in range(0, len(t), tile):
        tt = t[v0:v0 + tile].astype(f32)
        ref_start = ref
        P = np.zeros(len(tt), dtype=f32)
        lsum = f32(0.0)
        for c0 in range(0, len(tt), block):
            x = tt[c0:c0 + block]
            cm = x.max()
            if cm > ref + k_emergency:
                if ref == -np.inf:
                    newref, alpha = f32(np.ceil(cm)), f32(0.0)
                else:
                    k = f32(np.ceil(f32(cm - ref)))
                    newref, alpha = f32(ref + k), _exp2_neg_int(k)
                P[:c0] = (P[:c0] * alpha).astype(f32)  # a power of two: no second rounding
                l, lsum, ref = f32(l * alpha), f32(lsum * alpha), newref
            refe = f32(0.0) if ref == -np.inf else ref
            p = np.exp2(x - refe).astype(f32)
            lsum = f32(lsum + p.sum(dtype=f32))
            P[c0:c0 + block] = rnd(p.astype(np.float64)).astype(f32)
        l = f32(l + lsum)
        if v0 > 0 and ref != ref_start:
            alpha = f32(0.0) if ref_start == -np.inf else _exp2_neg_int(ref - ref_start)
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
    """The rising row moves the reference in most blocks, so the rescale path is what the
    comparison above checks."""
    t = np.linspace(-30.0, 300.0, 1000)
    moves, ref = 0, -np.inf
    for c0 in range(0, 1000, 32):
        cm = t[c0:c0 + 32].max()
        if cm > ref + 64:
            moves, ref = moves + 1, (np.ceil(cm) if ref == -np.inf else ref + np.ceil(cm - ref))
    assert moves >= 4


@pytest.mark.parametrize("kind", ["rising", "staircase"])
def test_rescaled_probabilities_keep_one_rounding(kind):
    """After every rescale inside a tile, each bf16 P value is within one rounding (2^-8
    relative: half the spacing of 7 stored fraction bits) of the exact 2^(t - ref) for the
    tile's final reference -- a second rounding could reach about 2^-7.  The staircase puts values just under the margin next to values just
    over it, so rescaled values stay large."""
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
