"""A model of the forward kernel's barrier protocol (swvr_b200/csrc/tc_fwd.cu, fwd_kernel).

Roles, restated from the kernel with its counters and parity expressions: the TMA producer of
each CTA (h / W stage ring, E tiles into two buffers), the MMA-issuing thread of the pair
(S of tile g into S buffer g & 1, then O += P . E of the previous tile), the in-order tensor
pipe, and the softmax warps of each CTA (P written back over S, O rescaled when the running
reference max moves, O read out at the end of a unit).  Under randomised interleavings the
model checks the parity of every wait (tests/protocol_model.py) and these hazards: a stage,
an E buffer or an S buffer overwritten while still needed; O rescaled before the previous
tile's P . E completed or read out before the unit's last one; a unit's first P . E
overwriting O before the previous unit's O was read out.  A planted mistake (the rescale's
wait left out) must be caught.  The kernel itself is checked against the oracle on the GPU.
"""
import random

import pytest

from tests.protocol_model import Bar, Wait, schedule


def run(cfg, seed, skip_pe_done_wait=False):
    NS, KB, units = cfg["NS"], cfg["KB"], cfg["units"]
    full = [Bar(f"full{i}", 2) for i in range(NS)]
    empty = [[Bar(f"empty{i}.r{r}", 1) for i in range(NS)] for r in range(2)]
    s_full = [[Bar(f"s_full{i}.r{r}", 1) for i in range(2)] for r in range(2)]
    p_ready = [Bar(f"p_ready{i}", 2) for i in range(2)]
    e_full = [Bar(f"e_full{i}", 2) for i in range(2)]
    e_empty = [[Bar(f"e_empty{i}.r{r}", 1) for i in range(2)] for r in range(2)]
    pe_done = [Bar(f"pe_done.r{r}", 1) for r in range(2)]
    o_free = Bar("o_free", 2)
    tiles = [ui for ui, (a, b) in enumerate(units) for _ in range(b - a)]  # global tile -> unit
    nonempty = [ui for ui, (a, b) in enumerate(units) if b > a]
    st = dict(pipe=[], stage_exec=[0] * NS, s_exec={}, pe_exec=set(), e_loaded={0: set(), 1: set()},
              p_written={0: set(), 1: set()}, o_read={0: set(), 1: set()})

    def producer(rank):
        stage = sphase = 0
        uses = [0] * NS
        g = 0
        for vt0, vt1 in units:
            for _ in range(vt0, vt1):
                for _kb in range(KB):
                    yield Wait(empty[rank][stage], sphase ^ 1, uses[stage] - 1)
                    assert st["stage_exec"][stage] >= uses[stage], "stage overwrite"
                    full[stage].arrive(uses[stage])
                    uses[stage] += 1
                    stage += 1
                    if stage == NS:
                        stage, sphase = 0, sphase ^ 1
                eb, use = g & 1, g >> 1
                yield Wait(e_empty[rank][eb], (use & 1) ^ 1, use - 1)
                assert g < 2 or (g - 2) in st["pe_exec"], ("E overwrite", g)
                e_full[eb].arrive(use)
                st["e_loaded"][rank].add(g)
                g += 1

    def issuer():
        stage = sphase = 0
        uses = [0] * NS
        g = uc = 0
        for ui, (vt0, vt1) in enumerate(units):
            ntiles = vt1 - vt0
            if ntiles <= 0:
                continue
            for j in range(ntiles + 1):
                if j < ntiles:
                    b = g & 1
                    for kb in range(KB):
                        yield Wait(full[stage], sphase, uses[stage])
                        st["pipe"].append(("S", g, kb, stage, uses[stage]))
                        st["pipe"].append(("commit", [empty[0][stage], empty[1][stage]], uses[stage]))
                        uses[stage] += 1
                        stage += 1
                        if stage == NS:
                            stage, sphase = 0, sphase ^ 1
                    st["pipe"].append(("commit", [s_full[0][b], s_full[1][b]], g >> 1))
                    g += 1
                if j > 0:
                    gg = g - 1 - (1 if j < ntiles else 0)
                    bb, use = gg & 1, gg >> 1
                    first = j == 1
                    yield Wait(p_ready[bb], use & 1, use)
                    yield Wait(e_full[bb], use & 1, use)
                    if first and uc > 0:
                        yield Wait(o_free, (uc - 1) & 1, uc - 1)
                    st["pipe"].append(("PE", gg, first, ui))
                    st["pipe"].append(("commit", [pe_done[0], pe_done[1]], gg))
                    st["pipe"].append(("commit", [e_empty[0][bb], e_empty[1][bb]], use))
            uc += 1

    def pipe_step(op):
        if op[0] == "commit":
            for bar in op[1]:
                bar.arrive(op[2])
        elif op[0] == "S":
            _, g, kb, stage, use = op
            if kb == 0 and g >= 2:  # S buffer g & 1: tile g-2's P consumed by its P . E
                assert (g - 2) in st["pe_exec"], ("S overwrite", g)
            assert st["stage_exec"][stage] == use
            st["stage_exec"][stage] += 1
            st["s_exec"][g] = st["s_exec"].get(g, 0) + 1
        else:
            _, gg, first, ui = op
            assert all(gg in st["p_written"][r] for r in (0, 1)), ("P.E before P", gg)
            assert all(gg in st["e_loaded"][r] for r in (0, 1)), ("P.E before E", gg)
            if first:
                prevs = [u for u in nonempty if u < ui]
                if prevs:
                    assert all(prevs[-1] in st["o_read"][r] for r in (0, 1)), ("O overwrite", ui)
            st["pe_exec"].add(gg)

    def softmax(rank):
        g = uc = 0
        for ui, (vt0, vt1) in enumerate(units):
            if vt1 <= vt0:
                continue
            for vt in range(vt0, vt1):
                b = g & 1
                yield Wait(s_full[rank][b], (g >> 1) & 1, g >> 1)
                assert st["s_exec"].get(g, 0) == KB and st["s_exec"].get(g + 2, 0) == 0, ("S read", g)
                if vt > vt0:
                    if not skip_pe_done_wait:
                        yield Wait(pe_done[rank], (g - 1) & 1, g - 1)
                    # O is rescaled in place: the previous tile's P . E must have completed
                    assert (g - 1) in st["pe_exec"], ("O rescaled before the previous P.E", g)
                st["p_written"][rank].add(g)
                p_ready[b].arrive(g >> 1)
                g += 1
                yield None
            yield Wait(pe_done[rank], (g - 1) & 1, g - 1)
            assert all(t in st["pe_exec"] for t in range(g - (vt1 - vt0), g)), ("O read early", ui)
            st["o_read"][rank].add(ui)
            o_free.arrive(uc)
            uc += 1

    roles = {"p0": producer(0), "p1": producer(1), "mma": issuer(), "s0": softmax(0), "s1": softmax(1)}
    schedule(roles, st["pipe"], pipe_step, seed)
    assert sorted(st["pe_exec"]) == list(range(len(tiles)))


def _configs(n, seed=2):
    rnd = random.Random(seed)
    out = []
    for _ in range(n):
        units, t = [], 0
        for _ in range(rnd.choice([1, 2, 3, 5])):
            k = rnd.choice([0, 1, 1, 2, 3, 6])
            units.append((t, t + k))
            t += k
        if all(b <= a for a, b in units):
            units.append((t, t + 1))
        out.append(dict(NS=rnd.choice([2, 3, 4]), KB=rnd.choice([1, 2, 3, 5, 20]), units=units))
    return out


_CONFIGS = _configs(200)


@pytest.mark.parametrize("idx", range(len(_CONFIGS)))
def test_protocol_holds_under_random_interleavings(idx):
    for s in range(3):
        run(_CONFIGS[idx], seed=idx * 10 + s)


def test_a_missing_wait_is_caught():
    """Planted mistake: the softmax warps rescale O without waiting for the previous tile's
    P . E.  Some interleaving must expose it."""
    cfg = dict(NS=3, KB=3, units=[(0, 4), (4, 8)])
    caught = 0
    for s in range(40):
        try:
            run(cfg, seed=s, skip_pe_done_wait=True)
        except AssertionError:
            caught += 1
    assert caught > 0
