"""A model of the staggered score kernel's barrier protocol (swvr_b200/csrc/tc_bwd_stagger.cu).

bwd_scores_stagger_kernel runs 128-token tiles whose K loops are offset by half a loop, so two
tiles of a unit are in flight at every stage and share its W K-block: tile i of a unit owns
stages [i*H, i*H + KB) (H = ceil(KB / 2)) and reads K-block (stage mod KB) there.  Its S^T
accumulator lives in one of three tensor-memory regions (global tile g in region g mod 3);
when a tile's last stage is done its two 64-token dP^T chunks, gradient pass and dE follow
while the next tiles stream.  The roles -- W / h producer and gO / E producer of each CTA, the
MMA-issuing thread, the in-order tensor pipe and the gradient warps of each CTA -- are
restated here as Python generators with the kernel's counters, parity expressions and order,
run under randomised interleavings, and checked:
  * every wait passes on the phase it means, and no arrival lands in a later phase;
  * no buffer is overwritten while a reader still needs it: the W / h stage ring (and which
    tiles' h it holds), the S regions, the dP buffer, the K- and MN-major gO copies, E and the
    dE accumulator;
  * the MMA thread issues the deferred dP chunks and dE products (tested without blocking
    between stages, forced before a region is reused) without deadlock.
Configurations cover 1-20 K-blocks per tile (odd and even), ring depths 2-4 and ragged /
empty units.  A planted mistake (the dP-free test skipped) must be caught.
"""
import random

import pytest

from tests.protocol_model import Bar, Wait, schedule

NCH = 2  # 64-token dP^T chunks per 128-token tile


def active(s, n, H, KB):
    """Unit-local tiles in flight at unit stage s (older first)."""
    return [i for i in (s // H - 1, s // H) if 0 <= i < n and i * H <= s < i * H + KB]


def run(cfg, seed, skip_dp_free_test=False):
    NS, KB, need_de, units = cfg["NS"], cfg["KB"], cfg["need_de"], cfg["units"]
    H = (KB + 1) // 2
    full = [Bar(f"full{i}", 2) for i in range(NS)]
    empty = [[Bar(f"empty{i}.r{r}", 1) for i in range(NS)] for r in range(2)]
    s_full = [[Bar(f"s_full{i}.r{r}", 1) for i in range(3)] for r in range(2)]
    p_ready = [Bar(f"p_ready{i}", 2) for i in range(3)]
    dp_full = [Bar(f"dp_full.r{r}", 1) for r in range(2)]
    dp_free = Bar("dp_free", 2)
    e_full, e_empty = Bar("e_full", 2), [Bar(f"e_empty.r{r}", 1) for r in range(2)]
    gok_full, gok_empty = Bar("gok_full", 2), [Bar(f"gok_empty.r{r}", 1) for r in range(2)]
    gom_full, gom_empty = Bar("gom_full", 2), [Bar(f"gom_empty.r{r}", 1) for r in range(2)]
    de_full, de_free = [Bar(f"de_full.r{r}", 1) for r in range(2)], Bar("de_free", 2)

    live = [(ui, it1 - it0) for ui, (it0, it1) in enumerate(units) if it1 > it0]
    tile_unit, tile_first, tile_last = [], [], []
    for k, (ui, n) in enumerate(live):
        for i in range(n):
            tile_unit.append(k)
            tile_first.append(i == 0)
            tile_last.append(i == n - 1)
    T = len(tile_unit)
    st = dict(pipe=[], s_exec={}, stage_exec=[0] * NS, stage_content={0: [None] * NS, 1: [None] * NS}, dp_exec=0,
              dp_of_tile={},
              dp_read={0: -1, 1: -1}, grad_done={0: set(), 1: set()}, de_exec=set(), de_unit={},
              de_read={0: set(), 1: set()}, gok={0: set(), 1: set()}, gom={0: set(), 1: set()},
              e={0: set(), 1: set()})

    def producer(rank):
        stage, uses, g0 = 0, [0] * NS, 0
        for k, (ui, n) in enumerate(live):
            for s in range((n - 1) * H + KB):
                use = uses[stage]
                yield Wait(empty[rank][stage], (use & 1) ^ 1, use - 1)
                assert st["stage_exec"][stage] >= use, "stage overwrite"
                st["stage_content"][rank][stage] = (k, s % KB, tuple(g0 + i for i in active(s, n, H, KB)))
                full[stage].arrive(use)
                uses[stage] += 1
                stage = (stage + 1) % NS
            g0 += n

    def aux(rank):
        g, uc = 0, 0
        for k, (ui, n) in enumerate(live):
            for i in range(n):
                if i == 0:
                    yield Wait(e_empty[rank], (uc & 1) ^ 1, uc - 1)
                    if uc > 0:
                        prev = [t for t in range(T) if tile_unit[t] == k - 1]
                        assert all(st["dp_of_tile"].get(t, 0) == NCH for t in prev), "E overwrite"
                    e_full.arrive(uc)
                    st["e"][rank].add(k)
                yield Wait(gok_empty[rank], (g & 1) ^ 1, g - 1)
                if g > 0:
                    assert st["dp_of_tile"].get(g - 1, 0) == NCH, ("gok overwrite", g)
                gok_full.arrive(g)
                st["gok"][rank].add(g)
                yield Wait(gom_empty[rank], (g & 1) ^ 1, g - 1)
                if g > 0 and need_de:
                    assert (g - 1) in st["de_exec"], ("gom overwrite", g)
                gom_full.arrive(g)
                st["gom"][rank].add(g)
                g += 1
            uc += 1

    def issue(op):
        st["pipe"].append(op)

    def issuer():
        stage, uses = 0, [0] * NS
        q = [0]
        pend_dp, pend_de = [], []  # (tile, chunk), tile

        def try_dp(block):
            """Issue the oldest deferred dP chunk; False if a test failed (non-blocking mode)."""
            gt, jj = pend_dp[0]
            if q[0] > 0:
                if block:
                    yield Wait(dp_free, (q[0] - 1) & 1, q[0] - 1)
                elif not (skip_dp_free_test or dp_free.test((q[0] - 1) & 1)):
                    return False
            if jj == 0:
                k = tile_unit[gt]
                for bar, m in ((e_full, k), (gok_full, gt)):
                    if block:
                        yield Wait(bar, m & 1, m)
                    elif not bar.test(m & 1):
                        return False
            pend_dp.pop(0)
            issue(("dP", gt, jj, q[0]))
            if jj == NCH - 1:
                issue(("commit", gok_empty, gt))
                if tile_last[gt]:
                    issue(("commit", e_empty, tile_unit[gt]))
            issue(("commit", dp_full, q[0]))
            q[0] += 1
            return True

        def try_de(block):
            gt = pend_de[0]
            k = tile_unit[gt]
            waits = [(p_ready[gt % 3], gt // 3), (gom_full, gt)]
            if need_de and tile_first[gt] and k > 0:
                waits.append((de_free, k - 1))
            for bar, m in waits:
                if block:
                    yield Wait(bar, m & 1, m)
                elif not bar.test(m & 1):
                    return False
            pend_de.pop(0)
            if need_de:
                issue(("dE", gt, tile_first[gt], k))
            issue(("commit", gom_empty, gt))
            if need_de and tile_last[gt]:
                issue(("commit", de_full, k))
            return True

        def side_work():
            while pend_dp:
                ok = yield from try_dp(False)
                if not ok:
                    break
            while pend_de and not (pend_dp and pend_dp[0][0] <= pend_de[0]):
                ok = yield from try_de(False)
                if not ok:
                    break

        def flush_through(gt):
            """Blocking: every deferred dP chunk and dE product of tiles up to gt, tile by tile
            (a tile's dE before the next tile's dP: the gO / E producer loads the next tile's
            K-major gO and E only after this tile's MN-major gO, whose buffer dE frees)."""
            while True:
                heads = ([pend_dp[0][0]] if pend_dp else []) + ([pend_de[0]] if pend_de else [])
                t = min(heads, default=None)
                if t is None or t > gt:
                    return
                while pend_dp and pend_dp[0][0] == t:
                    yield from try_dp(True)
                if pend_de and pend_de[0] == t:
                    yield from try_de(True)

        g0 = 0
        for k, (ui, n) in enumerate(live):
            for s in range((n - 1) * H + KB):
                act = active(s, n, H, KB)
                for i in act:
                    if s == i * H and g0 + i >= 3:
                        yield from flush_through(g0 + i - 3)  # the region's previous tile is finished
                use = uses[stage]
                yield Wait(full[stage], use & 1, use)
                for i in act:
                    issue(("S", g0 + i, k, s % KB, stage, use, s == i * H))
                issue(("commit", empty, use, stage))
                for i in act:
                    if s == i * H + KB - 1:
                        g = g0 + i
                        issue(("commit", s_full, g // 3, g % 3))
                        pend_dp.extend([(g, 0), (g, 1)])
                        pend_de.append(g)
                uses[stage] += 1
                stage = (stage + 1) % NS
                yield from side_work()
                yield None
            g0 += n
        yield from flush_through(T - 1)

    def pipe_step(op):
        kind = op[0]
        if kind == "commit":
            bars, phase = op[1], op[2]
            if bars is empty:
                for r in range(2):
                    empty[r][op[3]].arrive(phase)
            elif bars is s_full:
                for r in range(2):
                    s_full[r][op[3]].arrive(phase)
            elif isinstance(bars, list):
                for b in bars:
                    b.arrive(phase)
            else:
                bars.arrive(phase)
        elif kind == "S":
            _, g, k, kw, stage, use, first = op
            assert st["stage_exec"][stage] == use
            for r in (0, 1):
                content = st["stage_content"][r][stage]
                assert content[0] == k and content[1] == kw and g in content[2], ("stage holds other data", g, content)
            if first:
                assert st["s_exec"].get(g, 0) == 0
                if g >= 3:
                    assert all(g - 3 in st["grad_done"][r] for r in (0, 1)), ("S region reused before grad", g)
                    if need_de:
                        assert g - 3 in st["de_exec"], ("S region reused before dE", g)
            st["s_exec"][g] = st["s_exec"].get(g, 0) + 1
        elif kind == "dP":
            _, gt, jj, qq = op
            assert st["dp_exec"] == qq
            assert st["s_exec"].get(gt, 0) == KB, "dP before S"
            if qq > 0:
                assert all(st["dp_read"][r] >= qq - 1 for r in (0, 1)), ("dP overwrite", qq)
            assert all(gt in st["gok"][r] for r in (0, 1)), "gok not loaded"
            assert all(tile_unit[gt] in st["e"][r] for r in (0, 1)), "E not loaded"
            st["dp_exec"] += 1
            st["dp_of_tile"][gt] = st["dp_of_tile"].get(gt, 0) + 1
            assert st["dp_of_tile"][gt] == jj + 1
        elif kind == "dE":
            _, gt, first, k = op
            assert all(gt in st["grad_done"][r] for r in (0, 1)), ("dE before P", gt)
            assert all(gt in st["gom"][r] for r in (0, 1)), ("dE before gom", gt)
            if first and k > 0:
                assert all(k - 1 in st["de_read"][r] for r in (0, 1)), ("dE overwrite", k)
            st["de_exec"].add(gt)
            st["de_unit"][k] = st["de_unit"].get(k, 0) + 1

        # the stage ring: the pipe consumed a stage when its commit executed
        if kind == "commit" and op[1] is empty:
            st["stage_exec"][op[3]] += 1

    def grad(rank):
        g = q = 0
        for k, (ui, n) in enumerate(live):
            for i in range(n):
                yield Wait(s_full[rank][g % 3], (g // 3) & 1, g // 3)
                assert st["s_exec"].get(g, 0) == KB
                for jj in range(NCH):
                    yield Wait(dp_full[rank], q & 1, q)
                    assert st["dp_exec"] == q + 1, ("dP read mismatch", q, st["dp_exec"])
                    assert st["s_exec"].get(g + 3, 0) == 0, "S region overwritten while read"
                    st["dp_read"][rank] = q
                    if jj == NCH - 1:
                        st["grad_done"][rank].add(g)
                    dp_free.arrive(q)
                    if jj == NCH - 1:
                        p_ready[g % 3].arrive(g // 3)
                    q += 1
                    yield None
                g += 1
            if need_de:
                yield Wait(de_full[rank], k & 1, k)
                assert st["de_unit"].get(k, 0) == n, ("dE read early", k)
                st["de_read"][rank].add(k)
                de_free.arrive(k)

    roles = {"p0": producer(0), "p1": producer(1), "a0": aux(0), "a1": aux(1), "mma": issuer(),
             "g0": grad(0), "g1": grad(1)}
    schedule(roles, st["pipe"], pipe_step, seed)
    assert st["dp_exec"] == NCH * T
    assert len(st["de_exec"]) == (T if need_de else 0)


def _configs(n, seed=2):
    rnd = random.Random(seed)
    out = []
    for _ in range(n):
        units, t = [], 0
        for _ in range(rnd.choice([1, 2, 3, 5])):
            k = rnd.choice([0, 1, 1, 2, 3, 5, 8])
            units.append((t, t + k))
            t += k
        if all(b <= a for a, b in units):
            units.append((t, t + 1))
        out.append(dict(NS=rnd.choice([2, 3, 4]), KB=rnd.choice([1, 2, 3, 4, 5, 7, 20]), need_de=rnd.random() < 0.8,
                        units=units))
    return out


_CONFIGS = _configs(300)


@pytest.mark.parametrize("idx", range(len(_CONFIGS)))
def test_protocol_holds_under_random_interleavings(idx):
    cfg = _CONFIGS[idx]
    for s in range(3):
        run(cfg, seed=idx * 10 + s)


def test_two_tiles_share_every_middle_stage():
    """The stagger: with KB even, all but the first and last H stages of a unit carry two tiles."""
    KB, n = 20, 8
    H = KB // 2
    counts = [len(active(s, n, H, KB)) for s in range((n - 1) * H + KB)]
    assert counts[:H] == [1] * H and counts[-H:] == [1] * H
    assert all(c == 2 for c in counts[H:-H])
    # every tile reads every K-block exactly once
    for i in range(n):
        assert sorted(s % KB for s in range(i * H, i * H + KB)) == list(range(KB))


def test_a_missing_wait_is_caught():
    """A planted mistake: the MMA thread issues deferred dP chunks without testing that both
    CTAs' gradient passes have read the previous chunk.  Some interleaving must flag it."""
    cfg = dict(NS=3, KB=6, need_de=True, units=[(0, 4), (4, 8)])
    caught = 0
    for s in range(60):
        try:
            run(cfg, seed=s, skip_dp_free_test=True)
        except AssertionError:
            caught += 1
    assert caught > 0
