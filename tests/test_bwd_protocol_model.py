"""A model of the backward score kernel's barrier protocol (swvr_b200/csrc/tc_bwd.cu).

bwd_scores_kernel is four roles that hand buffers to each other through mbarriers: the TMA
producer of each CTA (with ``aux_loads`` a second one, warp 2, loads gO and E), the
MMA-issuing thread of the pair, the tensor pipe (which executes issued MMAs and commits in
order) and the gradient warps of each CTA.  This model restates
each role's loop, waits and arrivals as Python generators (same counters, same parity
expressions, same order as the kernel), runs them under randomised interleavings, and
checks:
  * every wait passes on the phase it means (mbarrier parity semantics: a wait on parity P
    passes when the current phase's parity differs from P), and no arrival lands in a later
    phase than the one it belongs to;
  * no buffer is overwritten while a reader still needs it: the W/h stage ring, the K-major
    and MN-major gO copies, E, both S buffers, the dP buffer and the dE accumulator;
  * no interleaving deadlocks.
Configurations cover single- and double-buffered S, one or three dP chunks per tile, ring
depths 2-4, 1-20 stages per tile and ragged / empty units.  A planted mistake (one wait left
out) must be caught.  The model checks the protocol's design; the kernel itself is checked
against the oracle on the GPU (test_gpu_parity.py).
"""
import random

import pytest

from tests.protocol_model import Bar, Wait, schedule


def run(cfg, seed, skip_dp_free_test=False):
    NS, KB, NCH, single, need_de, units = cfg["NS"], cfg["KB"], cfg["NCH"], cfg["single"], cfg["need_de"], cfg["units"]
    aux = cfg.get("aux", False)
    GOK_NB = 2 if NCH > 1 else 1
    kx = min(NS, KB - 1)
    # barriers: leader-only (issuer waits) and per-CTA copies (multicast commits)
    full = [Bar(f"full{i}", 2) for i in range(NS)]
    empty = [[Bar(f"empty{i}.r{r}", 1) for i in range(NS)] for r in range(2)]
    e_full, e_empty = Bar("e_full", 2), [Bar(f"e_empty.r{r}", 1) for r in range(2)]
    gok_full = [Bar(f"gok_full{i}", 2) for i in range(2)]
    gok_empty = [[Bar(f"gok_empty{i}.r{r}", 1) for i in range(2)] for r in range(2)]
    gom_full, gom_empty = Bar("gom_full", 2), [Bar(f"gom_empty.r{r}", 1) for r in range(2)]
    s_full = [[Bar(f"s_full{i}.r{r}", 1) for i in range(2)] for r in range(2)]
    dp_full = [Bar(f"dp_full.r{r}", 1) for r in range(2)]
    dp_free = Bar("dp_free", 2)
    p_ready = [Bar(f"p_ready{i}", 2) for i in range(2)]
    de_full = [Bar(f"de_full.r{r}", 1) for r in range(2)]
    de_free = Bar("de_free", 2)

    # global tile index -> unit index, first tile of the unit, etc.
    tiles = []  # (unit, j, n)
    for ui, (it0, it1) in enumerate(units):
        for j in range(it1 - it0):
            tiles.append((ui, j, it1 - it0))
    T = len(tiles)
    tile_unit_idx = []
    k = 0
    for ui, (it0, it1) in enumerate(units):
        if it1 > it0:
            tile_unit_idx += [k] * (it1 - it0)
            k += 1
    st = dict(
        pipe=[],  # FIFO of ops
        s_exec={},  # tile -> number of S stages executed
        dp_exec=0,  # dP chunks executed
        de_exec=set(),  # tiles whose dE executed
        grad_done={0: set(), 1: set()},  # tiles whose gradient pass finished per rank
        dp_read={0: -1, 1: -1},  # last dP chunk fully read per rank
        stage_exec=[0] * NS,  # uses of each stage consumed by the pipe
        stage_load=[0] * NS,
        gok_loaded={0: set(), 1: set()},  # tiles whose K-major gO is loaded per rank
        gom_loaded={0: set(), 1: set()},
        e_loaded={0: set(), 1: set()},
        dp_of_tile_exec={},  # tile -> chunks executed
        de_read={0: set(), 1: set()},  # units whose dE was read out per rank
        de_unit_exec={},  # unit -> dE MMAs executed
        q_tile=[],  # chunk q -> tile
    )

    def producer(rank):
        stage = sphase = 0
        g = uc = 0
        prev_it = 0
        prev_g_tile = None
        uses = [0] * NS
        for ui, (it0, it1) in enumerate(units):
            if it1 <= it0:
                continue
            for it in range(it0, it1):
                for kb in range(KB):
                    yield Wait(empty[rank][stage], sphase ^ 1, uses[stage] - 1)
                    assert st["stage_exec"][stage] >= uses[stage], "stage overwrite"
                    full[stage].arrive(uses[stage])
                    uses[stage] += 1
                    stage += 1
                    if stage == NS:
                        stage, sphase = 0, sphase ^ 1
                    if kb == kx and not aux:
                        kbuf = g % GOK_NB
                        f = g // GOK_NB
                        yield Wait(gok_empty[rank][kbuf], (f & 1) ^ 1, f - 1)
                        if g - GOK_NB >= 0:
                            assert st["dp_of_tile_exec"].get(g - GOK_NB, 0) == NCH, ("gok overwrite", g)
                        gok_full[kbuf].arrive(f)
                        st["gok_loaded"][rank].add(g)
                        if single or g > 0:
                            fill = g if single else g - 1
                            yield Wait(gom_empty[rank], (fill & 1) ^ 1, fill - 1)
                            if need_de and fill - 1 >= 0:
                                assert (fill - 1) in st["de_exec"], ("gom overwrite", fill)
                            gom_full.arrive(fill)
                            st["gom_loaded"][rank].add(fill)
                    if not aux and it == it0 and kb == (kx if single else KB - 1):
                        yield Wait(e_empty[rank], (uc & 1) ^ 1, uc - 1)
                        prevs = [u for u in range(ui) if units[u][1] > units[u][0]]
                        if prevs:
                            prev_tiles = [t for t in range(T) if tiles[t][0] == prevs[-1]]
                            assert all(st["dp_of_tile_exec"].get(t, 0) == NCH for t in prev_tiles), "E overwrite"
                        e_full.arrive(uc)
                        st["e_loaded"][rank].add(ui)
                prev_it = it
                g += 1
            uc += 1
        if not aux and not single and g > 0:
            fill = g - 1
            yield Wait(gom_empty[rank], (fill & 1) ^ 1, fill - 1)
            if need_de and fill - 1 >= 0:
                assert (fill - 1) in st["de_exec"], "gom overwrite (tail)"
            gom_full.arrive(fill)
            st["gom_loaded"][rank].add(fill)

    def load_e(rank, ui, uc):
        yield Wait(e_empty[rank], (uc & 1) ^ 1, uc - 1)
        prevs = [u for u in range(ui) if units[u][1] > units[u][0]]
        if prevs:
            prev_tiles = [t for t in range(T) if tiles[t][0] == prevs[-1]]
            assert all(st["dp_of_tile_exec"].get(t, 0) == NCH for t in prev_tiles), "E overwrite"
        e_full.arrive(uc)
        st["e_loaded"][rank].add(ui)

    def load_gok(rank, g):
        kbuf = g % GOK_NB
        f = g // GOK_NB
        yield Wait(gok_empty[rank][kbuf], (f & 1) ^ 1, f - 1)
        if g - GOK_NB >= 0:
            assert st["dp_of_tile_exec"].get(g - GOK_NB, 0) == NCH, ("gok overwrite", g)
        gok_full[kbuf].arrive(f)
        st["gok_loaded"][rank].add(g)

    def load_gom(rank, fill):
        yield Wait(gom_empty[rank], (fill & 1) ^ 1, fill - 1)
        if need_de and fill - 1 >= 0:
            assert (fill - 1) in st["de_exec"], ("gom overwrite", fill)
        gom_full.arrive(fill)
        st["gom_loaded"][rank].add(fill)

    def aux_producer(rank):
        """warp 2 (aux_loads): per tile the unit's E (first tile), the K-major gO, and the
        MN-major gO of the tile whose dE comes next, each once its buffer is free."""
        g = uc = 0
        for ui, (it0, it1) in enumerate(units):
            if it1 <= it0:
                continue
            for it in range(it0, it1):
                if it == it0:
                    yield from load_e(rank, ui, uc)
                yield from load_gok(rank, g)
                if single or g > 0:
                    yield from load_gom(rank, g if single else g - 1)
                g += 1
            uc += 1
        if not single and g > 0:
            yield from load_gom(rank, g - 1)

    def issue(op):
        st["pipe"].append(op)

    def issuer():
        stage = [0]
        sphase = [0]
        g = 0
        uc = 0
        q = 0
        uses = [0] * NS

        def issue_s(gt, b, kb):
            s_ = stage[0]
            issue(("S", gt, b, kb, s_, uses[s_]))
            issue(("commit", [empty[0][s_], empty[1][s_]], uses[s_]))
            uses[s_] += 1
            stage[0] += 1
            if stage[0] == NS:
                stage[0], sphase[0] = 0, sphase[0] ^ 1

        def issue_dp(gt, jj, qq, unit_last):
            kbuf = gt % GOK_NB
            issue(("dP", gt, jj, qq))
            if jj == NCH - 1:
                issue(("commit", [gok_empty[0][kbuf], gok_empty[1][kbuf]], gt // GOK_NB))
                if unit_last:
                    issue(("commit", [e_empty[0], e_empty[1]], tile_unit_idx[gt]))
            issue(("commit", [dp_full[0], dp_full[1]], qq))

        def issue_de(gt, unit_first, unit_last, guc):
            yield Wait(gom_full, gt & 1, gt)
            if need_de:
                if unit_first and guc > 0:
                    yield Wait(de_free, (guc - 1) & 1, guc - 1)
                issue(("dE", gt, unit_first, tiles[gt][0]))
            issue(("commit", [gom_empty[0], gom_empty[1]], gt))
            if need_de and unit_last:
                issue(("commit", [de_full[0], de_full[1]], guc))

        if single:
            for ui, (it0, it1) in enumerate(units):
                n = it1 - it0
                if n <= 0:
                    continue
                for j in range(n):
                    for kb in range(KB):
                        yield Wait(full[stage[0]], sphase[0], uses[stage[0]])
                        issue_s(g, 0, kb)
                    issue(("commit", [s_full[0][0], s_full[1][0]], g))
                    if q > 0:
                        yield Wait(dp_free, (q - 1) & 1, q - 1)
                    if j == 0:
                        yield Wait(e_full, uc & 1, uc)
                    yield Wait(gok_full[0], g & 1, g)
                    issue_dp(g, 0, q, j == n - 1)
                    q += 1
                    yield Wait(p_ready[0], g & 1, g)
                    yield from issue_de(g, j == 0, j == n - 1, uc)
                    g += 1
                uc += 1
            return
        pj = NCH
        prev_first = prev_last = False
        prev_uc = 0
        for ui, (it0, it1) in enumerate(units):
            n = it1 - it0
            if n <= 0:
                continue
            for j in range(n):
                b = g & 1
                for kb in range(KB):
                    yield Wait(full[stage[0]], sphase[0], uses[stage[0]])
                    issue_s(g, b, kb)
                    if NCH > 1 and pj < NCH and (skip_dp_free_test or dp_free.test((q - 1) & 1)):
                        assert skip_dp_free_test or dp_free.done >= q, "dp_free test aliasing"
                        issue_dp(g - 1, pj, q, prev_last)
                        pj += 1
                        q += 1
                issue(("commit", [s_full[0][b], s_full[1][b]], g >> 1))
                while pj < NCH:
                    yield Wait(dp_free, (q - 1) & 1, q - 1)
                    issue_dp(g - 1, pj, q, prev_last)
                    pj += 1
                    q += 1
                have_prev = g > 0
                if have_prev:
                    yield Wait(p_ready[(g - 1) & 1], ((g - 1) >> 1) & 1, (g - 1) >> 1)
                    if prev_last:
                        yield from issue_de(g - 1, prev_first, True, prev_uc)
                if q > 0:
                    yield Wait(dp_free, (q - 1) & 1, q - 1)
                if j == 0:
                    yield Wait(e_full, uc & 1, uc)
                yield Wait(gok_full[g % GOK_NB], (g // GOK_NB) & 1, g // GOK_NB)
                issue_dp(g, 0, q, j == n - 1)
                q += 1
                pj = 1
                if have_prev and not prev_last:
                    yield from issue_de(g - 1, prev_first, False, prev_uc)
                prev_first, prev_last, prev_uc = j == 0, j == n - 1, uc
                g += 1
            uc += 1
        if g > 0:
            while pj < NCH:
                yield Wait(dp_free, (q - 1) & 1, q - 1)
                issue_dp(g - 1, pj, q, prev_last)
                pj += 1
                q += 1
            yield Wait(p_ready[(g - 1) & 1], ((g - 1) >> 1) & 1, (g - 1) >> 1)
            yield from issue_de(g - 1, prev_first, True, prev_uc)

    def pipe_step(op):
        kind = op[0]
        if kind == "commit":
            for bar in op[1]:
                bar.arrive(op[2])
        elif kind == "S":
            _, g, b, kb, stage, use = op
            if kb == 0:
                prev = g - (1 if single else 2)
                if prev >= 0:
                    assert all(prev in st["grad_done"][r] for r in (0, 1)), ("S overwrite before grad", g)
                    if need_de:
                        assert prev in st["de_exec"], ("S overwrite before dE", g)
            st["s_exec"][g] = st["s_exec"].get(g, 0) + 1
            assert st["stage_exec"][stage] == use
            st["stage_exec"][stage] += 1
        elif kind == "dP":
            _, gt, jj, qq = op
            assert st["dp_exec"] == qq
            if qq > 0:
                assert all(st["dp_read"][r] >= qq - 1 for r in (0, 1)), ("dP overwrite", qq)
            assert all(gt in st["gok_loaded"][r] for r in (0, 1)), "gok not loaded"
            ui = tiles[gt][0]
            assert all(ui in st["e_loaded"][r] for r in (0, 1)), "E not loaded"
            assert st["s_exec"].get(gt, 0) == KB, "dP before S"  # order only (not a hazard)
            st["dp_exec"] += 1
            st["dp_of_tile_exec"][gt] = st["dp_of_tile_exec"].get(gt, 0) + 1
            assert st["dp_of_tile_exec"][gt] == jj + 1
        elif kind == "dE":
            _, gg, first, ui = op
            assert all(gg in st["grad_done"][r] for r in (0, 1)), ("dE before P", gg)
            assert all(gg in st["gom_loaded"][r] for r in (0, 1)), ("dE before gom", gg)
            if first and ui > 0:
                # previous unit's dE read out by both CTAs (units in order; skip empty ones)
                prevs = [u for u in range(ui) if units[u][1] > units[u][0]]
                if prevs:
                    assert all(prevs[-1] in st["de_read"][r] for r in (0, 1)), ("dE overwrite", ui)
            st["de_exec"].add(gg)
            st["de_unit_exec"][ui] = st["de_unit_exec"].get(ui, 0) + 1

    def grad(rank):
        g = uc = q = 0
        for ui, (it0, it1) in enumerate(units):
            if it1 <= it0:
                continue
            for it in range(it0, it1):
                b = 0 if single else (g & 1)
                s_m = g if single else (g >> 1)
                yield Wait(s_full[rank][b], s_m & 1, s_m)
                assert st["s_exec"].get(g, 0) == KB
                for jj in range(NCH):
                    yield Wait(dp_full[rank], q & 1, q)
                    assert st["dp_exec"] == q + 1, ("dP read mismatch", q, st["dp_exec"])
                    # S of this tile not yet overwritten
                    nxt = g + (1 if single else 2)
                    assert st["s_exec"].get(nxt, 0) == 0, "S overwritten while read"
                    st["dp_read"][rank] = q
                    last = jj == NCH - 1
                    if last:
                        st["grad_done"][rank].add(g)
                    dp_free.arrive(q)
                    if last:
                        p_ready[b].arrive(g >> 1 if not single else g)
                    q += 1
                    yield None  # let others run between chunks
                g += 1
            if need_de:
                yield Wait(de_full[rank], uc & 1, uc)
                n = it1 - it0
                assert st["de_unit_exec"].get(ui, 0) == n, ("dE read early", ui)
                st["de_read"][rank].add(ui)
                de_free.arrive(uc)
            uc += 1

    roles = {"p0": producer(0), "p1": producer(1), "mma": issuer(), "g0": grad(0), "g1": grad(1)}
    if aux:
        roles.update(a0=aux_producer(0), a1=aux_producer(1))
    schedule(roles, st["pipe"], pipe_step, seed)


def _configs(n, seed=1):
    rnd = random.Random(seed)
    out = []
    for _ in range(n):
        nch, single = rnd.choice([(1, False), (3, False), (1, True), (3, False)])
        units, t = [], 0
        for _ in range(rnd.choice([1, 2, 3, 5])):
            k = rnd.choice([0, 1, 1, 2, 3, 7])
            units.append((t, t + k))
            t += k
        if all(b <= a for a, b in units):
            units.append((t, t + 1))
        out.append(dict(NS=rnd.choice([2, 3, 4]), KB=rnd.choice([1, 2, 3, 4, 7, 20]), NCH=nch, single=single,
                        need_de=rnd.random() < 0.8, units=units, aux=rnd.random() < 0.6))
    return out


_CONFIGS = _configs(300)


@pytest.mark.parametrize("idx", range(len(_CONFIGS)))
def test_protocol_holds_under_random_interleavings(idx):
    cfg = _CONFIGS[idx]
    for s in range(3):
        run(cfg, seed=idx * 10 + s)


@pytest.mark.parametrize("aux", [False, True])
def test_a_missing_wait_is_caught(aux):
    """A planted mistake: the MMA thread issues a tile's later dP chunks between S stages
    without testing that both CTAs' gradient passes have read the previous chunk.  The model
    must flag it (the dP buffer overwritten while read, or a barrier arrival in the wrong
    phase) in some interleaving."""
    cfg = dict(NS=3, KB=6, NCH=3, single=False, need_de=True, units=[(0, 4), (4, 8)], aux=aux)
    caught = 0
    for s in range(40):
        try:
            run(cfg, seed=s, skip_dp_free_test=True)
        except AssertionError:
            caught += 1
    assert caught > 0
