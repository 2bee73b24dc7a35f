"""A model of the backward GEMM kernel's protocol (swvr_b200/csrc/tc_gemm.cu, gemm_kernel).

Roles, restated from the kernel with its counters and parity expressions: the TMA producer
of each CTA (A / B stage ring), the MMA-issuing thread of the pair (each pair tile into TMEM
accumulator tc & 1, after the epilogues of tile tc - 2 released it), the in-order tensor
pipe, the epilogue warps of each CTA (accumulator slabs staged through two shared-memory
slabs and written by TMA stores / add-reductions, the slab reused only after
`cp.async.bulk.wait_group.read 1`), and each CTA's bulk-copy engine, which finishes the
oldest store group at random times.  Checked: the parity of every mbarrier wait
(tests/protocol_model.py); no stage, accumulator or staging slab is overwritten while still
needed; every store group has finished before the kernel ends.  A planted mistake (the slab
wait left out) must be caught.
"""
import random

import pytest

from tests.protocol_model import Bar, Until, Wait, schedule


def run(cfg, seed, skip_slab_wait=False):
    NS, tiles = cfg["NS"], cfg["tiles"]  # tiles: (k-blocks, slabs) of this pair's tiles, in order
    full = [Bar(f"full{i}", 2) for i in range(NS)]
    empty = [[Bar(f"empty{i}.r{r}", 1) for i in range(NS)] for r in range(2)]
    acc_full = [[Bar(f"acc_full{i}.r{r}", 1) for i in range(2)] for r in range(2)]
    acc_empty = [Bar(f"acc_empty{i}", 2) for i in range(2)]
    st = dict(pipe=[], stage_exec=[0] * NS, mma_exec={}, acc_read={0: set(), 1: set()},
              pending={0: [], 1: []}, epi_done={0: False, 1: False})

    def producer(rank):
        stage = sphase = 0
        uses = [0] * NS
        for kblocks, _ in tiles:
            for _ in range(kblocks):
                yield Wait(empty[rank][stage], sphase ^ 1, uses[stage] - 1)
                assert st["stage_exec"][stage] >= uses[stage], "stage overwrite"
                full[stage].arrive(uses[stage])
                uses[stage] += 1
                stage += 1
                if stage == NS:
                    stage, sphase = 0, sphase ^ 1

    def issuer():
        stage = sphase = 0
        uses = [0] * NS
        for tc, (kblocks, _) in enumerate(tiles):
            ab = tc & 1
            yield Wait(acc_empty[ab], ((tc >> 1) & 1) ^ 1, (tc >> 1) - 1)
            for kb in range(kblocks):
                yield Wait(full[stage], sphase, uses[stage])
                st["pipe"].append(("MMA", tc, kb, stage, uses[stage]))
                st["pipe"].append(("commit", [empty[0][stage], empty[1][stage]], uses[stage]))
                uses[stage] += 1
                stage += 1
                if stage == NS:
                    stage, sphase = 0, sphase ^ 1
            st["pipe"].append(("commit", [acc_full[0][ab], acc_full[1][ab]], tc >> 1))

    def pipe_step(op):
        if op[0] == "commit":
            for bar in op[1]:
                bar.arrive(op[2])
            return
        _, tc, kb, stage, use = op
        if kb == 0 and tc >= 2:  # accumulator tc & 1 overwritten: tile tc - 2 read out by both CTAs
            assert all(tc - 2 in st["acc_read"][r] for r in (0, 1)), ("accumulator overwrite", tc)
        assert st["stage_exec"][stage] == use
        st["stage_exec"][stage] += 1
        st["mma_exec"][tc] = st["mma_exec"].get(tc, 0) + 1

    def epilogue(rank):
        pend = st["pending"][rank]
        sl = 0
        for tc, (kblocks, nslab) in enumerate(tiles):
            ab = tc & 1
            yield Wait(acc_full[rank][ab], (tc >> 1) & 1, tc >> 1)
            assert st["mma_exec"].get(tc, 0) == kblocks and st["mma_exec"].get(tc + 2, 0) == 0, ("acc read", tc)
            for _ in range(nslab):
                if not skip_slab_wait:  # cp.async.bulk.wait_group.read 1
                    yield Until(lambda: len(pend) <= 1, f"bulk read groups r{rank}")
                buf = sl & 1
                assert buf not in pend, ("staging slab overwritten while a store reads it", sl)
                pend.append(buf)  # stage the slab, issue the store, commit its group
                sl += 1
                yield None
            st["acc_read"][rank].add(tc)
            acc_empty[ab].arrive(tc >> 1)
        yield Until(lambda: not pend, f"all bulk groups r{rank}")  # cp.async.bulk.wait_group 0
        st["epi_done"][rank] = True

    def engine(rank):
        pend = st["pending"][rank]
        while not (st["epi_done"][rank] and not pend):
            if pend:
                pend.pop(0)
            yield None

    roles = {"p0": producer(0), "p1": producer(1), "mma": issuer(), "e0": epilogue(0), "e1": epilogue(1),
             "bulk0": engine(0), "bulk1": engine(1)}
    schedule(roles, st["pipe"], pipe_step, seed)


def _configs(n, seed=3):
    rnd = random.Random(seed)
    return [dict(NS=rnd.choice([2, 3, 4]),
                 tiles=[(rnd.choice([1, 2, 3, 8]), rnd.choice([4, 8])) for _ in range(rnd.choice([1, 2, 3, 6]))])
            for _ in range(n)]


_CONFIGS = _configs(150)


@pytest.mark.parametrize("idx", range(len(_CONFIGS)))
def test_protocol_holds_under_random_interleavings(idx):
    for s in range(3):
        run(_CONFIGS[idx], seed=idx * 10 + s)


def test_a_missing_wait_is_caught():
    """Planted mistake: a staging slab rewritten without waiting for the store that reads it."""
    cfg = dict(NS=3, tiles=[(2, 8), (2, 8), (2, 4)])
    caught = 0
    for s in range(40):
        try:
            run(cfg, seed=s, skip_slab_wait=True)
        except AssertionError:
            caught += 1
    assert caught > 0
