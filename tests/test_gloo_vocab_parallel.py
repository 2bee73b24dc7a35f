"""Vocabulary-parallel collective logic on CPU gloo ranks (world size 2 and 3).

The per-shard compute is the numpy oracle injected through ``vocab_parallel.set_backend``
(the CUDA kernels need a GPU); everything else -- shard ranges, the all-gather of the
online-softmax states, the rank-ordered merge, the dh all-reduce and the autograd wiring --
is the production code.  Checked against the unsharded oracle.  A second test kills one
rank before the collective and checks that the survivor fails with an error within the
process-group timeout instead of hanging.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import swvr_oracle as orc


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class OracleBackend:
    """numpy oracle standing in for the CUDA kernels on CPU ranks (fp64)."""

    @staticmethod
    def partial(h, W, E, bias, scale, chunk, cdt):
        b = None if bias is None else bias.detach().numpy()
        m2, l, acc = orc.shard_partials(h.detach().numpy(), W.detach().numpy(), E.detach().numpy(), b, scale, 1)
        return torch.from_numpy(m2[0]), torch.from_numpy(l[0]), torch.from_numpy(acc[0])

    @staticmethod
    def combine(m2s, ls, accs):
        O, lse = orc.combine_partials(m2s.numpy(), ls.numpy(), accs.numpy())
        return torch.from_numpy(O), torch.from_numpy(lse)

    @staticmethod
    def backward(gO, glse, h, W, E, bias, O, lse, scale, chunk, cdt, need_h, need_W, need_E, need_b):
        b = None if bias is None else bias.detach().numpy()
        gh, gW, gE, gb = orc.chunked_backward(gO.numpy(), glse.numpy(), h.detach().numpy(), W.detach().numpy(),
                                              E.detach().numpy(), b, O.numpy(), lse.numpy(), scale, chunk, "fp64",
                                              need_h, need_W, need_E, need_b)
        t = lambda x: None if x is None else torch.from_numpy(np.ascontiguousarray(x))
        return t(gh), t(gW), t(gE), t(gb), None


def _inputs(N=7, K=12, V=41, D=5):
    g = torch.Generator().manual_seed(0)
    h, W, E, b = (torch.randn(*s, generator=g, dtype=torch.float64) for s in ((N, K), (V, K), (V, D), (V,)))
    gO = torch.randn(N, D, generator=g, dtype=torch.float64)
    glse = torch.randn(N, generator=g, dtype=torch.float64)
    return h, W, E, b, gO, glse


def _worker(rank, world, port, out_dir, V):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    from swvr_b200 import vocab_parallel as vp
    vp.set_backend(OracleBackend)
    h, W, E, b, gO, glse = _inputs(V=V)
    v0, v1 = vp.shard_range(W.shape[0], world, rank)
    h = h.clone().requires_grad_(True)
    Ws, Es, bs = (x[v0:v1].clone().requires_grad_(True) for x in (W, E, b))
    O, lse = vp.softmax_readout_vocab_parallel(h, Ws, Es, bs, logit_scale=0.5, chunk_size=8)
    ((O * gO).sum() + (lse * glse).sum()).backward()
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), O=O.detach().numpy(), lse=lse.detach().numpy(),
             gh=h.grad.numpy(), gW=Ws.grad.numpy(), gE=Es.grad.numpy(), gb=bs.grad.numpy(), v0=v0, v1=v1)
    dist.destroy_process_group()


@pytest.mark.parametrize("world,V", [(2, 41), (3, 41), (3, 2)])  # V=2 on 3 ranks: rank 0's shard is empty
def test_vocab_parallel_matches_unsharded(tmp_path, world, V):
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path), V), nprocs=world, join=True)
    h, W, E, b, gO, glse = (x.numpy() for x in _inputs(V=V))
    O_ref, lse_ref = orc.softmax_readout_reference(h, W, E, b, 0.5)
    gh, gW, gE, gb = orc.readout_grads(h, W, E, b, gO, glse, 0.5)
    outs = [dict(np.load(tmp_path / f"rank{r}.npz")) for r in range(world)]
    covered = 0
    for r, o in enumerate(outs):
        # O and LSE are identical on every rank (same rank-ordered merge)
        np.testing.assert_array_equal(o["O"], outs[0]["O"])
        np.testing.assert_allclose(o["O"], O_ref, rtol=1e-12, atol=1e-14)
        np.testing.assert_allclose(o["lse"], lse_ref, rtol=1e-12)
        np.testing.assert_allclose(o["gh"], gh, rtol=1e-10, atol=1e-13)
        v0, v1 = int(o["v0"]), int(o["v1"])
        np.testing.assert_allclose(o["gW"], gW[v0:v1], rtol=1e-10, atol=1e-13)
        np.testing.assert_allclose(o["gE"], gE[v0:v1], rtol=1e-10, atol=1e-13)
        np.testing.assert_allclose(o["gb"], gb[v0:v1], rtol=1e-10, atol=1e-13)
        assert v0 == covered
        covered = v1
    assert covered == W.shape[0]


def _failing_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    from swvr_b200 import vocab_parallel as vp
    vp.set_backend(OracleBackend)
    h, W, E, b, _, _ = _inputs()
    if rank == 1:
        # this rank dies between steps, before its collective: no exit handshake
        os._exit(3)
    v0, v1 = vp.shard_range(W.shape[0], world, rank)
    try:
        vp.softmax_readout_vocab_parallel(h, W[v0:v1], E[v0:v1], b[v0:v1])
        status = "completed"
    except Exception as exc:  # the all-gather must fail, not hang
        status = f"raised {type(exc).__name__}"
    with open(os.path.join(out_dir, "rank0.txt"), "w") as f:
        f.write(status)
    os._exit(0)


def test_dead_rank_is_detected_by_timeout(tmp_path):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=90)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung instead of failing"
    assert procs[1].exitcode == 3
    status = (tmp_path / "rank0.txt").read_text()
    assert status.startswith("raised"), status


def _replicate_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    from swvr_b200 import vocab_parallel as vp
    g = torch.Generator().manual_seed(11)
    host_h = torch.randn(7, 5, generator=g, dtype=torch.float64)   # 7 rows: not a multiple of world
    host_w = torch.rand(7, generator=g)
    got_h = vp.replicate_from_host(host_h)
    buf = torch.full((7,), -1.0)
    got_w = vp.replicate_from_host(host_w, out=buf)
    np.savez(os.path.join(out_dir, f"rep{rank}.npz"), h=got_h.numpy(), w=got_w.numpy(), same=got_w is buf,
             ref_h=host_h.numpy(), ref_w=host_w.numpy())
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_replicate_from_host(tmp_path, world):
    """Each rank copies a slab of the host tensor; the all-gather rebuilds it exactly everywhere."""
    mp.spawn(_replicate_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        z = np.load(tmp_path / f"rep{r}.npz")
        np.testing.assert_array_equal(z["h"], z["ref_h"])
        np.testing.assert_array_equal(z["w"], z["ref_w"])
        assert bool(z["same"])


# ---------------------------------------------------------------------- DDP x vocabulary-parallel grid
class _GridModel(torch.nn.Module):
    """A trunk (replicated) feeding a readout whose head / embedding rows are this rank's
    vocabulary shard; the loss (plain torch on O, LSE) is the same on the ranks of a shard group."""

    def __init__(self, trunk_w, trunk_b, Ws, Es, bs, tp_group):
        super().__init__()
        self.trunk = torch.nn.Linear(trunk_w.shape[1], trunk_w.shape[0], dtype=torch.float64)
        with torch.no_grad():
            self.trunk.weight.copy_(trunk_w)
            self.trunk.bias.copy_(trunk_b)
        self.Ws, self.Es, self.bs = (torch.nn.Parameter(x.clone()) for x in (Ws, Es, bs))
        self.tp_group = tp_group

    def forward(self, x, t):
        from swvr_b200 import vocab_parallel as vp
        h = torch.tanh(self.trunk(x))
        O, lse = vp.softmax_readout_vocab_parallel(h, self.Ws, self.Es, self.bs, logit_scale=0.5, chunk_size=8,
                                                   group=self.tp_group)
        return ((O - t) ** 2).mean() + 1e-3 * (lse ** 2).mean()


def _grid_inputs(N=6, K=12, V=41, D=5):
    g = torch.Generator().manual_seed(3)
    r = lambda *s: torch.randn(*s, generator=g, dtype=torch.float64)
    return dict(x=r(2 * N, K), t=r(2 * N, D), tw=0.3 * r(K, K), tb=0.1 * r(K), W=r(V, K), E=r(V, D), b=r(V), N=N)


def _grid_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    from swvr_b200 import vocab_parallel as vp
    vp.set_backend(OracleBackend)
    # 2 x 2 grid: data replica dp = rank // 2, vocabulary shard tp = rank % 2; every rank
    # creates every group, in the same order
    tp_groups = [dist.new_group([0, 1]), dist.new_group([2, 3])]
    dp_groups = [dist.new_group([0, 2]), dist.new_group([1, 3])]
    dp, tp = rank // 2, rank % 2
    z = _grid_inputs()
    v0, v1 = vp.shard_range(z["W"].shape[0], 2, tp)
    model = _GridModel(z["tw"], z["tb"], z["W"][v0:v1], z["E"][v0:v1], z["b"][v0:v1], tp_groups[dp])
    ddp = torch.nn.parallel.DistributedDataParallel(model, process_group=dp_groups[tp])
    rows = slice(dp * z["N"], (dp + 1) * z["N"])
    ddp(z["x"][rows], z["t"][rows]).backward()
    m = ddp.module
    np.savez(os.path.join(out_dir, f"grid{rank}.npz"), tw=m.trunk.weight.grad.numpy(), tb=m.trunk.bias.grad.numpy(),
             gW=m.Ws.grad.numpy(), gE=m.Es.grad.numpy(), gb=m.bs.grad.numpy(), v0=v0, v1=v1)
    dist.destroy_process_group()


def test_ddp_over_vocab_parallel_grid(tmp_path):
    """DDP over the data-parallel group composed with the vocabulary-parallel readout over the
    shard group (2 x 2 ranks): every rank's gradients equal the full-batch, unsharded model's
    (trunk on every rank, head / embedding / bias rows on their shard's ranks)."""
    mp.spawn(_grid_worker, args=(4, _free_port(), str(tmp_path)), nprocs=4, join=True)
    z = _grid_inputs()
    trunk = torch.nn.Linear(z["tw"].shape[1], z["tw"].shape[0], dtype=torch.float64)
    with torch.no_grad():
        trunk.weight.copy_(z["tw"])
        trunk.bias.copy_(z["tb"])
    W, E, b = (z[k].clone().requires_grad_(True) for k in ("W", "E", "b"))
    S = 0.5 * torch.tanh(trunk(z["x"])) @ W.t() + b
    O, lse = torch.softmax(S, dim=1) @ E, torch.logsumexp(S, dim=1)
    (((O - z["t"]) ** 2).mean() + 1e-3 * (lse ** 2).mean()).backward()
    for r in range(4):
        o = np.load(tmp_path / f"grid{r}.npz")
        v0, v1 = int(o["v0"]), int(o["v1"])
        np.testing.assert_allclose(o["tw"], trunk.weight.grad.numpy(), rtol=1e-9, atol=1e-12)
        np.testing.assert_allclose(o["tb"], trunk.bias.grad.numpy(), rtol=1e-9, atol=1e-12)
        np.testing.assert_allclose(o["gW"], W.grad[v0:v1].numpy(), rtol=1e-9, atol=1e-12)
        np.testing.assert_allclose(o["gE"], E.grad[v0:v1].numpy(), rtol=1e-9, atol=1e-12)
        np.testing.assert_allclose(o["gb"], b.grad[v0:v1].numpy(), rtol=1e-9, atol=1e-12)


# ---------------------------------------------------------------------- torch.compile and checkpointing
def _compile_ckpt_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    from swvr_b200 import vocab_parallel as vp
    vp.set_backend(OracleBackend)
    h, W, E, b, gO, glse = _inputs()
    v0, v1 = vp.shard_range(W.shape[0], world, rank)

    def loss_fn(x, Ws, Es, bs):
        O, lse = vp.softmax_readout_vocab_parallel(x, Ws, Es, bs, logit_scale=0.5, chunk_size=8)
        return (O * gO).sum() + (lse * glse).sum()

    def leaves():
        return [h.clone().requires_grad_(True)] + [x[v0:v1].clone().requires_grad_(True) for x in (W, E, b)]

    out = {"v0": v0, "v1": v1}
    # activation checkpointing: the sharded forward (and its all-gather) re-runs in the backward
    xs = leaves()
    torch.utils.checkpoint.checkpoint(loss_fn, *xs, use_reentrant=False).backward()
    out.update({f"ckpt_{k}": x.grad.numpy() for k, x in zip("hWEb", xs)})
    # torch.compile with fullgraph=True: the custom-op pair is opaque, so there is no graph break
    xs = leaves()
    torch.compile(loss_fn, fullgraph=True, backend="aot_eager")(*xs).backward()
    out.update({f"comp_{k}": x.grad.numpy() for k, x in zip("hWEb", xs)})
    np.savez(os.path.join(out_dir, f"cc{rank}.npz"), **out)
    dist.destroy_process_group()


def test_vocab_parallel_under_checkpoint_and_compile(tmp_path):
    """The sharded readout under ``torch.utils.checkpoint`` and under
    ``torch.compile(fullgraph=True)`` gives the unsharded gradients on every rank."""
    world = 2
    mp.spawn(_compile_ckpt_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    h, W, E, b, gO, glse = (x.numpy() for x in _inputs())
    ref = dict(zip("hWEb", orc.readout_grads(h, W, E, b, gO, glse, 0.5)))
    for r in range(world):
        o = np.load(tmp_path / f"cc{r}.npz")
        v0, v1 = int(o["v0"]), int(o["v1"])
        for mode in ("ckpt", "comp"):
            np.testing.assert_allclose(o[f"{mode}_h"], ref["h"], rtol=1e-10, atol=1e-13)
            for k in "WEb":
                np.testing.assert_allclose(o[f"{mode}_{k}"], ref[k][v0:v1], rtol=1e-10, atol=1e-13)
