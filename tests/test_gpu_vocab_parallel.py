"""Vocabulary-sharded readout on 2 GPUs over NCCL against the single-GPU path.

Two ranks (spawned processes, one GPU each, NCCL with a short process-group timeout) own
halves of W, E and b; their O, LSE, dh (the sum over shards) and shard gradients must match
the single-GPU API on the full vocabulary.  The per-shard kernels are the same as on one GPU
but the merge order differs (the softmax state of the shards is combined in rank order, dh
is summed by a reduce-scatter), so the bound is the bf16 tolerance.  Skipped with fewer than
two GPUs; the host logic of this path is covered on CPU gloo ranks
(test_gloo_vocab_parallel.py).
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

N, K, V, D = 1000, 512, 30011, 64


def _inputs():
    g = torch.Generator().manual_seed(5)
    h = torch.randn(N, K, generator=g).to(torch.bfloat16)
    W = (K ** -0.5 * torch.randn(V, K, generator=g)).to(torch.bfloat16)
    E = (0.02 * torch.randn(V, D, generator=g)).to(torch.bfloat16)
    b = (0.02 * torch.randn(V, generator=g)).to(torch.bfloat16)
    t = 0.02 * torch.randn(N, D, generator=g)
    w = (torch.rand(N, generator=g) < 0.9).float()
    return h, W, E, b, t, w


def _worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    from swvr_b200 import vocab_parallel as vp
    h, W, E, b, t, w = (x.cuda() for x in _inputs())
    v0, v1 = vp.shard_range(V, world, rank)
    hh = h.clone().requires_grad_(True)
    Ws, Es, bs = (x[v0:v1].clone().requires_grad_(True) for x in (W, E, b))
    loss = vp.softmax_readout_mse_vocab_parallel(hh, Ws, Es, t, bs, weight=w, z_loss_weight=1e-4, chunk_size=4096)
    loss.backward()
    O, lse = vp.softmax_readout_vocab_parallel(h, Ws.detach(), Es.detach(), bs.detach(), chunk_size=4096)
    # the same step under activation checkpointing and under torch.compile(fullgraph=True)
    def step(x, Wp, Ep, bp):
        return vp.softmax_readout_mse_vocab_parallel(x, Wp, Ep, t, bp, weight=w, z_loss_weight=1e-4, chunk_size=4096)
    extra = {}
    for mode, fn in (("ckpt", lambda *a: torch.utils.checkpoint.checkpoint(step, *a, use_reentrant=False)),
                     ("comp", torch.compile(step, fullgraph=True))):
        xs = [hh.detach().clone().requires_grad_(True)] + [x.detach().clone().requires_grad_(True) for x in (Ws, Es, bs)]
        fn(*xs).backward()
        extra.update({f"{mode}_{k}": x.grad.float().cpu().numpy() for k, x in zip("hWEb", xs)})
    torch.cuda.synchronize()
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), **extra, loss=loss.item(), O=O.float().cpu().numpy(),
             lse=lse.float().cpu().numpy(), gh=hh.grad.float().cpu().numpy(), gW=Ws.grad.float().cpu().numpy(),
             gE=Es.grad.float().cpu().numpy(), gb=bs.grad.float().cpu().numpy(), v0=v0, v1=v1)
    dist.barrier()
    dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_vocab_parallel_matches_single_gpu(tmp_path):
    import swvr_b200 as swvr
    from tests.helpers import rel_err

    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]

    h, W, E, b, t, w = (x.cuda() for x in _inputs())
    hh, Wf, Ef, bf = (x.clone().requires_grad_(True) for x in (h, W, E, b))
    loss = swvr.softmax_readout_mse(hh, Wf, Ef, t, bf, weight=w, z_loss_weight=1e-4, chunk_size=4096)
    loss.backward()
    O, lse = swvr.softmax_readout(h, W, E, b, chunk_size=4096)
    for r in range(2):
        z = np.load(os.path.join(str(tmp_path), f"rank{r}.npz"))
        v0, v1 = int(z["v0"]), int(z["v1"])
        assert abs(float(z["loss"]) - loss.item()) <= 1e-3 * abs(loss.item())
        assert rel_err(torch.from_numpy(z["O"]), O) < 2e-2
        assert np.max(np.abs(z["lse"] - lse.float().cpu().numpy())) < 1e-2
        assert rel_err(torch.from_numpy(z["gh"]), hh.grad) < 2e-2
        assert rel_err(torch.from_numpy(z["gW"]), Wf.grad[v0:v1]) < 2e-2
        assert rel_err(torch.from_numpy(z["gE"]), Ef.grad[v0:v1]) < 2e-2
        assert rel_err(torch.from_numpy(z["gb"]), bf.grad[v0:v1]) < 2e-2
        for mode in ("ckpt", "comp"):  # checkpointing and torch.compile give the plain step's gradients
            for k in "hWEb":
                assert rel_err(torch.from_numpy(z[f"{mode}_{k}"]), torch.from_numpy(z[f"g{k}"])) < 1e-6, (mode, k)


@pytest.mark.parametrize("G,mode", [(2, "bf16"), (3, "bf16"), (8, "bf16"), (3, "fp32_params"), (2, "wide")])
def test_sharded_compute_on_one_gpu(G, mode):
    """The vocabulary-sharded path's GPU work on one device: every shard's partial forward
    (swvr_fwd_partial) and shard backward (dh partial in fp32, local dW / dE / db, the last
    chunk's dW rows deferred and computed on a bounded set of SMs), merged as the ranks merge
    them -- states stacked in rank order through swvr_combine, dh partials summed -- with only
    the NCCL transport replaced by in-process stacking.  Checked against the single-GPU API on
    the full vocabulary and against the fp64 oracle.  Modes: bf16 shards; fp32 shard
    parameters computed in bf16 (autocast over fp32 parameters: W and E cast one vocabulary
    chunk at a time); D = 300 (wider than the tensor-core kernels take: the exact fp32 engine).
    Runs on one GPU, so it needs no second device; the collectives themselves are covered by
    the gloo CPU tests and the 2-GPU NCCL test above."""
    import swvr_b200 as swvr
    from oracle import swvr_oracle as orc
    from swvr_b200 import vocab_parallel as vp
    from tests.helpers import npy, rel_err

    h, W, E, b, t, w = (x.cuda() for x in _inputs())
    cdt = torch.bfloat16
    if mode == "fp32_params":
        W, E, b = W.float(), E.float(), b.float()
    elif mode == "wide":
        E = (0.02 * torch.randn(V, 300, generator=torch.Generator().manual_seed(6))).to(torch.bfloat16).cuda()
    Dm = E.shape[1]
    spans = [vp.shard_range(V, G, r) for r in range(G)]
    states = [vp.NativeBackend.partial(h, W[a:z], E[a:z], b[a:z], 1.0, 4096, cdt) for a, z in spans]
    O, lse = vp.NativeBackend.combine(*(torch.stack([s[i] for s in states]) for i in range(3)))
    with torch.autocast("cuda", dtype=torch.bfloat16, enabled=mode == "fp32_params"):
        O_ref, lse_ref = swvr.softmax_readout(h, W, E, b, chunk_size=4096)
    assert rel_err(O, O_ref) < 2e-2
    assert float((lse - lse_ref).abs().max()) < 1e-2
    Oo, lo = orc.softmax_readout_reference(npy(h), npy(W), npy(E), npy(b))
    assert rel_err(O, Oo) < 2e-2 and float(np.abs(npy(lse) - lo).max()) < 1e-2

    g = torch.Generator().manual_seed(9)
    gO = (0.02 * torch.randn(N, Dm, generator=g)).cuda()
    glse = (0.01 * torch.randn(N, generator=g)).cuda()
    dh = torch.zeros(N, K, dtype=torch.float32, device="cuda")
    gW, gE, gb = [], [], []
    for a, z in spans:
        d, x, y, c, finish = vp.NativeBackend.backward(gO, glse, h, W[a:z], E[a:z], b[a:z], O, lse, 1.0, 4096, cdt,
                                                       True, True, True, True)
        if finish is not None:
            finish(16)  # the last chunk's dW rows on a bounded set of SMs
        assert d.dtype == torch.float32 and d.shape == (N, K)
        assert x.dtype == W.dtype and y.dtype == E.dtype and c.dtype == b.dtype
        dh += d
        gW.append(x), gE.append(y), gb.append(c)
    gr = orc.readout_grads(npy(h), npy(W), npy(E), npy(b), npy(gO), npy(glse))
    for name, got, ref in zip("hWEb", [dh, torch.cat(gW), torch.cat(gE), torch.cat(gb)], gr):
        assert rel_err(got, ref) < 2e-2, (name, rel_err(got, ref))


@pytest.mark.parametrize("K,max_sms", [(512, 0), (300, 16), (1024, 132)])
def test_split_backward_equals_one_call(K, max_sms):
    """swvr_bwd_split + swvr_bwd_finish (the last vocabulary chunk's dW rows computed later, on a
    bounded set of SMs) give bit for bit the gradients of one swvr_bwd call: the same kernels
    compute the same tiles.  K = 300 takes the zero-padded K path."""
    from swvr_b200.ops import _backward

    N_, V_, D_ = 700, 9000, 64
    h, W, E, b = (x.detach() for x in make_inputs_gpu(N_, K, V_, D_))
    g = torch.Generator().manual_seed(3)
    gO = (0.02 * torch.randn(N_, D_, generator=g)).cuda()
    glse = (0.01 * torch.randn(N_, generator=g)).cuda()
    from swvr_b200 import softmax_readout
    O, lse = softmax_readout(h, W, E, b, chunk_size=2048)
    args = (gO, glse, h, W, E, b, O, lse, 1.0, 2048, torch.bfloat16, True, True, True, True)
    ref = _backward(*args, dh_partial=True)
    dh, gW, gE, gb, finish = _backward(*args, dh_partial=True, split=True)
    assert finish is not None
    finish(max_sms)
    torch.cuda.synchronize()
    for name, a, r in zip(("dh", "gW", "gE", "gb"), (dh, gW, gE, gb), ref):
        assert torch.equal(a, r), name


def make_inputs_gpu(N_, K, V_, D_):
    g = torch.Generator().manual_seed(8)
    h = torch.randn(N_, K, generator=g).to(torch.bfloat16).cuda()
    W = (K ** -0.5 * torch.randn(V_, K, generator=g)).to(torch.bfloat16).cuda()
    E = (0.02 * torch.randn(V_, D_, generator=g)).to(torch.bfloat16).cuda()
    b = (0.02 * torch.randn(V_, generator=g)).to(torch.bfloat16).cuda()
    return h, W, E, b
