"""DDP x vocabulary-parallel on GPUs: a 2 x 2 grid of NCCL ranks (the reference's
tests/ddp_smoke.py composed with vocabulary sharding).

Rank r is data replica r // 2 and vocabulary shard r % 2.  DDP averages the trunk and the
shard parameters over the data-parallel group; the readout (``vocab_parallel``) exchanges
softmax states and dh over the shard group.  Every rank's gradients must match a
single-GPU run of the unsharded model on the full batch (bf16 readout, 2e-2 norm-wise).
Needs 4 GPUs; the same composition runs on CPU gloo ranks in test_gloo_vocab_parallel.py.
"""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from torch import nn

pytestmark = pytest.mark.gpu

N, K, V, D = 512, 256, 20000, 64


def _inputs():
    g = torch.Generator().manual_seed(4)
    r = lambda *s, scale=1.0: scale * torch.randn(*s, generator=g)
    return dict(x=r(2 * N, K), t=r(2 * N, D, scale=0.02), tw=r(K, K, scale=K ** -0.5), tb=r(K, scale=0.1),
                W=r(V, K, scale=K ** -0.5), E=r(V, D, scale=0.02), b=r(V, scale=0.02))


class _Trunk(nn.Module):
    def __init__(self, z, dev):
        super().__init__()
        self.lin = nn.Linear(K, K).to(dev)
        with torch.no_grad():
            self.lin.weight.copy_(z["tw"])
            self.lin.bias.copy_(z["tb"])


class _ShardModel(nn.Module):
    def __init__(self, z, v0, v1, dev, tp_group):
        super().__init__()
        self.trunk = _Trunk(z, dev)
        self.W = nn.Parameter(z["W"][v0:v1].to(dev, torch.bfloat16))
        self.E = nn.Parameter(z["E"][v0:v1].to(dev, torch.bfloat16))
        self.b = nn.Parameter(z["b"][v0:v1].to(dev, torch.bfloat16))
        self.tp_group = tp_group

    def forward(self, x, t):
        from swvr_b200 import vocab_parallel as vp
        h = torch.tanh(self.trunk.lin(x)).to(torch.bfloat16)
        return vp.softmax_readout_mse_vocab_parallel(h, self.W, self.E, t, self.b, z_loss_weight=1e-3,
                                                     chunk_size=4096, group=self.tp_group)


def _worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    from swvr_b200 import vocab_parallel as vp
    import swvr_b200 as swvr
    tp_groups = [dist.new_group([0, 1]), dist.new_group([2, 3])]
    dp_groups = [dist.new_group([0, 2]), dist.new_group([1, 3])]
    dpi, tpi = rank // 2, rank % 2
    z = _inputs()
    v0, v1 = vp.shard_range(V, 2, tpi)
    model = _ShardModel(z, v0, v1, dev, tp_groups[dpi])
    ddp = nn.parallel.DistributedDataParallel(model, device_ids=[dev.index], process_group=dp_groups[tpi])
    x, t = z["x"].to(dev), z["t"].to(dev)
    rows = slice(dpi * N, (dpi + 1) * N)
    ddp(x[rows], t[rows]).backward()
    # the unsharded model on the full batch, on this GPU
    ref = _ShardModel(z, 0, V, dev, None)
    h = torch.tanh(ref.trunk.lin(x)).to(torch.bfloat16)
    swvr.softmax_readout_mse(h, ref.W, ref.E, t, ref.b, z_loss_weight=1e-3, chunk_size=4096).backward()
    rel = lambda a, r: ((a.float() - r.float()).norm() / r.float().norm().clamp_min(1e-30)).item()
    m = ddp.module
    errs = {"trunk.w": rel(m.trunk.lin.weight.grad, ref.trunk.lin.weight.grad),
            "trunk.b": rel(m.trunk.lin.bias.grad, ref.trunk.lin.bias.grad),
            "W": rel(m.W.grad, ref.W.grad[v0:v1]), "E": rel(m.E.grad, ref.E.grad[v0:v1]),
            "b": rel(m.b.grad, ref.b.grad[v0:v1])}
    with open(os.path.join(out_dir, f"rank{rank}.txt"), "w") as f:
        f.write(repr(errs))
    dist.barrier()
    dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 4, reason="needs 4 GPUs")
def test_ddp_over_vocab_parallel_on_four_gpus(tmp_path):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 4, port, str(tmp_path))) for r in range(4)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=400)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for r in range(4):
        errs = eval((tmp_path / f"rank{r}.txt").read_text())
        for k, e in errs.items():
            assert e < 2e-2, (r, k, e)
