"""DDP composition (the reference's tests/ddp_smoke.py, run as a test).

Two ranks each run half of a batch through a model whose loss is ``SoftmaxReadoutMSE`` (an
``nn.Linear`` head and an ``nn.Embedding`` codebook with fp32 parameters, under bf16
autocast); the DDP-averaged gradients must match a single-process run on the full batch.
With two GPUs the ranks use NCCL on one GPU each; with one GPU both ranks share it over gloo
(our kernels never wait on another rank's kernels, so two processes on one GPU are safe).
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


class _Model(nn.Module):
    def __init__(self, K=256, V=20000, D=16):
        super().__init__()
        import swvr_b200 as swvr
        self.trunk = nn.Linear(K, K)
        self.head = nn.Linear(K, V)
        self.embed = nn.Embedding(V, D)
        self.loss = swvr.SoftmaxReadoutMSE(self.head, self.embed, z_loss_weight=1e-3, chunk_size=4096)

    def forward(self, x, target):
        return self.loss(torch.tanh(self.trunk(x)), target)


def _worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    two_gpus = torch.cuda.device_count() >= world
    dev = torch.device("cuda", rank if two_gpus else 0)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl" if two_gpus else "gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    torch.manual_seed(0)
    model = _Model().to(dev)
    ref = _Model().to(dev)
    ref.load_state_dict(model.state_dict())
    ddp = nn.parallel.DistributedDataParallel(model, device_ids=[dev.index])
    g = torch.Generator(device=dev).manual_seed(1)
    x = torch.randn(world * 512, 256, device=dev, generator=g)
    t = torch.randn(world * 512, 16, device=dev, generator=g)
    shard = slice(rank * 512, (rank + 1) * 512)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        ddp(x[shard], t[shard]).backward()
        ref(x, t).backward()
    worst = 0.0
    for (name, p), q in zip(model.named_parameters(), ref.parameters()):
        err = ((p.grad - q.grad).norm() / q.grad.norm()).item()
        worst = max(worst, err)
    with open(os.path.join(out_dir, f"rank{rank}.txt"), "w") as f:
        f.write(f"{worst}")
    dist.barrier()
    dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_ddp_matches_full_batch(tmp_path):
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
    for r in range(2):
        worst = float((tmp_path / f"rank{r}.txt").read_text())
        assert worst < 2e-2, (r, worst)
