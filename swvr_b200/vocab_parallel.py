"""Vocabulary-parallel readout across the GPUs of one node (one process per GPU).

Rank r owns the contiguous rows ``shard_range(V, G, r)`` of W, E and bias; h, target, weight,
O and LSE are replicated.  The reference library has no counterpart (it supports only
user-level DDP); this is the vocabulary sharding of the online softmax:

forward   each rank runs the fused kernel over its shard and keeps the per-row state
          (m2, l, acc) un-normalised (``swvr_fwd_partial``); one all-gather of [G, N, D+2]
          fp32 moves the states, and every rank merges them in rank order
          (``swvr_combine``), so O and LSE are bit-identical on all ranks.
backward  every rank gets the same (dO, dLSE) because the loss is computed on the
          replicated O, LSE; it runs the fused backward over its shard (dW, dE, db are
          local and final) and accumulates its partial dh in fp32; a reduce-scatter (SUM)
          of dh [N, K] fp32 and an all-gather of the slabs cast to h's dtype finish dh.
          The reduce-scatter starts as soon as dh is final: the dW rows of the shard's last
          vocabulary chunk are computed beside it (``swvr_bwd_split`` / ``swvr_bwd_finish``).

The compute backend is pluggable so the collective logic can be exercised on CPU ``gloo``
ranks in tests; the default is libswvr_b200.so and nothing else runs in production.
"""
from __future__ import annotations

import os
from typing import List, Optional, Tuple

import torch
import torch.distributed as dist
from torch import nn

from . import _native as nat
from .api import _check, _compute_dtype
from .ops import _backward, _forward_state, acc_dtype, default_chunk_size, mse_loss_op


def shard_range(V: int, world: int, rank: int):
    """Contiguous, balanced vocabulary rows of ``rank``: ``[rank*V//world, (rank+1)*V//world)``."""
    return rank * V // world, (rank + 1) * V // world


class NativeBackend:
    """The CUDA library: partial forward, combine and shard backward.  The engine choice (tensor
    cores, or the exact SIMT kernels for wide embeddings) and the per-chunk parameter casts of
    autocast over fp32 parameters are the single-GPU path's (``ops``)."""

    @staticmethod
    def partial(h, W, E, bias, scale, chunk, cdt):
        return _forward_state(h, W, E, bias, scale, chunk, cdt)

    @staticmethod
    def combine(m2s, ls, accs):
        G, N = m2s.shape
        D = accs.shape[2]
        dev = m2s.device
        O = torch.empty(N, D, dtype=accs.dtype, device=dev)
        lse = torch.empty(N, dtype=accs.dtype, device=dev)
        if N:
            with torch.cuda.device(dev):
                nat.check(nat.lib().swvr_combine(G, N, D, nat.dtype_code(accs.dtype), m2s.data_ptr(), ls.data_ptr(),
                                                 accs.data_ptr(), O.data_ptr(), lse.data_ptr(), nat.stream_ptr(dev)),
                          "swvr_combine")
        return O, lse

    @staticmethod
    def backward(gO, glse, h, W, E, bias, O, lse, scale, chunk, cdt, need_h, need_W, need_E, need_b):
        """(this shard's dh in the accumulation dtype or None, gW, gE, gb, finish): ``finish`` is
        None or a function ``finish(max_sms)`` computing the last vocabulary chunk's dW rows,
        which may run beside the dh exchange (dh is final before it)."""
        return _backward(gO, glse, h, W, E, bias, O, lse, scale, chunk, cdt, need_h, need_W, need_E, need_b,
                         dh_partial=True, split=True)


_BACKEND = NativeBackend


def set_backend(backend) -> None:
    """Replace the compute backend (tests use a CPU oracle backend on gloo ranks)."""
    global _BACKEND
    _BACKEND = backend if backend is not None else NativeBackend


def _group_name(group) -> str:
    return (group if group is not None else dist.group.WORLD).group_name


def _resolve(group_name: str):
    return dist.distributed_c10d._resolve_process_group(group_name)


def comm_sms() -> int:
    """SMs left free for the dh reduce-scatter while the last dW rows are computed beside it
    (env ``SWVR_VP_COMM_SMS``, default 16; 0 gives the finish kernel every SM)."""
    return max(0, int(os.environ.get("SWVR_VP_COMM_SMS", "16")))


def _sum_dh_over_shards(dh: torch.Tensor, out_dtype: torch.dtype, group, finish=None) -> torch.Tensor:
    """The sum over ranks of the shards' dh partials, in ``out_dtype`` on every rank.

    A reduce-scatter in the accumulation dtype (each rank sums one slab of rows, in a fixed
    order) followed by an all-gather of the slabs already cast to h's dtype: the same fp32
    sum as an all-reduce, with 3/4 of its traffic for a 16-bit h.  ``finish`` (the deferred
    last dW rows, see NativeBackend.backward) runs on the current stream while the
    reduce-scatter runs on the process group's stream."""
    world = dist.get_world_size(group)
    N, K = dh.shape
    rows = -(-N // world)
    if rows * world != N:
        dh = torch.nn.functional.pad(dh, (0, 0, 0, rows * world - N))
    slab = torch.empty(rows, K, dtype=dh.dtype, device=dh.device)
    work = dist.reduce_scatter_tensor(slab, dh.contiguous(), op=dist.ReduceOp.SUM, group=group, async_op=True)
    if finish is not None:
        sms = torch.cuda.get_device_properties(dh.device).multi_processor_count if dh.is_cuda else 0
        finish(max(2, sms - comm_sms()) if comm_sms() else 0)
    work.wait()
    full = torch.empty(rows * world, K, dtype=out_dtype, device=dh.device)
    dist.all_gather_into_tensor(full, slab.to(out_dtype), group=group)
    return full[:N]


# The sharded readout is an opaque custom-op pair like the single-GPU one (ops.py), so
# torch.compile(fullgraph=True) and activation checkpointing treat it the same way.  The process
# group travels as its registered name (a custom op's schema has no ProcessGroup type).  The
# collectives run inside the ops; every rank calls them in the same order, and the ranks must
# agree on which inputs are frozen (a frozen h skips the dh exchange on every rank).

@torch.library.custom_op("swvr_b200::vp_fwd", mutates_args=())
def _vp_fwd_op(h: torch.Tensor, W: torch.Tensor, E: torch.Tensor, bias: Optional[torch.Tensor], logit_scale: float,
               chunk: int, cdt: torch.dtype, group_name: str) -> Tuple[torch.Tensor, torch.Tensor]:
    group = _resolve(group_name)
    world = dist.get_world_size(group)
    m2, l, acc = _BACKEND.partial(h, W, E, bias, logit_scale, chunk, cdt)
    N, D = acc.shape
    packed = torch.cat([m2[:, None], l[:, None], acc], dim=1).contiguous()
    gathered = torch.empty(world * N, D + 2, dtype=packed.dtype, device=packed.device)
    dist.all_gather_into_tensor(gathered, packed, group=group)
    gathered = gathered.view(world, N, D + 2)
    return _BACKEND.combine(gathered[:, :, 0].contiguous(), gathered[:, :, 1].contiguous(),
                            gathered[:, :, 2:].contiguous())


@_vp_fwd_op.register_fake
def _(h, W, E, bias, logit_scale, chunk, cdt, group_name):
    adt = acc_dtype(cdt)
    return h.new_empty(h.shape[0], E.shape[1], dtype=adt), h.new_empty(h.shape[0], dtype=adt)


@torch.library.custom_op("swvr_b200::vp_bwd", mutates_args=())
def _vp_bwd_op(gO: torch.Tensor, glse: torch.Tensor, h: torch.Tensor, W: torch.Tensor, E: torch.Tensor,
               bias: Optional[torch.Tensor], O: torch.Tensor, lse: torch.Tensor, logit_scale: float, chunk: int,
               cdt: torch.dtype, group_name: str, need_h: bool, need_W: bool, need_E: bool,
               need_b: bool) -> List[torch.Tensor]:
    group = _resolve(group_name)
    dh, gW, gE, gb, finish = _BACKEND.backward(gO, glse, h, W, E, bias, O, lse, logit_scale, chunk, cdt, need_h,
                                               need_W, need_E, need_b)
    if need_h:
        gh = _sum_dh_over_shards(dh, h.dtype, group, finish)
    else:
        gh = None
        if finish is not None:
            finish(0)
    return [x if x is not None else h.new_empty(0) for x in (gh, gW, gE, gb)]


@_vp_bwd_op.register_fake
def _(gO, glse, h, W, E, bias, O, lse, logit_scale, chunk, cdt, group_name, need_h, need_W, need_E, need_b):
    out = []
    for wanted, param in ((need_h, h), (need_W, W), (need_E, E), (need_b and bias is not None, bias)):
        out.append(torch.empty_like(param) if wanted else h.new_empty(0))
    return out


def _vp_save(ctx, inputs, output):
    h, W, E, bias, logit_scale, chunk, cdt, group_name = inputs
    ctx.save_for_backward(h, W, E, bias, *output)
    ctx.consts = (logit_scale, chunk, cdt, group_name)


def _vp_backward(ctx, gO, glse):
    h, W, E, bias, O, lse = ctx.saved_tensors
    want = [bool(x) for x in ctx.needs_input_grad[:4]]
    want[3] = want[3] and bias is not None
    gO = torch.zeros_like(O) if gO is None else gO
    glse = torch.zeros_like(lse) if glse is None else glse
    grads = _vp_bwd_op(gO, glse, h, W, E, bias, O, lse, *ctx.consts, *want)
    return tuple(x if w else None for x, w in zip(grads, want)) + (None,) * len(ctx.consts)


_vp_fwd_op.register_autograd(_vp_backward, setup_context=_vp_save)


def softmax_readout_vocab_parallel(h, W_shard, E_shard, bias_shard=None, *, logit_scale=1.0, chunk_size=None,
                                   group=None):
    """``(O, LSE)`` of the full-vocabulary readout from this rank's vocabulary shard.

    ``W_shard``/``E_shard``/``bias_shard`` hold this rank's rows (``shard_range``); ``h`` is
    the same on every rank.  O and LSE come back identical on every rank.
    """
    _check(h, W_shard, E_shard, bias_shard)
    lead = h.shape[:-1]
    h2 = h.reshape(-1, h.shape[-1])
    chunk = int(chunk_size) if chunk_size else default_chunk_size()
    if chunk <= 0:
        raise ValueError(f"chunk_size must be positive, got {chunk}")
    cdt = _compute_dtype(h, W_shard)
    with torch.autocast(h.device.type, enabled=False):
        O, lse = _vp_fwd_op(h2, W_shard, E_shard, bias_shard, float(logit_scale), chunk, cdt, _group_name(group))
    return O.view(*lead, E_shard.shape[1]), lse.view(lead)


def softmax_readout_mse_vocab_parallel(h, W_shard, E_shard, target, bias_shard=None, *, weight=None,
                                       reduction="mean", z_loss_weight=0.0, logit_scale=1.0, chunk_size=None,
                                       group=None):
    """``softmax_readout_mse`` over a vocabulary-sharded head; the loss is the same on every rank."""
    if reduction not in ("none", "sum", "mean"):
        raise ValueError(f"unknown reduction {reduction!r}")
    O, lse = softmax_readout_vocab_parallel(h, W_shard, E_shard, bias_shard, logit_scale=logit_scale,
                                            chunk_size=chunk_size, group=group)
    lead = O.shape[:-1]
    loss = mse_loss_op(O.reshape(-1, O.shape[-1]), lse.reshape(-1), target, weight, z_loss_weight, reduction)
    return loss.view(lead) if reduction == "none" else loss


def replicate_from_host(host: torch.Tensor, device=None, group=None, out: Optional[torch.Tensor] = None):
    """A host tensor that every rank needs (h, target, weight), on this rank's device.

    Each rank copies one slab of ceil(rows / G) rows from host memory (pinned, for an
    asynchronous copy) and the slabs are all-gathered over NVLink, so each rank moves 1/G of
    the tensor across PCIe instead of all of it.  Every rank must pass the same host data.
    ``out`` (optional) is a device buffer of the full shape to gather into.
    """
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    device = torch.device(device) if device is not None else (out.device if out is not None else torch.device("cpu"))
    rows = host.shape[0]
    slab = -(-rows // world)
    r0, r1 = min(rank * slab, rows), min((rank + 1) * slab, rows)
    mine = torch.empty((slab, *host.shape[1:]), dtype=host.dtype, device=device)
    if r1 > r0:
        mine[:r1 - r0].copy_(host[r0:r1], non_blocking=True)
    if r1 - r0 < slab:
        mine[r1 - r0:].zero_()
    full = torch.empty((slab * world, *host.shape[1:]), dtype=host.dtype, device=device)
    dist.all_gather_into_tensor(full, mine, group=group)
    if out is None:
        return full[:rows]
    out.copy_(full[:rows])
    return out


class VocabParallelSoftmaxReadoutMSE(nn.Module):
    """``SoftmaxReadoutMSE`` whose head / embedding rows are sharded over ``group``."""

    def __init__(self, head_shard, embedding_shard, bias_shard=None, *, z_loss_weight=0.0, logit_scale=1.0,
                 reduction="mean", chunk_size=None, group=None):
        super().__init__()
        self.head_shard, self.embedding_shard, self.bias_shard = head_shard, embedding_shard, bias_shard
        self.z_loss_weight, self.logit_scale = z_loss_weight, logit_scale
        self.reduction, self.chunk_size, self.group = reduction, chunk_size, group

    def forward(self, h, target, weight=None):
        return softmax_readout_mse_vocab_parallel(
            h, self.head_shard, self.embedding_shard, target, self.bias_shard, weight=weight,
            reduction=self.reduction, z_loss_weight=self.z_loss_weight, logit_scale=self.logit_scale,
            chunk_size=self.chunk_size, group=self.group)
