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

The compute backend is pluggable so the collective logic can be exercised on CPU ``gloo``
ranks in tests; the default is libswvr_b200.so and nothing else runs in production.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist
from torch import nn

from . import _native as nat
from .api import _check, _compute_dtype
from .ops import (_prepare, _problem, _require_cuda, _workspace, acc_dtype, default_chunk_size, mse_loss_op)


def shard_range(V: int, world: int, rank: int):
    """Contiguous, balanced vocabulary rows of ``rank``: ``[rank*V//world, (rank+1)*V//world)``."""
    return rank * V // world, (rank + 1) * V // world


class NativeBackend:
    """The CUDA library: partial forward, combine and shard backward."""

    @staticmethod
    def partial(h, W, E, bias, scale, chunk, cdt):
        dev = _require_cuda(h, W, E, bias)
        adt = acc_dtype(cdt)
        N, D = h.shape[0], E.shape[1]
        m2 = torch.empty(N, dtype=adt, device=dev)
        l = torch.empty(N, dtype=adt, device=dev)
        acc = torch.empty(N, D, dtype=adt, device=dev)
        if N == 0:
            return m2, l, acc
        if W.shape[0] == 0:
            return m2.fill_(float("-inf")), l.zero_(), acc.zero_()
        hc, Wc, Ec, b = _prepare(h, W, E, bias, cdt)
        p = _problem(hc, Wc, Ec, b, scale, chunk, cdt)
        nbytes = nat.c_size_t(0)
        with torch.cuda.device(dev):
            nat.check(nat.lib().swvr_fwd_workspace_size(p, nat.ctypes.byref(nbytes)), "swvr_fwd_workspace_size")
            ws = _workspace(nbytes.value, dev)
            nat.check(nat.lib().swvr_fwd_partial(p, m2.data_ptr(), l.data_ptr(), acc.data_ptr(), ws.data_ptr(),
                                                 ws.numel(), nat.stream_ptr(dev)), "swvr_fwd_partial")
        return m2, l, acc

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
    def backward(gO, glse, h, W, E, bias, O, lse, scale, chunk, cdt, need_W, need_E, need_b):
        """Returns (dh partial in the accumulation dtype, gW, gE, gb) for this shard."""
        dev = _require_cuda(h, W, E, bias)
        adt = O.dtype
        N, K, V, D = h.shape[0], h.shape[1], W.shape[0], E.shape[1]
        hc, Wc, Ec, b = _prepare(h, W, E, bias, cdt)
        K8 = hc.shape[1]
        dh = torch.zeros(N, K8, dtype=adt, device=dev)
        gW = torch.empty(V, K8, dtype=W.dtype if W.dtype in (cdt, torch.float32) else torch.float32,
                         device=dev) if need_W else None
        gE = torch.empty(E.shape, dtype=E.dtype, device=dev) if need_E else None
        gb = torch.empty(bias.shape, dtype=bias.dtype, device=dev) if (need_b and bias is not None) else None
        if N == 0 or V == 0:
            for x in (gW, gE, gb):
                if x is not None:
                    x.zero_()
        else:
            p = _problem(hc, Wc, Ec, b, scale, chunk, cdt)
            g = nat.Grads()
            gO = gO.to(adt).contiguous()
            glse = glse.to(adt).contiguous()
            g.grad_O, g.grad_lse, g.O, g.lse = gO.data_ptr(), glse.data_ptr(), O.data_ptr(), lse.data_ptr()
            g.grad_h_acc = dh.data_ptr()
            if gW is not None:
                g.grad_W, g.grad_W_dtype, g.ld_grad_W = gW.data_ptr(), nat.dtype_code(gW.dtype), K8
            if gE is not None:
                g.grad_E, g.grad_E_dtype, g.ld_grad_E = gE.data_ptr(), nat.dtype_code(gE.dtype), max(D, 1)
            if gb is not None:
                g.grad_bias, g.grad_bias_dtype = gb.data_ptr(), nat.dtype_code(gb.dtype)
            nbytes = nat.c_size_t(0)
            with torch.cuda.device(dev):
                nat.check(nat.lib().swvr_bwd_workspace_size(p, g, nat.ctypes.byref(nbytes)), "swvr_bwd_workspace_size")
                ws = _workspace(nbytes.value, dev)
                nat.check(nat.lib().swvr_bwd(p, g, ws.data_ptr(), ws.numel(), nat.stream_ptr(dev)), "swvr_bwd")
        dh = dh if K8 == K else dh[:, :K].contiguous()
        if gW is not None:
            gW = gW[:, :K].to(W.dtype)
        return dh, gW, gE, gb


_BACKEND = NativeBackend


def set_backend(backend) -> None:
    """Replace the compute backend (tests use a CPU oracle backend on gloo ranks)."""
    global _BACKEND
    _BACKEND = backend if backend is not None else NativeBackend


def _sum_dh_over_shards(dh: torch.Tensor, out_dtype: torch.dtype, group) -> torch.Tensor:
    """The sum over ranks of the shards' dh partials, in ``out_dtype`` on every rank.

    A reduce-scatter in the accumulation dtype (each rank sums one slab of rows, in a fixed
    order) followed by an all-gather of the slabs already cast to h's dtype: the same fp32
    sum as an all-reduce, with 3/4 of its traffic for a 16-bit h.  Every rank takes both
    collectives exactly once per backward, frozen h or not."""
    world = dist.get_world_size(group)
    N, K = dh.shape
    rows = -(-N // world)
    if rows * world != N:
        dh = torch.nn.functional.pad(dh, (0, 0, 0, rows * world - N))
    slab = torch.empty(rows, K, dtype=dh.dtype, device=dh.device)
    dist.reduce_scatter_tensor(slab, dh.contiguous(), op=dist.ReduceOp.SUM, group=group)
    full = torch.empty(rows * world, K, dtype=out_dtype, device=dh.device)
    dist.all_gather_into_tensor(full, slab.to(out_dtype), group=group)
    return full[:N]


class _VocabParallelReadout(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, W, E, bias, scale, chunk, cdt, group):
        world = dist.get_world_size(group)
        m2, l, acc = _BACKEND.partial(h, W, E, bias, scale, chunk, cdt)
        N, D = acc.shape
        packed = torch.cat([m2[:, None], l[:, None], acc], dim=1).contiguous()
        gathered = torch.empty(world * N, D + 2, dtype=packed.dtype, device=packed.device)
        dist.all_gather_into_tensor(gathered, packed, group=group)
        gathered = gathered.view(world, N, D + 2)
        O, lse = _BACKEND.combine(gathered[:, :, 0].contiguous(), gathered[:, :, 1].contiguous(),
                                  gathered[:, :, 2:].contiguous())
        ctx.save_for_backward(h, W, E, bias, O, lse)
        ctx.args = (scale, chunk, cdt, group)
        return O, lse

    @staticmethod
    def backward(ctx, gO, glse):
        h, W, E, bias, O, lse = ctx.saved_tensors
        scale, chunk, cdt, group = ctx.args
        gO = gO if gO is not None else torch.zeros_like(O)
        glse = glse if glse is not None else torch.zeros_like(lse)
        need_h, need_W, need_E, need_b = ctx.needs_input_grad[:4]
        dh, gW, gE, gb = _BACKEND.backward(gO, glse, h, W, E, bias, O, lse, scale, chunk, cdt, need_W, need_E,
                                           need_b and bias is not None)
        gh = _sum_dh_over_shards(dh, h.dtype, group)
        gh = gh if need_h else None
        return (gh, gW if need_W else None, gE if need_E else None, gb if need_b else None, None, None, None, None)


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
        O, lse = _VocabParallelReadout.apply(h2, W_shard, E_shard, bias_shard, float(logit_scale), chunk, cdt, group)
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
