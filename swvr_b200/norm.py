"""The trunk's final RMSNorm fused into the readout: ``rmsnorm_softmax_readout`` and
``rmsnorm_softmax_readout_mse``.

A model that normalises its trunk output before the readout (``h = RMSNorm(x)``, then
``softmax_readout_mse(h, W, E, ...)``) can hand the library ``x`` and the norm's weight
instead.  The norm then runs as the readout's producer and consumer in libswvr_b200.so:

* forward: one kernel writes ``h = x * rstd * weight`` (fp32 math) once, rounded into the
  readout's compute dtype, which is the dtype the readout's TMA loads read: no separate cast
  or fp32 copy of h;
* backward: the readout's dh is not rounded to h's dtype and cast back; the norm's backward
  reads the library's fp32 dh accumulator directly and returns dx and the weight gradient
  (a fixed-order reduction, deterministic).

The readout in between is the same custom-op code as ``softmax_readout`` (``ops.py``).
Semantics of the norm: ``torch.nn.functional.rms_norm(x, (K,), weight, eps)`` with
``eps=None`` meaning ``torch.finfo(x.dtype).eps`` (as ``nn.RMSNorm``), computed in fp32 and
rounded once.  No counterpart in the reference library, whose callers run the norm
themselves; this is the step on the producer side of its readout (swvr/api.py:69-93 wraps
the head and the codebook, not the norm).
"""
from __future__ import annotations

from typing import List, Optional, Tuple

import torch
from torch import nn

from . import _native as nat
from .api import _check, _compute_dtype
from .ops import _backward, _forward, _no_grad_marker, _require_cuda, acc_dtype, default_chunk_size, mse_loss_op


def _norm_math_dtype(x_dtype: torch.dtype, h_dtype: torch.dtype) -> torch.dtype:
    """The dtype of rstd and of the norm's arithmetic: fp64 when x or h is fp64, else fp32."""
    return torch.float64 if torch.float64 in (x_dtype, h_dtype) else torch.float32


def _rows(x2: torch.Tensor) -> torch.Tensor:
    """``x2`` with unit column stride (the kernels take any row pitch >= K)."""
    return x2 if x2.stride(1) == 1 and x2.stride(0) >= x2.shape[1] else x2.contiguous()


def _rmsnorm_fwd(x2: torch.Tensor, g: Optional[torch.Tensor], eps: float, hdt: torch.dtype):
    dev = _require_cuda(x2, g)
    N, K = x2.shape
    x2 = _rows(x2)
    h = torch.empty(N, K, dtype=hdt, device=dev)
    rstd = torch.empty(N, dtype=_norm_math_dtype(x2.dtype, hdt), device=dev)
    if N:
        with torch.cuda.device(dev):
            nat.check(nat.lib().swvr_rmsnorm_fwd(N, K, x2.data_ptr(), nat.dtype_code(x2.dtype), x2.stride(0),
                                                 nat.ptr(g), nat.dtype_code(g.dtype) if g is not None else 0,
                                                 float(eps), h.data_ptr(), nat.dtype_code(hdt), K, rstd.data_ptr(),
                                                 nat.stream_ptr(dev)), "swvr_rmsnorm_fwd")
    return h, rstd


def _rmsnorm_bwd(dh: torch.Tensor, x2: torch.Tensor, g: Optional[torch.Tensor], rstd: torch.Tensor, need_x: bool,
                 need_g: bool):
    """(dx or None, dg or None) from the readout's un-cast dh (fp32 or fp64, ``[N, K]``)."""
    dev = _require_cuda(dh, x2, g, rstd)
    N, K = x2.shape
    x2 = _rows(x2)
    dh = dh.contiguous()
    rstd = rstd.to(dh.dtype)  # the kernel reads rstd in dh's dtype
    dx = torch.empty(N, K, dtype=x2.dtype, device=dev) if need_x else None
    dg = torch.empty(K, dtype=g.dtype, device=dev) if (need_g and g is not None) else None
    if dx is None and dg is None:
        return None, None
    acc = nat.dtype_code(dh.dtype)
    lib = nat.lib()
    nbytes = nat.c_size_t(0)
    with torch.cuda.device(dev):
        nat.check(lib.swvr_rmsnorm_bwd_workspace_size(N, K, acc, int(dg is not None), nat.ctypes.byref(nbytes)),
                  "swvr_rmsnorm_bwd_workspace_size")
        ws = torch.empty(max(int(nbytes.value), 1), dtype=torch.uint8, device=dev)
        nat.check(lib.swvr_rmsnorm_bwd(N, K, dh.data_ptr(), acc, x2.data_ptr(), nat.dtype_code(x2.dtype), x2.stride(0),
                                       nat.ptr(g), nat.dtype_code(g.dtype) if g is not None else 0, rstd.data_ptr(),
                                       nat.ptr(dx), nat.dtype_code(x2.dtype), nat.ptr(dg),
                                       nat.dtype_code(dg.dtype) if dg is not None else 0, ws.data_ptr(), ws.numel(),
                                       nat.stream_ptr(dev)), "swvr_rmsnorm_bwd")
    return dx, dg


# Custom-op pair, like the readout's own (ops.py): torch.compile sees two opaque nodes and
# activation checkpointing re-runs the forward op.  h and rstd are outputs so that autograd
# keeps them for the backward; they take no gradient.

@torch.library.custom_op("swvr_b200::norm_fwd", mutates_args=())
def _norm_fwd_op(x: torch.Tensor, g: Optional[torch.Tensor], W: torch.Tensor, E: torch.Tensor,
                 bias: Optional[torch.Tensor], eps: float, logit_scale: float, chunk: int,
                 cdt: torch.dtype) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    h, rstd = _rmsnorm_fwd(x, g, eps, cdt)
    O, lse = _forward(h, W, E, bias, logit_scale, chunk, cdt)
    return O, lse, h, rstd


@_norm_fwd_op.register_fake
def _(x, g, W, E, bias, eps, logit_scale, chunk, cdt):
    adt = acc_dtype(cdt)
    N, K = x.shape
    return (x.new_empty(N, E.shape[1], dtype=adt), x.new_empty(N, dtype=adt), x.new_empty(N, K, dtype=cdt),
            x.new_empty(N, dtype=_norm_math_dtype(x.dtype, cdt)))


@torch.library.custom_op("swvr_b200::norm_bwd", mutates_args=())
def _norm_bwd_op(gO: torch.Tensor, glse: torch.Tensor, x: torch.Tensor, g: Optional[torch.Tensor], W: torch.Tensor,
                 E: torch.Tensor, bias: Optional[torch.Tensor], O: torch.Tensor, lse: torch.Tensor, h: torch.Tensor,
                 rstd: torch.Tensor, logit_scale: float, chunk: int, cdt: torch.dtype, need_x: bool, need_g: bool,
                 need_W: bool, need_E: bool, need_b: bool) -> List[torch.Tensor]:
    need_h = need_x or (need_g and g is not None)
    dh, dW, dE, db = _backward(gO, glse, h, W, E, bias, O, lse, logit_scale, chunk, cdt, need_h, need_W, need_E,
                               need_b, dh_partial=True)
    dx = dg = None
    if need_h:
        dx, dg = _rmsnorm_bwd(dh, x, g, rstd, need_x, need_g)
    return [t if t is not None else _no_grad_marker(x) for t in (dx, dg, dW, dE, db)]


@_norm_bwd_op.register_fake
def _(gO, glse, x, g, W, E, bias, O, lse, h, rstd, logit_scale, chunk, cdt, need_x, need_g, need_W, need_E, need_b):
    out = []
    for wanted, param in ((need_x, x), (need_g and g is not None, g), (need_W, W), (need_E, E),
                          (need_b and bias is not None, bias)):
        out.append(torch.empty_like(param) if wanted else _no_grad_marker(x))
    return out


def _norm_setup(ctx, inputs, output):
    x, g, W, E, bias, eps, logit_scale, chunk, cdt = inputs
    O, lse, h, rstd = output
    ctx.save_for_backward(x, g, W, E, bias, O, lse, h, rstd)
    ctx.consts = (logit_scale, chunk, cdt)


def _norm_backward(ctx, gO, glse, _gh, _grstd):
    x, g, W, E, bias, O, lse, h, rstd = ctx.saved_tensors
    want = [bool(v) for v in ctx.needs_input_grad[:5]]
    want[1] = want[1] and g is not None
    want[4] = want[4] and bias is not None
    # an output that did not reach the loss contributes zero
    gO = torch.zeros_like(O) if gO is None else gO
    glse = torch.zeros_like(lse) if glse is None else glse
    grads = _norm_bwd_op(gO, glse, x, g, W, E, bias, O, lse, h, rstd, *ctx.consts, *want)
    return tuple(t if w else None for t, w in zip(grads, want)) + (None,) * 4


_norm_fwd_op.register_autograd(_norm_backward, setup_context=_norm_setup)


def _norm_args(x, norm_weight, eps):
    K = x.shape[-1]
    if norm_weight is not None and tuple(norm_weight.shape) != (K,):
        raise ValueError(f"norm_weight must have shape ({K},), got {tuple(norm_weight.shape)}")
    if eps is None:
        eps = torch.finfo(x.dtype).eps
    eps = float(eps)
    if not eps >= 0.0:
        raise ValueError(f"eps must be non-negative, got {eps}")
    return eps


def rmsnorm_softmax_readout(x, norm_weight, W, E, bias=None, *, eps=None, logit_scale=1.0, chunk_size=None):
    """``softmax_readout(rms_norm(x, (K,), norm_weight, eps), W, E, bias)`` with the norm fused
    into the library (the norm's weight may be None).  ``x`` is ``[..., K]``; returns ``O``
    ``[..., D]`` and ``LSE`` ``[...]`` as ``softmax_readout`` does, differentiable in ``x``, the
    norm's weight, ``W``, ``E`` and ``bias``."""
    _check(x, W, E, bias)
    eps = _norm_args(x, norm_weight, eps)
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1])
    chunk = int(chunk_size) if chunk_size else default_chunk_size()
    if chunk <= 0:
        raise ValueError(f"chunk_size must be positive, got {chunk}")
    cdt = _compute_dtype(x, W)
    with torch.autocast(x2.device.type, enabled=False):
        O, lse, _, _ = _norm_fwd_op(x2, norm_weight, W, E, bias, eps, float(logit_scale), chunk, cdt)
    return O.view(*lead, E.shape[1]), lse.view(lead)


def rmsnorm_softmax_readout_mse(x, norm_weight, W, E, target, bias=None, *, eps=None, weight=None, reduction="mean",
                                z_loss_weight=0.0, logit_scale=1.0, chunk_size=None):
    """``softmax_readout_mse`` on ``rms_norm(x, (K,), norm_weight, eps)``, the norm fused into
    the library (see ``rmsnorm_softmax_readout``); the loss arguments are those of
    ``softmax_readout_mse``."""
    if reduction not in ("none", "sum", "mean"):
        raise ValueError(f"unknown reduction {reduction!r}")
    O, lse = rmsnorm_softmax_readout(x, norm_weight, W, E, bias, eps=eps, logit_scale=logit_scale,
                                     chunk_size=chunk_size)
    lead = O.shape[:-1]
    loss = mse_loss_op(O.reshape(-1, O.shape[-1]), lse.reshape(-1), target, weight, z_loss_weight, reduction)
    return loss.view(lead) if reduction == "none" else loss


def norm_parts(norm) -> Tuple[Optional[torch.Tensor], Optional[float]]:
    """(weight, eps) of an ``nn.RMSNorm`` over the last dimension (weight None without affine)."""
    if not isinstance(norm, nn.RMSNorm):
        raise ValueError(f"norm must be an nn.RMSNorm, got {type(norm).__name__}")
    if len(norm.normalized_shape) != 1:
        raise ValueError(f"norm must normalise the last dimension only, got shape {tuple(norm.normalized_shape)}")
    return norm.weight, norm.eps
