"""Public entry points: ``softmax_readout``, ``softmax_readout_mse`` and ``SoftmaxReadoutMSE``.

Drop-in for the reference's swvr/api.py: same names, arguments, defaults, return dtypes and
ValueErrors.  The readout runs in libswvr_b200.so through the custom ops of ``ops.py``, and
the MSE / z-loss / weight epilogue runs as a fused CUDA kernel pair instead of torch ops.
"""
import torch
from torch import nn

from .ops import default_chunk_size, mse_loss_op, softmax_readout_op


def _compute_dtype(h, W):
    """swvr/api.py:8-11: the autocast dtype if autocast is on, else ``promote_types(h, W)``."""
    if torch.is_autocast_enabled(h.device.type):
        return torch.get_autocast_dtype(h.device.type)
    return torch.promote_types(h.dtype, W.dtype)


def _check(h, W, E, bias):
    """swvr/api.py:14-22."""
    if W.dim() != 2 or E.dim() != 2:
        raise ValueError(f"W and E must be 2-D, got {tuple(W.shape)} and {tuple(E.shape)}")
    if h.shape[-1] != W.shape[1]:
        raise ValueError(f"h has hidden size {h.shape[-1]} but W is {tuple(W.shape)}")
    if E.shape[0] != W.shape[0]:
        raise ValueError(f"W has {W.shape[0]} vocabulary rows but E has {E.shape[0]}")
    if bias is not None and bias.shape != (W.shape[0],):
        raise ValueError(f"bias must have shape ({W.shape[0]},), got {tuple(bias.shape)}")


def softmax_readout(h, W, E, bias=None, *, logit_scale=1.0, chunk_size=None):
    """The softmax-weighted embedding readout (swvr/api.py:25-41).

    Scores are ``S = logit_scale * h @ W.T + bias`` over a vocabulary of V rows (W ``[V, K]``,
    optional bias ``[V]``); the result is the pair ``O = softmax(S) @ E`` (E ``[V, D]``) and
    ``LSE = logsumexp(S)``.  h may carry any leading dims ``[..., K]``: O comes back as
    ``[..., D]`` and LSE as ``[...]``, in fp32 (fp64 when the inputs are fp64), differentiable
    in every input that requires grad.  The kernels stream the vocabulary in tiles, so no
    ``[..., V]`` tensor is ever allocated; ``chunk_size`` (default 8192, env ``SWVR_CHUNK``)
    caps how many vocabulary rows of score gradients the backward keeps at once.
    """
    _check(h, W, E, bias)
    lead = h.shape[:-1]
    h2 = h.reshape(-1, h.shape[-1])
    chunk = int(chunk_size) if chunk_size else default_chunk_size()
    if chunk <= 0:
        raise ValueError(f"chunk_size must be positive, got {chunk}")
    O, lse = softmax_readout_op(h2, W, E, bias, logit_scale, chunk, _compute_dtype(h, W))
    return O.view(*lead, E.shape[1]), lse.view(lead)


def softmax_readout_mse(h, W, E, target, bias=None, *, weight=None, reduction="mean",
                        z_loss_weight=0.0, logit_scale=1.0, chunk_size=None):
    """Mean-squared error of the readout ``O`` against ``target`` (swvr/api.py:44-66).

    For each token the loss is the mean over the D embedding columns of ``(O - target)^2``,
    plus ``z_loss_weight * LSE^2`` when that weight is non-zero; an optional per-token
    ``weight`` (h's leading shape) multiplies it, so a zero weight drops the token.
    ``reduction`` is ``"mean"`` (sum over tokens divided by the sum of the weights, or by the
    token count without weights), ``"sum"`` or ``"none"`` (the per-token losses).  The
    epilogue and its gradient (also to ``target`` and ``weight``) run as one CUDA kernel pair.
    """
    if reduction not in ("none", "sum", "mean"):
        raise ValueError(f"unknown reduction {reduction!r}")
    O, lse = softmax_readout(h, W, E, bias, logit_scale=logit_scale, chunk_size=chunk_size)
    lead = O.shape[:-1]
    loss = mse_loss_op(O.reshape(-1, O.shape[-1]), lse.reshape(-1), target, weight, z_loss_weight, reduction)
    return loss.view(lead) if reduction == "none" else loss


def _weight_of(x):
    return x.weight if isinstance(x, nn.Module) else x


class SoftmaxReadoutMSE(nn.Module):
    """``softmax_readout_mse`` as an ``nn.Module`` bound to a model's head and codebook
    (swvr/api.py:69-93).

    ``head`` may be an ``nn.Linear(K, V)`` (whose bias, if any, becomes the score bias) or a
    plain ``[V, K]`` weight; ``embedding`` an ``nn.Embedding(V, D)`` or a ``[V, D]`` table.
    The module stores the objects it is given, never copies, so tied weights and the
    optimizer's view of the parameters are unaffected.  Optionally (not in the reference),
    ``norm``, an ``nn.RMSNorm(K)``, is applied to the input first, fused into the library
    (``rmsnorm_softmax_readout_mse``): ``forward`` then takes the trunk output before the norm.
    """

    def __init__(self, head, embedding, *, z_loss_weight=0.0, logit_scale=1.0,
                 reduction="mean", chunk_size=None, norm=None):
        super().__init__()
        self.head, self.embedding = head, embedding
        self.z_loss_weight, self.logit_scale = z_loss_weight, logit_scale
        self.reduction, self.chunk_size = reduction, chunk_size
        if norm is not None:
            from .norm import norm_parts
            norm_parts(norm)  # validates it
        self.norm = norm

    def forward(self, h, target, weight=None):
        bias = getattr(self.head, "bias", None) if isinstance(self.head, nn.Module) else None
        kw = dict(weight=weight, reduction=self.reduction, z_loss_weight=self.z_loss_weight,
                  logit_scale=self.logit_scale, chunk_size=self.chunk_size)
        if self.norm is not None:
            from .norm import norm_parts, rmsnorm_softmax_readout_mse
            g, eps = norm_parts(self.norm)
            return rmsnorm_softmax_readout_mse(h, g, _weight_of(self.head), _weight_of(self.embedding), target,
                                               bias, eps=eps, **kw)
        return softmax_readout_mse(h, _weight_of(self.head), _weight_of(self.embedding), target, bias, **kw)
