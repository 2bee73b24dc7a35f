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
    """Return ``(O, LSE)`` for ``S = logit_scale * h @ W.T + bias`` (swvr/api.py:25-41).

    ``O = softmax(S) @ E`` has shape ``[..., D]`` and ``LSE = logsumexp(S)`` has shape ``[...]``,
    both in fp32 (fp64 for fp64 inputs). ``h`` is ``[..., K]``, ``W`` is ``[V, K]``, ``E`` is
    ``[V, D]`` and ``bias`` is ``[V]``. Gradients flow to every input that requires them.
    The ``[..., V]`` scores are never materialised; ``chunk_size`` (default 8192, or env
    ``SWVR_CHUNK``) bounds the vocabulary rows whose score gradients the backward stages.
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
    """MSE between ``softmax(S) @ E`` and ``target`` (``[..., D]``), plus an optional z-loss.

    swvr/api.py:44-66. The per-token loss is ``mean_d (O - target)^2 + z_loss_weight * LSE^2``.
    ``weight`` (shape ``[...]``) scales each token's loss, and 0 masks it out.
    ``reduction="mean"`` divides by ``weight.sum()`` when a weight is given, else by the token
    count. ``"sum"`` and ``"none"`` are also accepted.
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
    """Loss module around an existing LM head and embedding table (swvr/api.py:69-93).

    ``head`` is an ``nn.Linear(K, V)`` (its bias is used if present) or a ``[V, K]`` tensor;
    ``embedding`` is an ``nn.Embedding(V, D)`` or a ``[V, D]`` tensor. The module keeps
    references, not copies, so weight tying and optimizer state stay intact.
    """

    def __init__(self, head, embedding, *, z_loss_weight=0.0, logit_scale=1.0,
                 reduction="mean", chunk_size=None):
        super().__init__()
        self.head, self.embedding = head, embedding
        self.z_loss_weight, self.logit_scale = z_loss_weight, logit_scale
        self.reduction, self.chunk_size = reduction, chunk_size

    def forward(self, h, target, weight=None):
        bias = getattr(self.head, "bias", None) if isinstance(self.head, nn.Module) else None
        return softmax_readout_mse(
            h, _weight_of(self.head), _weight_of(self.embedding), target, bias,
            weight=weight, reduction=self.reduction, z_loss_weight=self.z_loss_weight,
            logit_scale=self.logit_scale, chunk_size=self.chunk_size)
