"""Eager reference (public API): materialises the ``[N, V]`` scores. For small shapes only.

Kept for API compatibility with the reference library (swvr/reference.py:5-14), which
exports it as ``swvr.softmax_readout_reference``.  It is never called by the fused op.
"""
import torch


def softmax_readout_reference(h, W, E, bias=None, logit_scale=1.0):
    """Same contract as ``softmax_readout``, computed eagerly in at least fp32."""
    dtype = torch.float32
    for t in (h, W, E, bias):
        if t is not None:
            dtype = torch.promote_types(dtype, t.dtype)
    S = logit_scale * (h.to(dtype) @ W.to(dtype).T)
    if bias is not None:
        S = S + bias.to(dtype)
    return torch.softmax(S, dim=-1) @ E.to(dtype), torch.logsumexp(S, dim=-1)
