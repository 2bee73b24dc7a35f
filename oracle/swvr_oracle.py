"""CPU oracle for the softmax-weighted embedding readout -- TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product. Only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py`` (its ``cpu_baseline`` leg and its ``--impl reference`` arm) may import it.
The product path (``swvr_b200``) never imports or calls anything here and fails loudly when
its CUDA library is missing.

It restates, in numpy, the algorithm of the reference library pengzhangzhi/swvr:

* ``softmax_readout_reference``  -- the eager, materialising oracle (swvr/reference.py:5-14).
* ``chunked_forward``            -- the chunked online-softmax forward, torch path
                                    (swvr/chunked.py:82-105, with mm_acc 30-55 and _scores 72-79).
* ``chunked_backward``           -- the recomputing backward, torch path (swvr/chunked.py:108-151).
* ``readout_grads``              -- analytic gradients of the eager oracle (the autograd of
                                    swvr/reference.py:5-14, written out).
* ``mse_forward`` / ``mse_backward`` -- the loss epilogue of swvr/api.py:44-66 and its gradient.
* ``rmsnorm_forward`` / ``rmsnorm_backward`` -- the RMSNorm that the fused producer of h
                                    computes (torch.nn.functional.rms_norm over the last
                                    dimension; not part of the reference), in fp64.

Precision is restated exactly as the reference's torch path has it (swvr/chunked.py:1-13):
matrix-product operands are rounded to the compute dtype ``cdt`` (bf16/fp16 emulated by
round-to-nearest-even on the fp32 bit pattern), products accumulate in fp32 (fp64 for fp64),
scores are never rounded, ``P`` is rounded to ``cdt`` before ``P @ E`` (chunked.py:101) and
``P^T @ gO`` (chunked.py:137), and ``gS`` is scaled then rounded to ``cdt`` before the
``dh``/``dW`` products (chunked.py:142-145).

Parity is pinned: ``tests/test_oracle_golden.py`` checks every function here against golden
vectors produced by running the reference itself (``tests/golden/make_golden.py``).
"""
from __future__ import annotations

import numpy as np

LOG2E = 1.4426950408889634

# ---------------------------------------------------------------------------------------------
# dtype emulation
# ---------------------------------------------------------------------------------------------


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round an fp32 array to the nearest bf16 value (ties to even); returned as fp32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    bits = x.view(np.uint32).astype(np.uint64)
    rounded = (bits + 0x7FFF + ((bits >> 16) & 1)) & 0xFFFF0000
    out = rounded.astype(np.uint32).view(np.float32).copy()
    nan = np.isnan(x)
    if nan.any():
        out[nan] = np.nan
    return out


def round_fp16(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def round_to(x: np.ndarray, cdt: str) -> np.ndarray:
    """``x.to(cdt)`` followed by the upcast the reference's CPU ``mm_acc`` does (chunked.py:55)."""
    if cdt == "bf16":
        return round_bf16(x)
    if cdt == "fp16":
        return round_fp16(x)
    if cdt == "fp32":
        return np.asarray(x, dtype=np.float32)
    if cdt == "fp64":
        return np.asarray(x, dtype=np.float64)
    raise ValueError(f"unknown compute dtype {cdt!r}")


def acc_dtype(cdt: str):
    """swvr/chunked.py:26-27: fp64 accumulation for fp64 compute, else fp32."""
    return np.float64 if cdt == "fp64" else np.float32


# ---------------------------------------------------------------------------------------------
# eager oracle (swvr/reference.py:5-14)
# ---------------------------------------------------------------------------------------------


def softmax_readout_reference(h, W, E, bias=None, logit_scale=1.0, dtype=np.float64):
    """Materialise ``S = logit_scale * h @ W.T + bias``; return ``(softmax(S) @ E, logsumexp(S))``.

    Restates swvr/reference.py:5-14. ``dtype`` is the promoted dtype (at least fp32).
    """
    h, W, E = (np.asarray(x, dtype=dtype) for x in (h, W, E))
    S = dtype(logit_scale) * (h @ W.T)
    if bias is not None:
        S = S + np.asarray(bias, dtype=dtype)
    m = S.max(axis=-1, keepdims=True)
    m = np.where(np.isfinite(m), m, 0.0)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        ex = np.exp(S - m)
        l = ex.sum(axis=-1, keepdims=True)
        P = ex / l
        lse = (m + np.log(l))[..., 0]
    return P @ E, lse


def readout_grads(h, W, E, bias, gO, glse, logit_scale=1.0, dtype=np.float64):
    """Analytic gradients of ``softmax_readout_reference`` for upstream ``(gO, glse)``.

    ``dS = P * (gO @ E.T - delta)``, ``delta = rowsum(O * gO) - glse`` (the derivation in the
    reference's docs/DESIGN.md:23-33); ``dh = s dS W``, ``dW = s dS^T h``, ``dE = P^T gO``,
    ``db = colsum(dS)``. Returns ``(dh, dW, dE, db)`` (``db`` is None without a bias).
    """
    h, W, E = (np.asarray(x, dtype=dtype) for x in (h, W, E))
    gO = np.asarray(gO, dtype=dtype)
    glse = np.asarray(glse, dtype=dtype)
    S = dtype(logit_scale) * (h @ W.T)
    if bias is not None:
        S = S + np.asarray(bias, dtype=dtype)
    m = S.max(axis=-1, keepdims=True)
    m = np.where(np.isfinite(m), m, 0.0)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        ex = np.exp(S - m)
        P = ex / ex.sum(axis=-1, keepdims=True)
    O = P @ E
    delta = (O * gO).sum(-1) - glse
    dS = P * (gO @ E.T - delta[:, None])
    dS = np.where(P == 0, 0.0, dS)
    db = dS.sum(0) if bias is not None else None
    dE = P.T @ gO
    dSs = dS * dtype(logit_scale)
    return dSs @ W, dSs.T @ h, dE, db


# ---------------------------------------------------------------------------------------------
# chunked algorithm, torch path (swvr/chunked.py:82-151)
# ---------------------------------------------------------------------------------------------


def _scores(hc, W, bias, v0, v1, s, cdt):
    """swvr/chunked.py:72-79: ``s * hc @ W[v0:v1].T + bias[v0:v1]`` in the accumulation dtype."""
    adt = acc_dtype(cdt)
    S = (hc @ round_to(W[v0:v1], cdt).T).astype(adt)
    if s != 1.0:
        S *= adt(s)
    if bias is not None:
        S += np.asarray(bias[v0:v1], dtype=adt)
    return S


def chunked_forward(h, W, E, bias, logit_scale, chunk, cdt):
    """Online softmax over vocabulary chunks; returns ``(O [N, D], LSE [N])``.

    Restates swvr/chunked.py:82-105 (the torch branch, 96-104).
    """
    adt = acc_dtype(cdt)
    N, V, D = h.shape[0], W.shape[0], E.shape[1]
    hc = round_to(h, cdt)
    m = np.full(N, -np.inf, dtype=adt)
    l = np.zeros(N, dtype=adt)
    acc = np.zeros((N, D), dtype=adt)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        for v0 in range(0, V, chunk):
            v1 = min(v0 + chunk, V)
            S = _scores(hc, W, bias, v0, v1, logit_scale, cdt)
            m_new = np.maximum(m, S.max(axis=1)) if S.shape[1] else m
            # chunked.py:97-98: a row whose scores so far are all -inf is shifted by 0
            shift = np.where(np.isinf(m_new), 0.0, m_new).astype(adt)
            alpha = np.exp(m - shift).astype(adt)
            P = np.exp(S - shift[:, None]).astype(adt)
            l = l * alpha + P.sum(axis=1, dtype=adt)
            acc = acc * alpha[:, None] + (round_to(P, cdt) @ round_to(E[v0:v1], cdt)).astype(adt)
            m = m_new
        return (acc / l[:, None]).astype(adt), (m + np.log(l)).astype(adt)


def chunked_backward(gO, glse, h, W, E, bias, O, lse, logit_scale, chunk, cdt,
                     need_h=True, need_W=True, need_E=True, need_b=True):
    """Recompute backward; returns ``(gh, gW, gE, gb)`` in the accumulation dtype.

    Restates swvr/chunked.py:108-151 (the torch branch, 132-145, then the GEMMs 146-150).
    """
    adt = acc_dtype(cdt)
    N, V = h.shape[0], W.shape[0]
    s = logit_scale
    hc = round_to(h, cdt)
    O = np.asarray(O, dtype=adt)
    lse = np.asarray(lse, dtype=adt)
    delta = (O * np.asarray(gO, dtype=adt)).sum(axis=1, dtype=adt) - np.asarray(glse, dtype=adt)
    gOc = round_to(gO, cdt)
    gH = np.zeros((N, h.shape[1]), dtype=adt) if need_h else None
    gW = np.zeros(W.shape, dtype=adt) if need_W else None
    gE = np.zeros(E.shape, dtype=adt) if need_E else None
    need_b = need_b and bias is not None
    gb = np.zeros(V, dtype=adt) if need_b else None
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        for v0 in range(0, V, chunk):
            v1 = min(v0 + chunk, V)
            P = np.exp(_scores(hc, W, bias, v0, v1, s, cdt) - lse[:, None]).astype(adt)
            gS = ((gOc @ round_to(E[v0:v1], cdt).T).astype(adt) - delta[:, None]) * P
            if need_b:
                gb[v0:v1] = gS.sum(axis=0, dtype=adt)
            if need_E:
                gE[v0:v1] = round_to(P, cdt).T @ gOc
            if not (need_h or need_W):
                continue
            if s != 1.0:
                gS = gS * adt(s)
            gS = round_to(gS, cdt)
            Wc = round_to(W[v0:v1], cdt)
            if need_h:
                gH += (gS @ Wc).astype(adt)
            if need_W:
                gW[v0:v1] = gS.T @ hc
    return gH, gW, gE, gb


# ---------------------------------------------------------------------------------------------
# MSE / z-loss / per-token-weight epilogue (swvr/api.py:44-66)
# ---------------------------------------------------------------------------------------------


def mse_forward(O, lse, target, weight=None, reduction="mean", z_loss_weight=0.0):
    """swvr/api.py:54-66. ``O`` is ``[N, D]``, ``lse`` ``[N]``; returns the reduced loss."""
    O = np.asarray(O)
    dt = O.dtype
    per_tok = ((O - np.asarray(target, dtype=dt)) ** 2).mean(axis=-1)
    if z_loss_weight:
        per_tok = per_tok + dt.type(z_loss_weight) * np.asarray(lse, dtype=dt) ** 2
    if weight is not None:
        per_tok = per_tok * np.asarray(weight, dtype=dt)
    if reduction == "none":
        return per_tok
    if reduction == "sum":
        return per_tok.sum()
    if reduction == "mean":
        denom = np.asarray(weight, dtype=dt).sum() if weight is not None else per_tok.size
        return per_tok.sum() / denom
    raise ValueError(f"unknown reduction {reduction!r}")


def mse_backward(O, lse, target, weight=None, reduction="mean", z_loss_weight=0.0, grad=1.0):
    """Gradient of ``mse_forward`` w.r.t. ``(O, lse, target, weight)`` for upstream ``grad``.

    ``grad`` is a scalar for "mean"/"sum" and an ``[N]`` array for "none".
    """
    O = np.asarray(O)
    dt = O.dtype
    t = np.asarray(target, dtype=dt)
    lse = np.asarray(lse, dtype=dt)
    N, D = O.shape
    w = np.asarray(weight, dtype=dt) if weight is not None else None
    raw = ((O - t) ** 2).mean(axis=-1) + (dt.type(z_loss_weight) * lse ** 2 if z_loss_weight else 0)
    g = np.asarray(grad, dtype=dt)
    if reduction == "none":
        c = g * (w if w is not None else 1.0)
        gw = g * raw if w is not None else None
    elif reduction == "sum":
        c = g * (w if w is not None else np.ones(N, dtype=dt))
        gw = g * raw if w is not None else None
    elif reduction == "mean":
        denom = w.sum() if w is not None else dt.type(N)
        c = g * (w if w is not None else np.ones(N, dtype=dt)) / denom
        if w is not None:
            loss = (raw * w).sum() / denom
            gw = g * (raw - loss) / denom
        else:
            gw = None
    else:
        raise ValueError(f"unknown reduction {reduction!r}")
    c = np.broadcast_to(c, (N,))
    gO = c[:, None] * dt.type(2.0 / D) * (O - t)
    glse = c * dt.type(2.0 * z_loss_weight) * lse
    return gO, glse, -gO, gw


# ---------------------------------------------------------------------------------------------
# vocabulary-shard combine (the merge step of the online softmax across shards)
# ---------------------------------------------------------------------------------------------


def combine_partials(m2, l, acc):
    """Merge per-shard online-softmax states in shard order.

    ``m2 [G, N]`` are reference maxima in log2 units, ``l [G, N]`` the partial sums of
    ``2^(x*log2e - m2)`` and ``acc [G, N, D]`` the partial ``P @ E``. Returns ``(O, LSE)``.
    This is the combine of chunked.py:96-105 applied across shards instead of chunks.
    """
    m2 = np.asarray(m2, dtype=np.float64)
    l = np.asarray(l, dtype=np.float64)
    acc = np.asarray(acc, dtype=np.float64)
    m = m2.max(axis=0)
    ref = np.where(np.isinf(m), 0.0, m)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        scale = np.exp2(m2 - ref[None])
        L = (l * scale).sum(0)
        A = (acc * scale[..., None]).sum(0)
        return A / L[:, None], (ref + np.log2(L)) / LOG2E


def shard_partials(h, W, E, bias, logit_scale, G):
    """Per-shard ``(m2, l, acc)`` of an fp64 eager computation over ``G`` equal vocab shards."""
    V = W.shape[0]
    bounds = [(r * V) // G for r in range(G + 1)]
    m2s, ls, accs = [], [], []
    for r in range(G):
        v0, v1 = bounds[r], bounds[r + 1]
        S = float(logit_scale) * (np.asarray(h, np.float64) @ np.asarray(W[v0:v1], np.float64).T)
        if bias is not None:
            S = S + np.asarray(bias[v0:v1], np.float64)
        x2 = S * LOG2E
        with np.errstate(divide="ignore", invalid="ignore"):
            m2 = x2.max(axis=1) if v1 > v0 else np.full(S.shape[0], -np.inf)
            ref = np.where(np.isinf(m2), 0.0, m2)
            p = np.exp2(x2 - ref[:, None])
        m2s.append(m2)
        ls.append(p.sum(1))
        accs.append(p @ np.asarray(E[v0:v1], np.float64))
    return np.stack(m2s), np.stack(ls), np.stack(accs)


# ---------------------------------------------------------------------------------------------
# RMSNorm producer of h (no counterpart in the reference; the norm of
# torch.nn.functional.rms_norm over the last dimension, fp64)
# ---------------------------------------------------------------------------------------------


def rmsnorm_forward(x, weight=None, eps=1e-6):
    """(h, rstd): h = x * rstd * weight, rstd = 1 / sqrt(mean_k x^2 + eps), in fp64."""
    x = np.asarray(x, dtype=np.float64)
    rstd = 1.0 / np.sqrt((x * x).mean(axis=-1) + eps)
    h = x * rstd[..., None]
    if weight is not None:
        h = h * np.asarray(weight, dtype=np.float64)
    return h, rstd


def rmsnorm_backward(dh, x, weight=None, eps=1e-6):
    """(dx, dweight) of rmsnorm_forward for the upstream gradient dh, in fp64:
    dx = rstd * (a - xh * mean_k(a * xh)) with a = dh * weight and xh = x * rstd;
    dweight = sum over rows of dh * xh (None without a weight)."""
    x = np.asarray(x, dtype=np.float64)
    dh = np.asarray(dh, dtype=np.float64)
    _, rstd = rmsnorm_forward(x, None, eps)
    xh = x * rstd[..., None]
    g = np.ones(x.shape[-1]) if weight is None else np.asarray(weight, dtype=np.float64)
    a = dh * g
    dx = rstd[..., None] * (a - xh * (a * xh).mean(axis=-1, keepdims=True))
    dw = None if weight is None else (dh * xh).reshape(-1, x.shape[-1]).sum(axis=0)
    return dx, dw
