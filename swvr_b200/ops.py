"""The readout as opaque ``torch.library`` custom ops backed by the CUDA library.

Same contract as the reference's ``swvr::chunked_fwd`` / ``swvr::chunked_bwd``
(swvr/chunked.py:157-212): the ops are opaque to ``torch.compile`` (fake impls give shapes),
the forward saves ``h, W, E, bias, O, LSE``, the backward maps missing upstream grads to
zeros, frozen inputs skip their work, empty tensors stand for "no gradient", and grads
come back in each parameter's dtype.  The reference's ``use_triton`` argument is gone:
there is one implementation, CUDA only, and CPU tensors raise.

Operand preparation is plumbing only: inputs are cast to the compute dtype ``cdt`` (as the
reference's ``.to(cdt)``) and, on the tensor-core path, re-laid out when a row pitch or base
address is not 16-byte aligned.  All arithmetic happens in libswvr_b200.so.
"""
from __future__ import annotations

import os
from typing import List, Optional, Tuple

import torch

from . import _native as nat

DEFAULT_CHUNK = 8192
LOG2E = 1.4426950408889634


def acc_dtype(cdt: torch.dtype) -> torch.dtype:
    """swvr/chunked.py:26-27."""
    return torch.float64 if cdt == torch.float64 else torch.float32


def default_chunk_size() -> int:
    """swvr/chunked.py:57-59: env ``SWVR_CHUNK`` or 8192."""
    raw = os.environ.get("SWVR_CHUNK")
    return int(raw) if raw else DEFAULT_CHUNK


def _tensor_core(cdt: torch.dtype) -> bool:
    return cdt in (torch.bfloat16, torch.float16)


TC_MAX_D = 256  # widest embedding of the tensor-core kernels (O / dE accumulators in TMEM)


def _engine_dtype(cdt: torch.dtype, D: int) -> torch.dtype:
    """The dtype the library computes in.  bf16 / fp16 run the tensor-core kernels up to
    D = 256 (the reference's Triton path covers the same range); wider embeddings (the
    reference accepts any D) run the exact fp32 SIMT kernels on fp32 copies of the operands,
    which is at least as accurate as the 16-bit contract."""
    return torch.float32 if _tensor_core(cdt) and D > TC_MAX_D else cdt


def _require_cuda(*tensors) -> torch.device:
    dev = tensors[0].device
    if dev.type != "cuda":
        raise RuntimeError(
            "swvr_b200 runs on CUDA devices only (sm_100a); got a tensor on "
            f"{dev}. There is no CPU fallback.")
    for t in tensors[1:]:
        if t is not None and t.device != dev:
            raise ValueError(f"all inputs must be on {dev}, got one on {t.device}")
    return dev


def _aligned(t: torch.Tensor) -> bool:
    es = t.element_size()
    return t.data_ptr() % 16 == 0 and (t.dim() < 2 or (t.stride(0) * es) % 16 == 0 or t.shape[0] <= 1)


def _operand(x: torch.Tensor, cdt: torch.dtype, pad_cols: int = 0) -> torch.Tensor:
    """``x`` in ``cdt`` with a unit last stride (swvr/chunked.py:66-69); for the tensor-core
    path also a 16-byte aligned base and row pitch, padding the row pitch with zeros."""
    if x.dtype != cdt:
        x = x.to(cdt)
    if x.dim() == 2 and x.shape[1] > 0 and x.stride(1) != 1:
        x = x.contiguous()
    if not _tensor_core(cdt):
        return x
    rows, cols = x.shape
    pitch = x.stride(0) if x.stride(0) >= cols else cols
    need = max(cols + pad_cols, 8)
    need = (need + 7) // 8 * 8
    if _aligned(x) and pitch % 8 == 0 and pitch >= need:
        return x
    buf = torch.zeros(rows, need, dtype=cdt, device=x.device)
    buf[:, :cols] = x
    return buf[:, :cols]


def _ld(x: torch.Tensor) -> int:
    """Row pitch in elements of a 2-D tensor with a unit last stride."""
    return x.stride(0) if x.stride(0) >= x.shape[1] else max(x.shape[1], 1)


def _problem(h, W, E, bias, scale, chunk, cdt) -> nat.Problem:
    """The C struct for one call.  It holds raw device pointers only: the caller keeps h, W, E
    and bias referenced until the launch that uses it has been issued."""
    p = nat.Problem()
    p.n_tokens, p.hidden = h.shape[0], h.shape[1]
    p.vocab, p.embed_dim = W.shape[0], E.shape[1]
    p.compute_dtype = nat.dtype_code(cdt)
    p.bias_dtype = nat.dtype_code(bias.dtype) if bias is not None else 0
    p.h, p.ldh = h.data_ptr(), _ld(h)
    p.W, p.ldw = W.data_ptr(), _ld(W)
    p.E, p.lde = E.data_ptr(), _ld(E)
    p.bias = bias.data_ptr() if bias is not None else None
    p.logit_scale = float(scale)
    p.chunk = int(chunk)
    return p


def _prepare_k(x, cdt):
    """``x`` [rows, K] as the library takes it: in ``cdt``, with K zero-padded to a multiple of 8 on
    the tensor-core path (zero columns add nothing to h . W^T)."""
    K = x.shape[1]
    if _tensor_core(cdt) and K % 8 != 0:
        x = torch.nn.functional.pad(x.to(cdt), (0, (K + 7) // 8 * 8 - K))
    return _operand(x, cdt)


def _prepare(h, W, E, bias, cdt):
    """Operands as the library takes them (see ``_prepare_k``)."""
    b = bias.contiguous() if bias is not None else None
    return _prepare_k(h, cdt), _prepare_k(W, cdt), _operand(E, cdt), b


def _param_cast_chunks(W, E, cdt) -> bool:
    """16-bit compute with parameters in another dtype (autocast over fp32 parameters): W and E
    are cast one vocabulary chunk at a time, as the reference's ``W[v0:v1].to(cdt)``
    (swvr/chunked.py:90-95, 120-146), not as whole copies."""
    return _tensor_core(cdt) and (W.dtype != cdt or E.dtype != cdt)


def _chunk_rows(V: int, chunk: int):
    rows = max(int(chunk), 1)
    return [(v0, min(v0 + rows, V)) for v0 in range(0, V, rows)]


def _workspace(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


def _forward(h, W, E, bias, logit_scale, chunk, cdt):
    dev = _require_cuda(h, W, E, bias)
    adt = acc_dtype(cdt)
    N, V, D = h.shape[0], W.shape[0], E.shape[1]
    O = torch.empty(N, D, dtype=adt, device=dev)
    lse = torch.empty(N, dtype=adt, device=dev)
    if N == 0:
        return O, lse
    if V == 0:  # the reference's loop never runs: O = 0 / 0, LSE = -inf + log(0)
        return O.fill_(float("nan")), lse.fill_(float("-inf"))
    edt = _engine_dtype(cdt, D)
    if _param_cast_chunks(W, E, edt):
        return _forward_param_cast(h, W, E, bias, logit_scale, chunk, edt, O, lse, dev)
    hc, Wc, Ec, b = _prepare(h, W, E, bias, edt)
    p = _problem(hc, Wc, Ec, b, logit_scale, chunk, edt)
    lib = nat.lib()
    nbytes = nat.c_size_t(0)
    with torch.cuda.device(dev):
        nat.check(lib.swvr_fwd_workspace_size(p, nat.ctypes.byref(nbytes)), "swvr_fwd_workspace_size")
        ws = _workspace(nbytes.value, dev)
        nat.check(lib.swvr_fwd(p, O.data_ptr(), lse.data_ptr(), ws.data_ptr(), ws.numel(), nat.stream_ptr(dev)),
                  "swvr_fwd")
    return O, lse


def _forward_param_cast(h, W, E, bias, logit_scale, chunk, cdt, O, lse, dev):
    """The forward over vocabulary chunks whose W / E rows are cast to ``cdt`` one chunk at a
    time: each chunk's online-softmax state comes from ``swvr_fwd_partial`` and
    ``swvr_combine`` merges them in chunk order."""
    N, D = h.shape[0], E.shape[1]
    spans = _chunk_rows(W.shape[0], chunk)
    m2 = torch.empty(len(spans), N, dtype=O.dtype, device=dev)
    l = torch.empty(len(spans), N, dtype=O.dtype, device=dev)
    acc = torch.empty(len(spans), N, D, dtype=O.dtype, device=dev)
    hc = _prepare_k(h, cdt)
    lib = nat.lib()
    with torch.cuda.device(dev):
        for i, (v0, v1) in enumerate(spans):
            # the problem holds raw pointers: the cast chunks must stay referenced until the
            # launch, or the caching allocator may hand their memory to the workspace below
            Wc, Ec = _prepare_k(W[v0:v1], cdt), _operand(E[v0:v1], cdt)
            b = bias[v0:v1].contiguous() if bias is not None else None
            p = _problem(hc, Wc, Ec, b, logit_scale, chunk, cdt)
            nbytes = nat.c_size_t(0)
            nat.check(lib.swvr_fwd_workspace_size(p, nat.ctypes.byref(nbytes)), "swvr_fwd_workspace_size")
            ws = _workspace(nbytes.value, dev)
            nat.check(lib.swvr_fwd_partial(p, m2[i].data_ptr(), l[i].data_ptr(), acc[i].data_ptr(), ws.data_ptr(),
                                           ws.numel(), nat.stream_ptr(dev)), "swvr_fwd_partial")
        nat.check(lib.swvr_combine(len(spans), N, D, nat.dtype_code(O.dtype), m2.data_ptr(), l.data_ptr(),
                                   acc.data_ptr(), O.data_ptr(), lse.data_ptr(), nat.stream_ptr(dev)), "swvr_combine")
    return O, lse


def _forward_state(h, W, E, bias, logit_scale, chunk, cdt):
    """The un-normalised online-softmax state ``(m2, l, acc)`` of one vocabulary shard (for the
    vocabulary-parallel merge): ``m2`` the row maximum of ``S * log2(e)``, ``l`` the sum of
    ``2^(S log2 e - m2)`` and ``acc`` those weights times the rows of E.  Frozen shapes, wide
    embeddings (the SIMT engine) and autocast over fp32 parameters go through the same
    engine choice as the single-GPU forward; with per-chunk parameter casts the state is
    rebuilt from the shard's normalised result as ``(LSE log2 e, 1, O)``, which merges the same."""
    dev = _require_cuda(h, W, E, bias)
    adt = acc_dtype(cdt)
    N, V, D = h.shape[0], W.shape[0], E.shape[1]
    m2 = torch.empty(N, dtype=adt, device=dev)
    l = torch.empty(N, dtype=adt, device=dev)
    acc = torch.empty(N, D, dtype=adt, device=dev)
    if N == 0:
        return m2, l, acc
    if V == 0:
        return m2.fill_(float("-inf")), l.zero_(), acc.zero_()
    edt = _engine_dtype(cdt, D)
    if _param_cast_chunks(W, E, edt):
        O, lse = _forward_param_cast(h, W, E, bias, logit_scale, chunk, edt, acc, l, dev)
        torch.mul(lse, LOG2E, out=m2)
        dead = torch.isneginf(m2)  # every score -inf: an empty state, not 1 x NaN
        l.fill_(1.0).masked_fill_(dead, 0.0)
        return m2, l, O.masked_fill_(dead[:, None], 0.0)
    hc, Wc, Ec, b = _prepare(h, W, E, bias, edt)
    p = _problem(hc, Wc, Ec, b, logit_scale, chunk, edt)
    lib = nat.lib()
    nbytes = nat.c_size_t(0)
    with torch.cuda.device(dev):
        nat.check(lib.swvr_fwd_workspace_size(p, nat.ctypes.byref(nbytes)), "swvr_fwd_workspace_size")
        ws = _workspace(nbytes.value, dev)
        nat.check(lib.swvr_fwd_partial(p, m2.data_ptr(), l.data_ptr(), acc.data_ptr(), ws.data_ptr(), ws.numel(),
                                       nat.stream_ptr(dev)), "swvr_fwd_partial")
    return m2, l, acc


def _grad_buffer(x: torch.Tensor, cdt: torch.dtype, tc: bool) -> Tuple[torch.Tensor, torch.Tensor]:
    """(buffer the library writes, tensor returned to autograd) for a parameter's gradient."""
    out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    if tc and x.dim() == 2 and x.dtype not in (cdt, torch.float32):
        buf = torch.empty(x.shape, dtype=torch.float32, device=x.device)
        return buf, out
    return out, out


def _backward(gO, glse, h, W, E, bias, O, lse, logit_scale, chunk, cdt, need_h, need_W, need_E, need_b,
              dh_partial=False, split=False):
    """Gradients of one readout.  With ``dh_partial`` the first result is dh un-cast, in the
    accumulation dtype (a vocabulary shard's contribution, summed across shards by the caller)
    instead of dh in h's dtype.  With ``split`` (and ``dh_partial``) a fifth result is returned:
    None, or a function ``finish(max_sms)`` that must be called, after this call and before
    gW is read, to compute the dW rows of the last vocabulary chunk (``swvr_bwd_split`` /
    ``swvr_bwd_finish``): dh is final on the current stream as soon as this call returns, so
    its cross-device exchange can run beside the finish kernel."""
    res = _backward_impl(gO, glse, h, W, E, bias, O, lse, logit_scale, chunk, cdt, need_h, need_W, need_E, need_b,
                         dh_partial, split and dh_partial)
    return res if split else res[:4]


def _backward_impl(gO, glse, h, W, E, bias, O, lse, logit_scale, chunk, cdt, need_h, need_W, need_E, need_b,
                   dh_partial, split):
    dev = _require_cuda(h, W, E, bias, gO, glse, O, lse)
    adt = O.dtype
    N, K, V, D = h.shape[0], h.shape[1], W.shape[0], E.shape[1]
    cdt = _engine_dtype(cdt, D)
    tc = _tensor_core(cdt)
    need_b = need_b and bias is not None
    if dh_partial:  # the library overwrites it (accumulate_grad_h = 0); the V == 0 / N == 0 paths zero it
        gh = torch.empty(N, K, dtype=adt, device=dev) if need_h else None
    else:
        gh = torch.empty(h.shape, dtype=h.dtype, device=dev) if need_h else None
    gW_buf, gW = _grad_buffer(W, cdt, tc) if need_W else (None, None)
    gE = torch.empty(E.shape, dtype=E.dtype, device=dev) if need_E else None
    gb = torch.empty(bias.shape, dtype=bias.dtype, device=dev) if need_b else None
    if not (need_h or need_W or need_E or need_b):
        return gh, gW, gE, gb, None
    if V == 0 or N == 0:
        for x in (gh, gW, gE, gb):
            if x is not None:
                x.zero_()
        return gh, gW, gE, gb, None
    if _param_cast_chunks(W, E, cdt):
        return (*_backward_param_cast(gO, glse, h, W, E, bias, O, lse, logit_scale, chunk, cdt, gh, gW_buf, gW, gE,
                                      gb, dev), None)
    hc, Wc, Ec, b = _prepare(h, W, E, bias, cdt)
    K8 = hc.shape[1]
    padded_k = K8 != K
    gh_buf = gh
    if need_h and padded_k:
        gh_buf = torch.empty(N, K8, dtype=gh.dtype, device=dev)
    if need_W and padded_k:
        gW_buf = torch.empty(V, K8, dtype=gW_buf.dtype, device=dev)
    p = _problem(hc, Wc, Ec, b, logit_scale, chunk, cdt)
    g = nat.Grads()
    gO = gO.to(adt).contiguous()
    glse = glse.to(adt).contiguous()
    g.grad_O, g.grad_lse, g.O, g.lse = gO.data_ptr(), glse.data_ptr(), O.data_ptr(), lse.data_ptr()
    if gh_buf is not None:
        if dh_partial:
            g.grad_h_acc = gh_buf.data_ptr()
        else:
            g.grad_h, g.grad_h_dtype = gh_buf.data_ptr(), nat.dtype_code(gh_buf.dtype)
    if gW_buf is not None:
        g.grad_W, g.grad_W_dtype, g.ld_grad_W = gW_buf.data_ptr(), nat.dtype_code(gW_buf.dtype), gW_buf.shape[1]
    if gE is not None:
        g.grad_E, g.grad_E_dtype, g.ld_grad_E = gE.data_ptr(), nat.dtype_code(gE.dtype), max(D, 1)
    if gb is not None:
        g.grad_bias, g.grad_bias_dtype = gb.data_ptr(), nat.dtype_code(gb.dtype)
    lib = nat.lib()
    nbytes = nat.c_size_t(0)
    split = split and need_W and _tensor_core(cdt)
    with torch.cuda.device(dev):
        nat.check(lib.swvr_bwd_workspace_size(p, g, nat.ctypes.byref(nbytes)), "swvr_bwd_workspace_size")
        ws = _workspace(nbytes.value, dev)
        call = lib.swvr_bwd_split if split else lib.swvr_bwd
        nat.check(call(p, g, ws.data_ptr(), ws.numel(), nat.stream_ptr(dev)), "swvr_bwd_split" if split else "swvr_bwd")
    if need_h and gh_buf is not gh:
        gh.copy_(gh_buf[:, :K])

    def finish_w():
        if need_W and gW_buf is not gW:
            gW.copy_(gW_buf[:, :K])

    if not split:
        finish_w()
        return gh, gW, gE, gb, None

    keep = (hc, Wc, Ec, b, gO, glse)  # the struct holds raw pointers into these

    def finish(max_sms=0):
        # the operand copies, grads struct and workspace stay referenced by this closure until
        # the finish kernel has been issued on the same stream
        assert keep is not None
        with torch.cuda.device(dev):
            nat.check(lib.swvr_bwd_finish(p, g, ws.data_ptr(), ws.numel(), int(max_sms), nat.stream_ptr(dev)),
                      "swvr_bwd_finish")
        finish_w()
    return gh, gW, gE, gb, finish


def _backward_param_cast(gO, glse, h, W, E, bias, O, lse, logit_scale, chunk, cdt, gh, gW_buf, gW, gE, gb, dev):
    """The backward over vocabulary chunks whose W / E rows are cast to ``cdt`` one chunk at a
    time: one ``swvr_bwd`` per chunk writes that chunk's rows of dW, dE, db and adds its dh
    into one fp32 accumulator (``accumulate_grad_h``), which is copied into ``gh`` at the end
    (cast to h's dtype, or kept fp32 when ``gh`` is an fp32 partial)."""
    N, K = h.shape
    hc = _prepare_k(h, cdt)
    K8 = hc.shape[1]
    dh = torch.empty(N, K8, dtype=torch.float32, device=dev) if gh is not None else None
    if gW_buf is not None and K8 != K:
        gW_buf = torch.empty(W.shape[0], K8, dtype=gW_buf.dtype, device=dev)
    gO = gO.to(O.dtype).contiguous()
    glse = glse.to(O.dtype).contiguous()
    lib = nat.lib()
    with torch.cuda.device(dev):
        for i, (v0, v1) in enumerate(_chunk_rows(W.shape[0], chunk)):
            Wc, Ec = _prepare_k(W[v0:v1], cdt), _operand(E[v0:v1], cdt)  # referenced until the launch
            b = bias[v0:v1].contiguous() if bias is not None else None
            p = _problem(hc, Wc, Ec, b, logit_scale, chunk, cdt)
            g = nat.Grads()
            g.grad_O, g.grad_lse, g.O, g.lse = gO.data_ptr(), glse.data_ptr(), O.data_ptr(), lse.data_ptr()
            if dh is not None:
                g.grad_h_acc, g.accumulate_grad_h = dh.data_ptr(), 1 if i > 0 else 0
            if gW_buf is not None:
                g.grad_W, g.grad_W_dtype, g.ld_grad_W = gW_buf[v0].data_ptr(), nat.dtype_code(gW_buf.dtype), K8
            if gE is not None:
                g.grad_E, g.grad_E_dtype, g.ld_grad_E = gE[v0].data_ptr(), nat.dtype_code(gE.dtype), max(E.shape[1], 1)
            if gb is not None:
                g.grad_bias, g.grad_bias_dtype = gb[v0:].data_ptr(), nat.dtype_code(gb.dtype)
            nbytes = nat.c_size_t(0)
            nat.check(lib.swvr_bwd_workspace_size(p, g, nat.ctypes.byref(nbytes)), "swvr_bwd_workspace_size")
            ws = _workspace(nbytes.value, dev)
            nat.check(lib.swvr_bwd(p, g, ws.data_ptr(), ws.numel(), nat.stream_ptr(dev)), "swvr_bwd")
    if gh is not None:
        gh.copy_(dh[:, :K])
    if gW is not None and gW_buf is not gW:
        gW.copy_(gW_buf[:, :K])
    return gh, gW, gE, gb


# The readout is a pair of opaque custom ops: torch.compile traces through neither (the fake
# impls below give it output shapes), so the vocabulary loop inside the library is never
# unrolled into [N, V]-sized graph nodes.

@torch.library.custom_op("swvr_b200::fwd", mutates_args=())
def _fwd_op(h: torch.Tensor, W: torch.Tensor, E: torch.Tensor, bias: Optional[torch.Tensor],
            logit_scale: float, chunk: int, cdt: torch.dtype) -> Tuple[torch.Tensor, torch.Tensor]:
    return _forward(h, W, E, bias, logit_scale, chunk, cdt)


@_fwd_op.register_fake
def _(h, W, E, bias, logit_scale, chunk, cdt):
    adt = acc_dtype(cdt)
    return h.new_empty(h.shape[0], E.shape[1], dtype=adt), h.new_empty(h.shape[0], dtype=adt)


def _no_grad_marker(like: torch.Tensor) -> torch.Tensor:
    """A custom op's tensor-list result has no None: a zero-element tensor marks an input whose
    gradient was not asked for."""
    return like.new_empty(0)


@torch.library.custom_op("swvr_b200::bwd", mutates_args=())
def _bwd_op(gO: torch.Tensor, glse: torch.Tensor, h: torch.Tensor, W: torch.Tensor, E: torch.Tensor,
            bias: Optional[torch.Tensor], O: torch.Tensor, lse: torch.Tensor, logit_scale: float, chunk: int,
            cdt: torch.dtype, need_h: bool, need_W: bool, need_E: bool, need_b: bool) -> List[torch.Tensor]:
    grads = _backward(gO, glse, h, W, E, bias, O, lse, logit_scale, chunk, cdt, need_h, need_W, need_E, need_b)
    return [x if x is not None else _no_grad_marker(h) for x in grads]


@_bwd_op.register_fake
def _(gO, glse, h, W, E, bias, O, lse, logit_scale, chunk, cdt, need_h, need_W, need_E, need_b):
    out = []
    for wanted, param in ((need_h, h), (need_W, W), (need_E, E), (need_b and bias is not None, bias)):
        out.append(torch.empty_like(param) if wanted else _no_grad_marker(h))
    return out


def _save_readout(ctx, inputs, output):
    """Autograd keeps the operands and (O, LSE): the backward recomputes the scores from them."""
    h, W, E, bias, logit_scale, chunk, cdt = inputs
    ctx.save_for_backward(h, W, E, bias, *output)
    ctx.consts = (logit_scale, chunk, cdt)


def _wanted_grads(ctx, bias) -> List[bool]:
    """Which of h, W, E, bias need a gradient (bias only when there is one)."""
    want = [bool(x) for x in ctx.needs_input_grad[:4]]
    want[3] = want[3] and bias is not None
    return want


def _readout_backward(ctx, gO, glse):
    h, W, E, bias, O, lse = ctx.saved_tensors
    want = _wanted_grads(ctx, bias)
    # an output that did not reach the loss has no incoming gradient: it contributes zero
    gO = torch.zeros_like(O) if gO is None else gO
    glse = torch.zeros_like(lse) if glse is None else glse
    grads = _bwd_op(gO, glse, h, W, E, bias, O, lse, *ctx.consts, *want)
    return tuple(x if w else None for x, w in zip(grads, want)) + (None,) * len(ctx.consts)


_fwd_op.register_autograd(_readout_backward, setup_context=_save_readout)


def softmax_readout_op(h2, W, E, bias, logit_scale, chunk, cdt):
    """``h2`` is ``[N, K]``; returns ``(O [N, D], LSE [N])`` in the accumulation dtype.

    Autocast is disabled inside, as in swvr/chunked.py:208-212.
    """
    with torch.autocast(h2.device.type, enabled=False):
        return _fwd_op(h2, W, E, bias, float(logit_scale), int(chunk), cdt)


# ------------------------------------------------------------------ MSE / z-loss / weight epilogue

_REDUCTIONS = {"none": nat.REDUCE_NONE, "sum": nat.REDUCE_SUM, "mean": nat.REDUCE_MEAN}


@torch.library.custom_op("swvr_b200::mse", mutates_args=())
def _mse_op(O: torch.Tensor, lse: torch.Tensor, target: torch.Tensor, weight: Optional[torch.Tensor],
            z_loss_weight: float, reduction: int) -> Tuple[torch.Tensor, torch.Tensor]:
    dev = _require_cuda(O, lse, target, weight)
    N, D = O.shape
    out = torch.empty((N,) if reduction == nat.REDUCE_NONE else (), dtype=O.dtype, device=dev)
    stats = torch.zeros(nat.MSE_STATS_LEN, dtype=O.dtype, device=dev)
    with torch.cuda.device(dev):
        nat.check(nat.lib().swvr_mse_fwd(N, D, nat.dtype_code(O.dtype), O.data_ptr(), lse.data_ptr(),
                                         target.data_ptr(), nat.ptr(weight), float(z_loss_weight), int(reduction),
                                         out.data_ptr(), stats.data_ptr(), nat.stream_ptr(dev)), "swvr_mse_fwd")
    return out, stats


@_mse_op.register_fake
def _(O, lse, target, weight, z_loss_weight, reduction):
    shape = (O.shape[0],) if reduction == nat.REDUCE_NONE else ()
    return O.new_empty(shape), O.new_empty(nat.MSE_STATS_LEN)


@torch.library.custom_op("swvr_b200::mse_bwd", mutates_args=())
def _mse_bwd_op(grad: torch.Tensor, O: torch.Tensor, lse: torch.Tensor, target: torch.Tensor,
                weight: Optional[torch.Tensor], stats: torch.Tensor, z_loss_weight: float, reduction: int,
                need_target: bool, need_weight: bool) -> List[torch.Tensor]:
    dev = _require_cuda(O, lse, target, weight, grad)
    N, D = O.shape
    grad = grad.to(O.dtype).contiguous()
    gO = torch.empty_like(O)
    glse = torch.empty_like(lse)
    gt = torch.empty_like(O) if need_target else None
    gw = torch.empty(N, dtype=O.dtype, device=dev) if (need_weight and weight is not None) else None
    with torch.cuda.device(dev):
        nat.check(nat.lib().swvr_mse_bwd(N, D, nat.dtype_code(O.dtype), O.data_ptr(), lse.data_ptr(),
                                         target.data_ptr(), nat.ptr(weight), float(z_loss_weight), int(reduction),
                                         grad.data_ptr(), stats.data_ptr(), gO.data_ptr(), glse.data_ptr(),
                                         nat.ptr(gt), nat.ptr(gw), nat.stream_ptr(dev)), "swvr_mse_bwd")
    return [gO, glse, gt if gt is not None else O.new_empty(0), gw if gw is not None else O.new_empty(0)]


@_mse_bwd_op.register_fake
def _(grad, O, lse, target, weight, stats, z_loss_weight, reduction, need_target, need_weight):
    return [torch.empty_like(O), torch.empty_like(lse),
            torch.empty_like(O) if need_target else O.new_empty(0),
            O.new_empty(O.shape[0]) if (need_weight and weight is not None) else O.new_empty(0)]


def _mse_setup(ctx, inputs, output):
    O, lse, target, weight, z, reduction = inputs
    ctx.save_for_backward(O, lse, target, weight, output[1])
    ctx.args = (z, reduction)


def _mse_backward(ctx, grad, _grad_stats):
    O, lse, target, weight, stats = ctx.saved_tensors
    z, reduction = ctx.args
    need_t = bool(ctx.needs_input_grad[2])
    need_w = bool(ctx.needs_input_grad[3]) and weight is not None
    if grad is None:
        grad = torch.zeros(O.shape[0] if reduction == nat.REDUCE_NONE else (), dtype=O.dtype, device=O.device)
    gO, glse, gt, gw = _mse_bwd_op(grad, O, lse, target, weight, stats, z, reduction, need_t, need_w)
    return gO, glse, (gt if need_t else None), (gw if need_w else None), None, None


_mse_op.register_autograd(_mse_backward, setup_context=_mse_setup)


def mse_loss_op(O, lse, target, weight, z_loss_weight, reduction: str):
    """The loss epilogue of swvr/api.py:54-66 on ``O [N, D]``, ``lse [N]``."""
    if reduction not in _REDUCTIONS:
        raise ValueError(f"unknown reduction {reduction!r}")
    N, D = O.shape
    t = target.to(O.dtype).reshape(N, D).contiguous()
    w = weight.to(O.dtype).reshape(N).contiguous() if weight is not None else None
    with torch.autocast(O.device.type, enabled=False):
        loss, _ = _mse_op(O, lse, t, w, float(z_loss_weight), _REDUCTIONS[reduction])
    return loss
