"""Drop-in B200 replacements for the reference's HBA attention functions.

Signatures and argument meaning follow the reference's
``src/hba/attention.py``:

* ``hba_attention_b200`` replaces ``hba_attention_eval(q, k, v, cos, sin, cfg,
  summ, qkn, cap, hier=False, equiv=False)`` (attention.py:610-713);
* ``hba_attention_b200_fused`` replaces ``hba_attention_fused`` /
  ``hba_attention_dense`` (attention.py:552, :306), returning ``(out, aux)``
  with a zero aux (the summarizer's aux-KL teacher is not built); it is
  differentiable in q, k, v and the QKNorm gains through the CUDA backward
  (``hba_b200_prefill_backward``).

``cfg`` is any object with the reference ``HBAConfig`` field names,
``summ`` a module holding ``probes [Hkv, m, dh]`` and ``proj [Hkv, dh, dh]``,
``qkn`` one holding ``q.gain [Hq]`` and ``k.gain [Hkv]``.  All compute runs in
the CUDA library (bf16 storage, fp32 accumulation); there is no CPU path.
"""

import ctypes
import math

import torch

from . import _lib

BF16 = torch.bfloat16


# ------------------------------------------------------- host scalar math ----
def content_scale(cfg, dh):
    """1/d ('inv_d', default) or 1/sqrt(d) ('inv_sqrt_d'); other modes raise
    ValueError (reference attention.py:123-141)."""
    mode = getattr(cfg, "content_scale_mode", "inv_d")
    if mode == "inv_d":
        return 1.0 / dh
    if mode == "inv_sqrt_d":
        return dh ** -0.5
    raise ValueError(f"unknown content_scale_mode {mode!r}")


def log_len_tau(cfg, n):
    """Clamped log-length temperature 1 + c*ln(max(n/n_cal, 1)); n_cal defaults
    to native_ctx; identity when c == 0 (reference attention.py:144-170)."""
    c = getattr(cfg, "temp_c", 0.0)
    if c == 0.0:
        return 1.0
    n_cal = getattr(cfg, "n_cal", None) or cfg.native_ctx
    return 1.0 + c * math.log(max(n / n_cal, 1.0))


def union_scale(cfg, dh, n):
    """The one logit scale shared by sinks, window and routed blocks: content
    scale x tau(n) under QKNorm, dh**-0.5 without (reference attention.py:183-198)."""
    if getattr(cfg, "qknorm", False):
        return content_scale(cfg, dh) * log_len_tau(cfg, n)
    return dh ** -0.5


def c_config(cfg, hier):
    """The C-ABI config struct for a reference-style config object."""
    return _lib.Config(n_heads=cfg.n_heads, n_kv=cfg.n_kv, head_dim=cfg.head_dim, block=cfg.block,
                       window=cfg.window, sinks=cfg.sinks, k_blocks=cfg.k_blocks, slots=cfg.slots,
                       fanout=getattr(cfg, "fanout", 16), beam=getattr(cfg, "beam", 4), hier=1 if hier else 0,
                       qknorm=1 if getattr(cfg, "qknorm", False) else 0, eps=1e-6)


# ----------------------------------------------------------- tensor prep -----
def ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def stream_of(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _need_cuda(*ts):
    for t in ts:
        if not t.is_cuda:
            raise RuntimeError("hba_b200 runs on CUDA tensors only (no CPU fallback)")


def as_bf16(t):
    t = t.detach()
    if t.dtype != BF16:
        t = t.to(BF16)
    return t.contiguous()


def as_f32(t, device):
    return t.detach().to(device=device, dtype=torch.float32).contiguous()


def gains(qkn, device):
    return as_f32(qkn.q.gain, device), as_f32(qkn.k.gain, device)


def summarizer_weights(summ, device):
    return as_f32(summ.probes, device), as_f32(summ.proj, device)


def _no_grad_guard(*ts):
    if torch.is_grad_enabled() and any(t.requires_grad for t in ts):
        raise NotImplementedError("hba_attention_b200 is the eval path (no backward); the differentiable training "
                                  "forward is hba_attention_b200_fused")


# ------------------------------------------------------------- forwards ------
def hba_attention_b200(q, k, v, cos, sin, cfg, summ, qkn, cap=None, hier=False, equiv=False, return_lse=False,
                       return_selection=False, check_status=True):
    """HBA attention forward on the B200 library; drop-in for
    ``hba_attention_eval`` (reference attention.py:610).

    q: [B, n, Hq, dh]; k, v: [B, n, Hkv, dh]; cos, sin: [n, dh].  ``cap`` (the
    reference's chunking memory cap) is accepted and ignored: the kernels never
    materialise per-chunk score tensors.  Returns out [B, n, Hq, dh] in q's
    dtype; with ``return_lse`` also lse [B, Hq, n] (fp32, natural log); with
    ``return_selection`` also (idx, score) [B, Hkv, n, k_blocks] (-1 = no pick).
    Raises AssertionError when n % cfg.block != 0, as the reference does, and
    HBAError when a bounded device-side wait expired (``check_status``, on by
    default, waits for the call's stream to read the kernels' status word)."""
    if equiv:
        raise NotImplementedError("equiv=True (dense uniform-RoPE attention) is not part of the HBA hot path")
    return _forward(q, k, v, cos, sin, cfg, summ, qkn, hier, 0, None, return_lse, return_selection, check_status)


def hba_attention_b200_range(q, k, v, cos, sin, cfg, summ, qkn, q_lo, n_total=None, return_lse=False,
                             return_selection=False, check_status=True):
    """Rows q_lo .. q_lo + n_q - 1 of ``hba_attention_b200`` for queries q
    [B, n_q, Hq, dh] at those positions over keys / values k, v [B, n, Hkv,
    dh] of tokens 0 .. n - 1 (n >= q_lo + n_q, a multiple of the block).
    The logit scale uses the temperature of ``n_total`` (default n): the
    length of the whole sequence whose rows these are, as the reference's
    forward applies one tau(n) to every row.  The piece a rank computes in a
    prefill split by token range.  Tensor-core path only (flat selection,
    QKNorm, block 64, G >= 4)."""
    return _forward(q, k, v, cos, sin, cfg, summ, qkn, False, int(q_lo), n_total, return_lse, return_selection,
                    check_status)


def _forward(q, k, v, cos, sin, cfg, summ, qkn, hier, q_lo, n_total, return_lse, return_selection, check_status):
    _need_cuda(q, k, v)
    _no_grad_guard(q, k, v)
    B, n_q, Hq, dh = q.shape
    n = k.shape[1]
    Hkv = k.shape[2]
    if Hq != cfg.n_heads or Hkv != cfg.n_kv or dh != cfg.head_dim:
        raise ValueError(f"shape {tuple(q.shape)}/{tuple(k.shape)} does not match the config heads")
    assert n % cfg.block == 0, (n, cfg.block)
    if q_lo < 0 or q_lo + n_q > n:
        raise ValueError(f"query rows [{q_lo}, {q_lo + n_q}) outside the {n} keys")
    dev = q.device
    with torch.cuda.device(dev):
        qb, kb, vb = as_bf16(q), as_bf16(k), as_bf16(v)
        cs, sn = as_f32(cos[:n], dev), as_f32(sin[:n], dev)
        qg, kg = gains(qkn, dev)
        probes, proj = summarizer_weights(summ, dev)
        scale = union_scale(cfg, dh, n if n_total is None else int(n_total))
        c = c_config(cfg, hier)
        L = _lib.load()
        ws_bytes = L.hba_b200_prefill_range_workspace_size(ctypes.byref(c), B, n, n_q)
        if ws_bytes == 0:
            _lib.check(_lib.ERR_UNSUPPORTED if n % cfg.block == 0 else _lib.ERR_NOT_BLOCK_MULTIPLE,
                       "hba_b200_prefill_workspace_size")
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        out = torch.empty_like(qb)
        lse = torch.empty(B, Hq, n_q, dtype=torch.float32, device=dev) if return_lse else None
        sel_i = sel_s = None
        if return_selection:
            sel_i = torch.empty(B, Hkv, n_q, cfg.k_blocks, dtype=torch.int32, device=dev)
            sel_s = torch.empty(B, Hkv, n_q, cfg.k_blocks, dtype=torch.float32, device=dev)
        st = L.hba_b200_prefill_range(ctypes.byref(c), B, n, q_lo, n_q, ctypes.c_float(scale), ptr(qb), ptr(kb),
                                      ptr(vb), ptr(cs), ptr(sn), ptr(qg), ptr(kg), ptr(probes), ptr(proj), ptr(out),
                                      ptr(lse), ptr(sel_i), ptr(sel_s), ptr(ws), ws_bytes, stream_of(dev))
        _lib.check(st, "hba_b200_prefill")
        if check_status:  # a bounded device wait that expired raises here instead of returning garbage
            _lib.check_device(ptr(ws), stream_of(dev), "hba_b200_prefill (device status)")
    res = (out.to(q.dtype),)
    if return_lse:
        res += (lse,)
    if return_selection:
        res += ((sel_i, sel_s),)
    return res[0] if len(res) == 1 else res


def hba_attention_b200_fused(q, k, v, cos, sin, cfg, summ, qkn):
    """The train-path contract ``(out, aux)`` (reference hba_attention_fused
    attention.py:552 / hba_attention_dense :306): the same union softmax,
    differentiable in q, k, v and the QKNorm gains ``qkn.q.gain`` /
    ``qkn.k.gain`` (the block selection, a top-k, has none, as in the
    reference).  aux is a zero scalar: the summarizer's aux-KL teacher
    (attention.py:478-549) is not built."""
    qg, kg = qkn.q.gain, qkn.k.gain
    needs = [t.requires_grad for t in (q, k, v, qg, kg)]
    if torch.is_grad_enabled() and any(needs):
        out = _UnionSoftmax.apply(q, k, v, qg, kg, cos, sin, cfg, summ)
    else:
        out = hba_attention_b200(q, k, v, cos, sin, cfg, summ, qkn)
    return out, q.new_zeros(())


class _Gains:
    """A stand-in for the reference's QKNorm module holding given gain tensors."""

    def __init__(self, qg, kg):
        self.q = type("G", (), {"gain": qg})()
        self.k = type("G", (), {"gain": kg})()


class _UnionSoftmax(torch.autograd.Function):
    """Forward: the prefill union softmax with its LSE and picks; backward:
    ``hba_b200_prefill_backward`` (dq, dk, dv, dgain_q, dgain_k)."""

    @staticmethod
    def forward(ctx, q, k, v, qg, kg, cos, sin, cfg, summ):
        out, lse, (sel_i, _) = _forward(q, k, v, cos, sin, cfg, summ, _Gains(qg, kg), False, 0, None, True, True, True)
        ctx.cfg = cfg
        ctx.dtypes = (q.dtype, k.dtype, v.dtype, qg.dtype, kg.dtype)
        ctx.save_for_backward(q, k, v, qg, kg, cos, sin, out, lse, sel_i)
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, qg, kg, cos, sin, out, lse, sel_i = ctx.saved_tensors
        cfg = ctx.cfg
        B, n, Hq, dh = q.shape
        Hkv = k.shape[2]
        dev = q.device
        with torch.cuda.device(dev):
            qb, kb, vb = as_bf16(q), as_bf16(k), as_bf16(v)
            ob, gb = as_bf16(out), as_bf16(dout)
            cs, sn = as_f32(cos[:n], dev), as_f32(sin[:n], dev)
            qgf, kgf = as_f32(qg, dev), as_f32(kg, dev)
            c = c_config(cfg, False)
            L = _lib.load()
            ws_bytes = L.hba_b200_prefill_backward_workspace_size(ctypes.byref(c), B, n)
            if ws_bytes == 0:
                _lib.check(_lib.ERR_UNSUPPORTED, "hba_b200_prefill_backward_workspace_size")
            ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
            dq = torch.empty_like(qb)
            dk = torch.empty_like(kb)
            dv = torch.empty_like(vb)
            dqg = torch.empty(Hq, dtype=torch.float32, device=dev)
            dkg = torch.empty(Hkv, dtype=torch.float32, device=dev)
            st = L.hba_b200_prefill_backward(ctypes.byref(c), B, n, ctypes.c_float(union_scale(cfg, dh, n)), ptr(qb),
                                             ptr(kb), ptr(vb), ptr(cs), ptr(sn), ptr(qgf), ptr(kgf), ptr(ob),
                                             ptr(lse), ptr(sel_i), ptr(gb), ptr(dq), ptr(dk), ptr(dv), ptr(dqg),
                                             ptr(dkg), ptr(ws), ws_bytes, stream_of(dev))
            _lib.check(st, "hba_b200_prefill_backward")
            _lib.check_device(ptr(ws), stream_of(dev), "hba_b200_prefill_backward (device status)")
        qd, kd, vd, qgd, kgd = ctx.dtypes
        qknorm = getattr(cfg, "qknorm", False)
        return (dq.to(qd), dk.to(kd), dv.to(vd), dqg.to(qgd) if qknorm else None, dkg.to(kgd) if qknorm else None,
                None, None, None, None)
