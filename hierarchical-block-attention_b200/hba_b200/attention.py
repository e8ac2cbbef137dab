"""Drop-in B200 replacements for the reference's HBA attention functions.

Signatures and argument meaning follow the reference's
``src/hba/attention.py``:

* ``hba_attention_b200`` replaces ``hba_attention_eval(q, k, v, cos, sin, cfg,
  summ, qkn, cap, hier=False, equiv=False)`` (attention.py:610-713);
* ``hba_attention_b200_fused`` replaces ``hba_attention_fused`` /
  ``hba_attention_dense`` (attention.py:552, :306), returning ``(out, aux)``:
  out is differentiable in q, k, v and the QKNorm gains through the CUDA
  backward (``hba_b200_prefill_backward``); aux is the summarizer's aux-KL
  loss (its teacher on the tensor cores, ``hba_b200_aux_teacher``),
  differentiable in the summarizer's probes and proj, or zero when
  ``cfg.aux_w == 0``.

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
    reference); aux the summarizer's aux-KL loss (``summarizer_aux_kl``), or
    a zero scalar when ``cfg.aux_w == 0`` (the reference's stage-3 skip,
    attention.py:604-606)."""
    qg, kg = qkn.q.gain, qkn.k.gain
    needs = [t.requires_grad for t in (q, k, v, qg, kg)]
    if torch.is_grad_enabled() and any(needs):
        out = _UnionSoftmax.apply(q, k, v, qg, kg, cos, sin, cfg, summ)
    else:
        out = hba_attention_b200(q, k, v, cos, sin, cfg, summ, qkn)
    if getattr(cfg, "aux_w", 1.0) == 0.0:
        return out, q.new_zeros(())
    return out, summarizer_aux_kl(q, k, cos, sin, cfg, summ, qkn)


def route_scale(cfg, dh):
    """The routing scores' scale (route_topk, attention.py:294): the content
    scale without the length temperature under QKNorm, dh**-0.5 without."""
    return content_scale(cfg, dh) if getattr(cfg, "qknorm", False) else dh ** -0.5


def aux_teacher_b200(q, k, cos, sin, cfg, qkn):
    """The aux-KL teacher pstar [B, Hkv, n, n / block] fp32 (reference
    _teacher_chunk / _aux_kl_chunked, attention.py:476-529) from raw q, k:
    per query and kv head, the group-mean of each candidate block's share of
    the NoPE softmax over all candidate keys (tensor-core kernel,
    ``hba_b200_aux_teacher``); 0 for non-candidate blocks and for queries
    without candidates (the reference's NaN rows, which its loss skips)."""
    _need_cuda(q, k)
    B, n, Hq, dh = q.shape
    Hkv = k.shape[2]
    dev = q.device
    with torch.cuda.device(dev), torch.no_grad():
        qb, kb = as_bf16(q), as_bf16(k)
        cs, sn = as_f32(cos[:n], dev), as_f32(sin[:n], dev)
        qg, kg = gains(qkn, dev)
        c = c_config(cfg, False)
        L = _lib.load()
        ws_bytes = L.hba_b200_aux_teacher_workspace_size(ctypes.byref(c), B, n)
        if ws_bytes == 0:
            _lib.check(_lib.ERR_UNSUPPORTED if n % cfg.block == 0 else _lib.ERR_NOT_BLOCK_MULTIPLE,
                       "hba_b200_aux_teacher_workspace_size")
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        pstar = torch.empty(B, Hkv, n, n // cfg.block, dtype=torch.float32, device=dev)
        st = L.hba_b200_aux_teacher(ctypes.byref(c), B, n, ctypes.c_float(union_scale(cfg, dh, n)), ptr(qb), ptr(kb),
                                    ptr(cs), ptr(sn), ptr(qg), ptr(kg), ptr(pstar), ptr(ws), ws_bytes, stream_of(dev))
        _lib.check(st, "hba_b200_aux_teacher")
        _lib.check_device(ptr(ws), stream_of(dev), "hba_b200_aux_teacher (device status)")
    return pstar


def summarizer_aux_kl(q, k, cos, sin, cfg, summ, qkn):
    """The summarizer's auxiliary KL (reference _aux_kl_chunked,
    attention.py:501-537; hba_attention_dense :364-383): -mean over (batch,
    kv head, query with a candidate) of sum_blocks pstar * log_softmax(bsc),
    pstar the teacher (``aux_teacher_b200``, no gradient) and bsc route_topk's
    block scores (``route_block_scores``).  The loss reaches only the
    summarizer's probes and proj, as in the reference; the summaries and
    scores are evaluated in fp32 by torch (the teacher is the O(n^2) part)."""
    pstar = aux_teacher_b200(q, k, cos, sin, cfg, qkn)
    with torch.no_grad():
        if getattr(cfg, "qknorm", False):
            from .ops import qknorm_b200
            qc, kc = qknorm_b200(q, qkn.q.gain), qknorm_b200(k, qkn.k.gain)
        else:
            qc, kc = q.detach(), k.detach()
    return aux_kl_from_teacher(pstar, route_block_scores(qc, kc, cfg, summ), cfg)


def route_block_scores(qc, kc, cfg, summ):
    """route_topk's block scores (attention.py:294-298), differentiable in
    the summarizer's probes / proj: the grouped query (summarizer.py:50-54)
    of the QKNorm'd queries against the slot summaries (summarizer.py:34-42)
    of the QKNorm'd keys, both detached, max over slots, x ``route_scale``,
    non-candidate blocks (attention.py:250-256) -inf.  qc [B, n, Hq, dh], kc
    [B, n, Hkv, dh] (any device, evaluated in fp32) -> [B, Hkv, n, nb]."""
    B, n, Hq, dh = qc.shape
    Hkv = kc.shape[2]
    G, Bk = Hq // Hkv, cfg.block
    nb = n // Bk
    with torch.no_grad():
        qgr = qc.detach().float().view(B, n, Hkv, G, dh).sum(3).transpose(1, 2)   # grouped query [B, Hkv, n, dh]
        kblk = kc.detach().float().view(B, nb, Bk, Hkv, dh)
    probes, proj = summ.probes.float(), summ.proj.float()
    att = (torch.einsum("hmd,bckhd->bhcmk", probes, kblk) * dh ** -0.5).softmax(-1)
    S = torch.einsum("bhcmd,hde->bhcme", torch.einsum("bhcmk,bckhd->bhcmd", att, kblk), proj)
    bsc = torch.einsum("bhid,bhcmd->bhicm", qgr, S).amax(-1) * route_scale(cfg, dh)
    return bsc.masked_fill(~_candidates(n, cfg, qc.device)[None, None], float("-inf"))


def _candidates(n, cfg, device):
    """attention.py:250-256: block b is a routed candidate of query i iff
    b >= 1 and (b + 1) * block <= i - window + 1.  -> bool [n, n / block]."""
    i = torch.arange(n, device=device)[:, None]
    blk = torch.arange(n // cfg.block, device=device)[None, :]
    return (blk >= 1) & ((blk + 1) * cfg.block <= i - cfg.window + 1)


def aux_kl_from_teacher(pstar, bsc, cfg):
    """attention.py:531-537: -mean over (batch, kv head, query with a
    candidate) of sum_blocks pstar * log_softmax(bsc), terms with pstar = 0
    dropped; a zero scalar when no query has a candidate."""
    n = bsc.shape[2]
    vq = _candidates(n, cfg, bsc.device).any(-1)
    if not bool(vq.any()):
        return bsc.new_zeros(())
    logp = torch.log_softmax(bsc[:, :, vq], dim=-1)
    pv = pstar[:, :, vq].to(logp.dtype)
    term = torch.where(pv > 0, pv * logp, torch.zeros_like(logp))
    return -term.sum(-1).mean()


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
