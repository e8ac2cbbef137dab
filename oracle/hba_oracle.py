"""CPU oracle for the HBA attention hot path.  TEST INFRASTRUCTURE ONLY.

This module is the checker, never the thing measured or shipped: only the
test suite, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` / reference
legs of ``bench.py`` may import it.  The product path (package ``hba_b200``)
runs on the CUDA library and fails loudly without it.

It restates, in numpy, the algorithm of the reference implementation
(``src/hba/attention.py`` and ``src/hba/summarizer.py`` of
nealxpatel/hierarchical-block-attention); every function names the lines it
follows.  Parity is pinned by ``tests/test_oracle_golden.py`` against vectors
produced by running the reference itself (``tests/golden/make_golden.py``).

Precision policy.  The GPU path stores q/k/v, QKNorm'd keys, block summaries
and super-summaries as bf16.  The oracle takes those stored values (as
float32 arrays that hold exact bf16 values) and evaluates everything after
them in float64, so the CUDA path is compared against the exact math on the
exact bytes it consumed.  Where the reference materialises a tensor in the
input dtype *and* the CUDA path does the same (QKNorm output, grouped routing
query, the RoPE'd window q and k of the tensor-core tiles), ``bf16=True``
applies the same round-to-nearest-even to bf16.

Selection order: ``torch.topk`` leaves tie order unspecified; the oracle
orders picks by (score descending, block index ascending).  Parity tests
accept a differing pick only where the two scores are within 1e-6 logit.
"""

import math

import numpy as np

NEG_INF = -np.inf


# ------------------------------------------------------------ bf16 helpers ----
def round_bf16(x):
    """Round float32 values to the nearest bf16 (ties to even), returned as
    float32.  Same rounding as ``torch.Tensor.to(torch.bfloat16)``."""
    a = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    u = a.view(np.uint32).astype(np.uint64)
    lsb = (u >> np.uint64(16)) & np.uint64(1)
    r = ((u + np.uint64(0x7FFF) + lsb) & np.uint64(0xFFFF0000)).astype(np.uint32)
    out = r.view(np.float32).reshape(a.shape)
    nan = np.isnan(a)
    if nan.any():
        out = out.copy()
        out[nan] = np.nan
    return out


# ------------------------------------------------------------- scalars --------
def content_scale(mode, dh):
    """attention.py:123-141 -- 1/d ('inv_d') or 1/sqrt(d) ('inv_sqrt_d')."""
    if mode == "inv_d":
        return 1.0 / dh
    if mode == "inv_sqrt_d":
        return dh ** -0.5
    raise ValueError(f"unknown content_scale_mode {mode!r}")


def log_len_tau(temp_c, n_cal, native_ctx, n):
    """attention.py:144-170 -- tau = 1 + c*ln(max(n/n_cal, 1)); identity when
    c == 0; n_cal defaults to native_ctx."""
    if temp_c == 0.0:
        return 1.0
    cal = n_cal or native_ctx
    return 1.0 + temp_c * math.log(max(n / cal, 1.0))


def union_scale(qknorm, mode, temp_c, n_cal, native_ctx, dh, n):
    """attention.py:183-198 (`_content_qk`'s scale): content_scale * tau under
    QKNorm, else the legacy dh**-0.5 with no temperature."""
    if qknorm:
        return content_scale(mode, dh) * log_len_tau(temp_c, n_cal, native_ctx, n)
    return dh ** -0.5


# ------------------------------------------------------------- QKNorm ---------
def head_rmsnorm(x, gain, eps=1e-6, bf16=False):
    """attention.py:88-94 (`_HeadRMSNorm.forward`): per head, x / sqrt(max(mean(x^2), eps))
    times a scalar gain; math in float32, cast back to the input dtype.
    x: [..., H, dh]; gain: [H]."""
    xf = np.asarray(x, np.float32)
    ms = np.mean(xf * xf, axis=-1, keepdims=True, dtype=np.float32)
    rms = np.sqrt(np.maximum(ms, np.float32(eps)))
    y = (xf / rms) * np.asarray(gain, np.float32)[:, None]
    y = y.astype(np.float32)
    return round_bf16(y) if bf16 else y


# ------------------------------------------------------------- RoPE -----------
def rope_tables(n, dh, theta):
    """attention.py:27-32: NeoX tables cat(fr, fr) with fr = pos * theta^(-2i/dh),
    float32.  Returns (cos, sin), each [n, dh]."""
    inv = (1.0 / (np.float32(theta) ** (np.arange(0, dh, 2, dtype=np.float32) / np.float32(dh)))
           ).astype(np.float32)
    pos = np.arange(n, dtype=np.float32)
    fr = np.outer(pos, inv).astype(np.float32)
    emb = np.concatenate([fr, fr], axis=-1)
    return np.cos(emb).astype(np.float32), np.sin(emb).astype(np.float32)


def rot_half(x):
    """attention.py:35-37: (-x[d/2:], x[:d/2])."""
    d = x.shape[-1] // 2
    return np.concatenate([-x[..., d:], x[..., :d]], axis=-1)


def apply_rope(x, cos_rows, sin_rows):
    """attention.py:40-44: x*cos + rot_half(x)*sin.  ``cos_rows``/``sin_rows``
    must broadcast against x (rows already gathered at x's positions)."""
    x = np.asarray(x, np.float64)
    return x * cos_rows + rot_half(x) * sin_rows


def apply_rope_bf16(x, cos_rows, sin_rows):
    """The RoPE'd tensor-core operand of the bf16 path: the same rotation of
    the stored bf16 values (x), evaluated in float32 as rn(rn(x*cos) +
    rn(rot_half(x)*sin)) -- numpy float32 ops round each product and the sum,
    with no fused multiply-add -- then rounded once to bf16.  The reference's
    bf16 path (attention.py:40-44 on bf16 tensors) rounds the same tensor to
    bf16; the CUDA kernels compute exactly this, so kernel and oracle hold
    bit-identical window operands."""
    x = np.asarray(x, np.float32)
    c = np.asarray(cos_rows, np.float32)
    s_ = np.asarray(sin_rows, np.float32)
    y = (x * c) + (rot_half(x) * s_)
    return round_bf16(y.astype(np.float32)).astype(np.float64)


# ------------------------------------------------------- slot summaries -------
def summarize(kc, probes, proj, Bk):
    """summarizer.py:34-42 (`SlotSummarizer.summarize`).
    kc: [B, n, Hkv, dh] QKNorm'd NoPE keys; probes: [Hkv, m, dh]; proj: [Hkv, dh, dh].
    Per 64-key block: att = softmax_k(probes . k * dh^-0.5); pooled = att @ k;
    S = pooled @ proj.  Returns S: [B, Hkv, nb, m, dh] (float64)."""
    kc = np.asarray(kc, np.float64)
    B, n, Hkv, dh = kc.shape
    nb = n // Bk
    kb = kc[:, : nb * Bk].reshape(B, nb, Bk, Hkv, dh)
    att = np.einsum("hmd,bckhd->bhcmk", np.asarray(probes, np.float64), kb) * dh ** -0.5
    att = att - att.max(-1, keepdims=True)
    att = np.exp(att)
    att /= att.sum(-1, keepdims=True)
    pooled = np.einsum("bhcmk,bckhd->bhcmd", att, kb)
    return np.einsum("bhcmd,hde->bhcme", pooled, np.asarray(proj, np.float64))


def grouped_query(qc, Hkv, bf16=False):
    """summarizer.py:50-54: sum of the G contiguous query heads of each KV
    group.  qc: [B, n, Hq, dh] -> [B, Hkv, n, dh].  In bf16 the reference
    materialises the sum in bf16; ``bf16=True`` reproduces that rounding."""
    qc = np.asarray(qc, np.float32)
    B, n, Hq, dh = qc.shape
    G = Hq // Hkv
    q5 = qc.reshape(B, n, Hkv, G, dh)
    s = q5[:, :, :, 0, :].copy()
    for h in range(1, G):                     # fp32 adds in head order (the CUDA path's order)
        s = (s + q5[:, :, :, h, :]).astype(np.float32)
    s = s.transpose(0, 2, 1, 3)
    return round_bf16(s) if bf16 else s


def route_candidates(pos, W, nb, Bk):
    """attention.py:250-256 (and the eval inline copy :689): block b is a
    routed candidate of the query at position i iff b >= 1 and
    (b+1)*Bk <= i - W + 1.  pos: [c] int -> bool [c, nb]."""
    pos = np.asarray(pos, np.int64)[:, None]
    b = np.arange(nb, dtype=np.int64)[None, :]
    return (b >= 1) & ((b + 1) * Bk <= pos - W + 1)


def build_super(S0, fanout):
    """attention.py:202-214: per-slot mean of `fanout` children, zero-padded
    with the last group's count corrected.  S0: [..., nb, m, dh] -> [..., ns, m, dh]."""
    S0 = np.asarray(S0, np.float64)
    nb = S0.shape[-3]
    ns = -(-nb // fanout)
    pad = ns * fanout - nb
    if pad:
        z = np.zeros(S0.shape[:-3] + (pad,) + S0.shape[-2:], np.float64)
        S0 = np.concatenate([S0, z], axis=-3)
    S1 = S0.reshape(S0.shape[:-3] + (ns, fanout) + S0.shape[-2:]).sum(-3)
    cnt = np.full((ns,), float(fanout))
    if pad:
        cnt[-1] = fanout - pad
    return S1 / cnt[:, None, None], ns


# ------------------------------------------------------------- top-k ----------
def topk_desc(scores, k):
    """Top-k along the last axis ordered by (score desc, index asc).
    Returns (idx int64, val float64), -inf entries kept (callers mask them,
    as the reference's eval path does at attention.py:693,698)."""
    scores = np.asarray(scores, np.float64)
    nb = scores.shape[-1]
    k = min(k, nb)
    order = np.lexsort((np.broadcast_to(np.arange(nb), scores.shape), -scores), axis=-1)
    idx = order[..., :k]
    return idx, np.take_along_axis(scores, idx, -1)


def slot_scores(qg, S, scale):
    """summarizer.py:45-47 and attention.py:695: max over slots of (qg . S) * scale.
    qg: [..., dh]; S: [..., nb, m, dh] -> [..., nb]."""
    qg = np.asarray(qg, np.float64)
    S = np.asarray(S, np.float64)
    return np.einsum("...d,...nmd->...nm", qg, S).max(-1) * scale


def flat_select(qg, S, cand, k, scale):
    """Flat scan, attention.py:694-698 (same pick set as route_topk :272-303):
    mask non-candidates to -inf, take top-k.
    qg: [c, dh]; S: [nb, m, dh]; cand: [c, nb] -> (idx [c,k], val [c,k])."""
    sc = np.einsum("cd,nmd->cnm", np.asarray(qg, np.float64), np.asarray(S, np.float64)).max(-1) * scale
    sc = np.where(cand, sc, NEG_INF)
    return topk_desc(sc, k)


def hier_select(qg, S0, S1, fanout, beam, k, cand, scale):
    """attention.py:217-246 (`hier_select`): score super-summaries (masked to
    supers holding any candidate), keep the top `beam`, expand to their
    children, score those (masked to candidates in range), keep top-k.
    qg: [c, dh]; S0: [nb, m, dh]; S1: [ns, m, dh]; cand: [c, nb].
    Returns (idx [c,kk], val [c,kk], n_comparisons)."""
    qg = np.asarray(qg, np.float64)
    S0 = np.asarray(S0, np.float64)
    S1 = np.asarray(S1, np.float64)
    c = qg.shape[0]
    nb, ns = S0.shape[0], S1.shape[0]
    pad = ns * fanout - nb
    cm = np.concatenate([cand, np.zeros((c, pad), bool)], 1) if pad else cand
    cand_sup = cm.reshape(c, ns, fanout).any(-1)
    ssc = np.einsum("cd,nmd->cnm", qg, S1).max(-1) * scale
    ssc = np.where(cand_sup, ssc, NEG_INF)
    b_eff = min(beam, ns)
    parents, _ = topk_desc(ssc, b_eff)
    child = (parents[..., None] * fanout + np.arange(fanout)).reshape(c, b_eff * fanout)
    in_range = child < nb
    child = np.clip(child, 0, nb - 1)
    Sg = S0[child]                                               # [c, beam*F, m, dh]
    csc = np.einsum("cd,cjmd->cjm", qg, Sg).max(-1) * scale
    cflat = np.take_along_axis(cand, child, 1) & in_range
    csc = np.where(cflat, csc, NEG_INF)
    kk = min(k, b_eff * fanout)
    sub, val = topk_desc(csc, kk)
    return np.take_along_axis(child, sub, 1), val, ns + b_eff * fanout


# ------------------------------------------------------ union softmax ---------
def union_attention_rows(pos, qc_rows, kc_g, v_g, cos, sin, sel_idx, sel_ok, S, W, Bk, scale, bf16=False):
    """The eval path's inner body for one (batch, KV head), attention.py:676-711:
    one softmax over [sinks (NoPE, j < S, j <= i) | window (RoPE, S <= j <= i,
    j > i - W) | routed blocks (NoPE, the valid picks)].
    pos: [c] query positions; qc_rows: [c, G, dh] QKNorm'd queries;
    kc_g, v_g: [n, dh]; cos/sin: [n_tab, dh]; sel_idx/sel_ok: [c, kk].
    ``bf16``: the RoPE'd window q and k are the bf16 path's rounded operands
    (``apply_rope_bf16``).  Returns (out [c, G, dh], lse [c, G]) in float64
    (natural-log LSE)."""
    rope = apply_rope_bf16 if bf16 else apply_rope
    kc_g = np.asarray(kc_g, np.float64)
    v_g = np.asarray(v_g, np.float64)
    cos = np.asarray(cos, np.float64)
    sin = np.asarray(sin, np.float64)
    c, G, dh = qc_rows.shape
    out = np.zeros((c, G, dh))
    lse = np.zeros((c, G))
    for r in range(c):
        i = int(pos[r])
        q = np.asarray(qc_rows[r], np.float64)                      # [G, dh]
        qr = rope(q, cos[i][None], sin[i][None])
        keys, vals, logits = [], [], []
        ns_ = min(S, i + 1)
        if ns_ > 0:
            logits.append(q @ kc_g[:ns_].T)
            vals.append(v_g[:ns_])
        w0 = max(S, i - W + 1)
        if w0 <= i:
            kw = rope(kc_g[w0:i + 1], cos[w0:i + 1], sin[w0:i + 1])
            logits.append(qr @ kw.T)
            vals.append(v_g[w0:i + 1])
        for b, ok in zip(sel_idx[r], sel_ok[r]):
            if not ok:
                continue
            b = int(b)
            logits.append(q @ kc_g[b * Bk:(b + 1) * Bk].T)
            vals.append(v_g[b * Bk:(b + 1) * Bk])
        lg = np.concatenate(logits, axis=1) * scale                  # [G, keys]
        vv = np.concatenate(vals, axis=0)
        m = lg.max(1, keepdims=True)
        e = np.exp(lg - m)
        l = e.sum(1, keepdims=True)
        out[r] = (e / l) @ vv
        lse[r] = (m + np.log(l))[:, 0]
    return out, lse


def select_rows(pos, qg_rows, S0, S1, cfg, scale, hier):
    """Routed selection for query positions `pos` of one (batch, KV head):
    flat (attention.py:694-698) or hierarchical (:690-693).
    Returns (idx [c, kk], val [c, kk], ok [c, kk])."""
    nb = S0.shape[0]
    cand = route_candidates(pos, cfg["window"], nb, cfg["block"])
    kk = min(cfg["k_blocks"], nb)
    if hier:
        idx, val, _ = hier_select(qg_rows, S0, S1, cfg["fanout"], cfg["beam"], kk, cand, scale)
    else:
        idx, val = flat_select(qg_rows, S0, cand, kk, scale)
    return idx, val, np.isfinite(val)


def eval_forward(q, k, v, cos, sin, cfg, probes, proj, q_gain, k_gain, hier=False,
                 bf16=False, rows=None, summaries=None, supers=None, kc=None, qc=None):
    """`hba_attention_eval` (attention.py:610-713), non-equiv branch, for the
    query positions `rows` (default: all).  q: [B,n,Hq,dh]; k, v: [B,n,Hkv,dh];
    cfg: dict with block, window, sinks, k_blocks, fanout, beam, qknorm,
    content_scale_mode, temp_c, n_cal, native_ctx.  `summaries`/`supers`
    override the summary build (to score the exact stored values).
    Returns dict(out [B,c,Hq,dh], lse [B,Hq,c], idx/val/ok [B,Hkv,c,kk])."""
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    B, n, Hq, dh = q.shape
    Hkv = k.shape[2]
    G = Hq // Hkv
    Bk = cfg["block"]
    assert n % Bk == 0, (n, Bk)
    if cfg["qknorm"]:
        qc = head_rmsnorm(q, q_gain, bf16=bf16) if qc is None else np.asarray(qc, np.float32)
        kc = head_rmsnorm(k, k_gain, bf16=bf16) if kc is None else np.asarray(kc, np.float32)
    else:
        qc, kc = q, k
    scale = union_scale(cfg["qknorm"], cfg.get("content_scale_mode", "inv_d"),
                        cfg.get("temp_c", 0.0), cfg.get("n_cal"), cfg["native_ctx"], dh, n)
    S0 = summarize(kc, probes, proj, Bk) if summaries is None else np.asarray(summaries, np.float64)
    qg = grouped_query(qc, Hkv, bf16=bf16)                            # [B,Hkv,n,dh]
    rows = np.arange(n) if rows is None else np.asarray(rows)
    c = len(rows)
    kk = min(cfg["k_blocks"], n // Bk)
    out = np.zeros((B, c, Hq, dh))
    lse = np.zeros((B, Hq, c))
    idx_all = np.zeros((B, Hkv, c, kk), np.int64)
    val_all = np.zeros((B, Hkv, c, kk))
    ok_all = np.zeros((B, Hkv, c, kk), bool)
    for b in range(B):
        for g in range(Hkv):
            Sh = S0[b, g]
            if hier:
                S1h = build_super(Sh, cfg["fanout"])[0] if supers is None else np.asarray(supers[b, g], np.float64)
            else:
                S1h = None
            idx, val, ok = select_rows(rows, qg[b, g, rows], Sh, S1h, cfg, scale, hier)
            idx_all[b, g], val_all[b, g], ok_all[b, g] = idx, val, ok
            o, ls = union_attention_rows(rows, qc[b, rows, g * G:(g + 1) * G], kc[b, :, g], v[b, :, g],
                                         cos, sin, idx, ok, cfg["sinks"], cfg["window"], Bk, scale, bf16=bf16)
            out[b, :, g * G:(g + 1) * G] = o
            lse[b, g * G:(g + 1) * G] = ls.T
    return dict(out=out, lse=lse, idx=idx_all, val=val_all, ok=ok_all, scale=scale)


def decode(q_rows, kc, v, cos, sin, S0, S1, cfg, scale, q_gain, hier=False, bf16=True,
           qknorm_q=True):
    """One new query per sequence at position i = n-1 over a cached context of
    n tokens: the last row of `hba_attention_eval` (attention.py:663-711 with
    cs = n-1), with the cache holding QKNorm'd keys and the stored summaries.
    q_rows: [B, Hq, dh] raw query; kc, v: [B, n, Hkv, dh]; S0: [B,Hkv,nb,m,dh];
    S1: [B,Hkv,ns,m,dh] or None.  Returns dict(out [B,Hq,dh], lse [B,Hq],
    idx/val/ok [B,Hkv,kk], qc [B,Hq,dh])."""
    q_rows = np.asarray(q_rows, np.float32)
    B, Hq, dh = q_rows.shape
    n = kc.shape[1]
    Hkv = kc.shape[2]
    G = Hq // Hkv
    i = n - 1
    qc = head_rmsnorm(q_rows, q_gain, bf16=bf16) if qknorm_q else q_rows
    qg = grouped_query(qc[:, None], Hkv, bf16=bf16)[:, :, 0]         # [B, Hkv, dh]
    nb = S0.shape[2]
    kk = min(cfg["k_blocks"], n // cfg["block"])
    out = np.zeros((B, Hq, dh))
    lse = np.zeros((B, Hq))
    idx_all = np.zeros((B, Hkv, kk), np.int64)
    val_all = np.zeros((B, Hkv, kk))
    ok_all = np.zeros((B, Hkv, kk), bool)
    pos = np.array([i])
    for b in range(B):
        for g in range(Hkv):
            S1h = None if S1 is None else S1[b, g]
            idx, val, ok = select_rows(pos, qg[b, g][None], S0[b, g, :nb], S1h, cfg, scale, hier)
            idx_all[b, g], val_all[b, g], ok_all[b, g] = idx[0], val[0], ok[0]
            o, ls = union_attention_rows(pos, qc[b, g * G:(g + 1) * G][None], kc[b, :, g], v[b, :, g],
                                         cos, sin, idx, ok, cfg["sinks"], cfg["window"], cfg["block"], scale,
                                         bf16=bf16)
            out[b, g * G:(g + 1) * G] = o[0]
            lse[b, g * G:(g + 1) * G] = ls[0]
    return dict(out=out, lse=lse, idx=idx_all, val=val_all, ok=ok_all, qc=qc)


def selection_parity(idx_a, val_a, ok_a, idx_b, val_b, ok_b, tie=1e-6, tie_rel=0.0):
    """Compare two pick lists of one query (any order).  Picks must agree as
    sets of valid block indices, except that a pick present in only one list
    is excused when its score lies within `tie` (plus `tie_rel` times the
    boundary's magnitude) of the other list's boundary (the smallest valid
    score), i.e. a top-k tie.  Returns (ok, detail)."""
    A = {int(i): float(v) for i, v, o in zip(idx_a, val_a, ok_a) if o}
    Bs = {int(i): float(v) for i, v, o in zip(idx_b, val_b, ok_b) if o}
    if len(A) != len(Bs):
        return False, f"valid pick count {len(A)} != {len(Bs)}"
    only_a = set(A) - set(Bs)
    only_b = set(Bs) - set(A)
    if not only_a:
        return True, ""
    ba = min(A.values())
    bb = min(Bs.values())
    for i in only_a:
        if abs(A[i] - bb) > tie + tie_rel * abs(bb):
            return False, f"block {i} score {A[i]!r} only in first list (boundary {bb!r})"
    for i in only_b:
        if abs(Bs[i] - ba) > tie + tie_rel * abs(ba):
            return False, f"block {i} score {Bs[i]!r} only in second list (boundary {ba!r})"
    return True, "tie"


# ------------------------------------------------------------ backward --------
def rope_backward(dy, cos_rows, sin_rows):
    """Transpose of ``apply_rope`` (attention.py:40-44): y = x*cos +
    rot_half(x)*sin with rot_half's matrix R antisymmetric, so dx = dy*cos -
    rot_half(dy*sin)."""
    dy = np.asarray(dy, np.float64)
    return dy * cos_rows - rot_half(dy * sin_rows)


def head_rmsnorm_backward(x, gain, dy, eps=1e-6):
    """Gradient of ``_HeadRMSNorm.forward`` (attention.py:88-94) w.r.t. its
    input and its per-head scalar gain.  With u = x / rms, rms = sqrt(max(
    mean(x^2), eps)): dx = (g / rms) * (dy - u * mean(dy * u)) where the mean
    is not clamped, dx = (g / rms) * dy where it is (the clamp's gradient is
    zero); dgain[h] = sum over every other axis of dy * u.
    x, dy: [..., H, dh]; gain: [H].  Returns (dx, dgain) in float64."""
    xf = np.asarray(x, np.float64)
    dy = np.asarray(dy, np.float64)
    ms = np.mean(xf * xf, axis=-1, keepdims=True)
    clamped = ms <= eps
    rms = np.sqrt(np.maximum(ms, eps))
    u = xf / rms
    g = np.asarray(gain, np.float64)[:, None]
    proj = np.mean(dy * u, axis=-1, keepdims=True)
    dx = (g / rms) * np.where(clamped, dy, dy - u * proj)
    dgain = (dy * u).sum(axis=-1).reshape(-1, xf.shape[-2]).sum(axis=0)
    return dx, dgain


def union_backward_rows(pos, qc_rows, kc_g, v_g, cos, sin, sel_idx, sel_ok, S, W, Bk, scale, dout_rows,
                        bf16=False, out_rows=None):
    """Gradient of the union softmax of ``union_attention_rows`` (the eval
    body attention.py:676-711, equal to the dense / fused training paths,
    :306-389 and :552-607) for one (batch, KV head), the selection held
    fixed (a top-k has no gradient).  Per query row: P = softmax(scale *
    logits) over [sinks | window | routed], dP = dout . v, dlogit = P *
    (dP - sum(P * dP)); the NoPE parts go to q and the keys directly, the
    window's through the transpose of RoPE at each position.
    Returns (dqc_rows [c, G, dh], dkc_g [n, dh], dv_g [n, dh]) in float64:
    gradients w.r.t. the QKNorm'd q and k (before RoPE) and v."""
    rope = apply_rope_bf16 if bf16 else apply_rope
    kc_g = np.asarray(kc_g, np.float64)
    v_g = np.asarray(v_g, np.float64)
    cos = np.asarray(cos, np.float64)
    sin = np.asarray(sin, np.float64)
    c, G, dh = qc_rows.shape
    n = kc_g.shape[0]
    dq = np.zeros((c, G, dh))
    dk = np.zeros((n, dh))
    dkr = np.zeros((n, dh))   # window keys: gradient w.r.t. the RoPE'd key, rotated back at the end
    dv = np.zeros((n, dh))
    for r in range(c):
        i = int(pos[r])
        q = np.asarray(qc_rows[r], np.float64)                      # [G, dh]
        qr = rope(q, cos[i][None], sin[i][None])
        do = np.asarray(dout_rows[r], np.float64)                   # [G, dh]
        parts = []                                                  # (key rows, RoPE'd?)
        ns_ = min(S, i + 1)
        if ns_ > 0:
            parts.append((np.arange(ns_), False))
        w0 = max(S, i - W + 1)
        if w0 <= i:
            parts.append((np.arange(w0, i + 1), True))
        for b, ok in zip(sel_idx[r], sel_ok[r]):
            if ok:
                parts.append((np.arange(int(b) * Bk, (int(b) + 1) * Bk), False))
        keys = []
        for rows_, rot in parts:
            keys.append(rope(kc_g[rows_], cos[rows_], sin[rows_]) if rot else kc_g[rows_])
        lg = np.concatenate([(qr if rot else q) @ kk.T for (rows_, rot), kk in zip(parts, keys)], axis=1) * scale
        m = lg.max(1, keepdims=True)
        p = np.exp(lg - m)
        p /= p.sum(1, keepdims=True)                                # [G, keys]
        idx = np.concatenate([rows_ for rows_, _ in parts])
        dp = do @ v_g[idx].T
        # D = sum_keys P dP = dout . out; from the stored output when given (a
        # bf16 path computes it from its rounded output)
        dd = (p * dp).sum(1, keepdims=True) if out_rows is None else \
            (do * np.asarray(out_rows[r], np.float64)).sum(1, keepdims=True)
        ds = p * (dp - dd) * scale
        np.add.at(dv, idx, p.T @ do)
        at = 0
        dqr = np.zeros((G, dh))
        for (rows_, rot), kk in zip(parts, keys):
            blk = ds[:, at:at + len(rows_)]
            at += len(rows_)
            if rot:
                dqr += blk @ kk
                np.add.at(dkr, rows_, blk.T @ qr)
            else:
                dq[r] += blk @ kk
                np.add.at(dk, rows_, blk.T @ q)
        dq[r] += rope_backward(dqr, cos[i][None], sin[i][None])
    dk += rope_backward(dkr, cos[:n], sin[:n])
    return dq, dk, dv


def eval_backward(q, k, v, cos, sin, cfg, probes, proj, q_gain, k_gain, dout, bf16=False, sel=None,
                  d_from_bf16_out=False):
    """Gradients of sum(out * dout) for the forward of ``eval_forward`` (the
    union softmax of attention.py:306-389 / :552-607 / :610-713) w.r.t. q, k,
    v and the QKNorm gains (attention.py:88-94), the block selection held
    fixed.  ``sel`` = (idx, ok) [B, Hkv, n, kk] replaces the oracle's own
    selection (to follow another implementation's picks).
    ``d_from_bf16_out``: each row's D = dout . out from the forward output
    rounded to bf16, as a bf16 path that keeps only its stored output
    computes it (exact: sum_keys P dP).  With sharply peaked rows (trained
    QKNorm gains) dP - D cancels on the dominant key and this rounding
    dominates the difference between the two.
    Returns dict(dq, dk, dv [input shapes], dq_gain [Hq], dk_gain [Hkv], plus
    the forward's out / lse / idx / ok)."""
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    v = np.asarray(v, np.float32)
    B, n, Hq, dh = q.shape
    Hkv = k.shape[2]
    G = Hq // Hkv
    fwd = eval_forward(q, k, v, cos, sin, cfg, probes, proj, q_gain, k_gain, bf16=bf16)
    idx_all, ok_all = (fwd["idx"], fwd["ok"]) if sel is None else (np.asarray(sel[0]), np.asarray(sel[1]))
    if cfg["qknorm"]:
        qc = head_rmsnorm(q, q_gain, bf16=bf16)
        kc = head_rmsnorm(k, k_gain, bf16=bf16)
    else:
        qc, kc = q, k
    scale = fwd["scale"]
    pos = np.arange(n)
    dqc = np.zeros((B, n, Hq, dh))
    dkc = np.zeros((B, n, Hkv, dh))
    dv = np.zeros((B, n, Hkv, dh))
    out, lse = fwd["out"], fwd["lse"]
    if sel is not None:  # the forward of the given picks
        out, lse = np.zeros_like(out), np.zeros_like(lse)
    dout = np.asarray(dout, np.float64)
    for b in range(B):
        for g in range(Hkv):
            if sel is not None:
                o, ls = union_attention_rows(pos, qc[b, :, g * G:(g + 1) * G], kc[b, :, g], v[b, :, g], cos, sin,
                                             idx_all[b, g], ok_all[b, g], cfg["sinks"], cfg["window"], cfg["block"],
                                             scale, bf16=bf16)
                out[b, :, g * G:(g + 1) * G] = o
                lse[b, g * G:(g + 1) * G] = ls.T
            o_rows = round_bf16(out[b, :, g * G:(g + 1) * G]) if d_from_bf16_out else None
            dq_, dk_, dv_ = union_backward_rows(pos, qc[b, :, g * G:(g + 1) * G], kc[b, :, g], v[b, :, g], cos, sin,
                                                idx_all[b, g], ok_all[b, g], cfg["sinks"], cfg["window"],
                                                cfg["block"], scale, dout[b, :, g * G:(g + 1) * G], bf16=bf16,
                                                out_rows=o_rows)
            dqc[b, :, g * G:(g + 1) * G] = dq_
            dkc[b, :, g] = dk_
            dv[b, :, g] = dv_
    if cfg["qknorm"]:
        dq, dqg = head_rmsnorm_backward(q, q_gain, dqc)
        dk, dkg = head_rmsnorm_backward(k, k_gain, dkc)
    else:
        dq, dk = dqc, dkc
        dqg, dkg = np.zeros(Hq), np.zeros(Hkv)
    return dict(dq=dq, dk=dk, dv=dv, dq_gain=dqg, dk_gain=dkg, dqc=dqc, dkc=dkc, out=out, lse=lse,
                idx=idx_all, ok=ok_all)


# ---------------------------------------------------------- aux-KL teacher ----
def aux_teacher(qc, kc, cfg, scale):
    """The summarizer's auxiliary-loss teacher (attention.py:476-490,
    `_teacher_chunk`, as `_aux_kl_chunked` :501-529 calls it; the same
    distribution as `hba_attention_dense`'s :364-369): per query i and KV
    head, the mean over the group's G heads of each candidate block's share
    of the softmax over all candidate keys (NoPE logits scale * qc . kc;
    softmax over blockwise LSEs == softmax over keys summed per block),
    renormalised over blocks.  qc: [B, n, Hq, dh]; kc: [B, n, Hkv, dh].
    Returns pstar [B, Hkv, n, nb] (float64); rows with no candidate block
    are NaN, as in the reference (its loss skips them)."""
    qc = np.asarray(qc, np.float64)
    kc = np.asarray(kc, np.float64)
    B, n, Hq, dh = qc.shape
    Hkv = kc.shape[2]
    G = Hq // Hkv
    Bk = cfg["block"]
    nb = n // Bk
    cand = route_candidates(np.arange(n), cfg["window"], nb, Bk)               # [n, nb]
    pstar = np.zeros((B, Hkv, n, nb))
    for b in range(B):
        for g in range(Hkv):
            pstar[b, g] = aux_teacher_rows(np.arange(n), qc[b, :, g * G:(g + 1) * G], kc[b, :, g], cfg, scale)
    return pstar


def aux_teacher_rows(pos, qc_rows, kc_g, cfg, scale):
    """``aux_teacher`` for the query positions `pos` of one (batch, KV
    head): qc_rows [c, G, dh], kc_g [n, dh] -> pstar rows [c, nb]."""
    qc_rows = np.asarray(qc_rows, np.float64)
    kc_g = np.asarray(kc_g, np.float64)
    c, G, dh = qc_rows.shape
    n = kc_g.shape[0]
    Bk = cfg["block"]
    nb = n // Bk
    cand = route_candidates(pos, cfg["window"], nb, Bk)                          # [c, nb]
    with np.errstate(invalid="ignore", divide="ignore"):
        s = np.einsum("ihd,jd->hij", qc_rows, kc_g) * scale                      # [G, c, n]
        s = s.reshape(G, c, nb, Bk)
        m = s.max(-1)
        blk = m + np.log(np.exp(s - m[..., None]).sum(-1))                       # [G, c, nb]
        blk = np.where(cand[None], blk, -np.inf)
        mx = blk.max(-1, keepdims=True)
        e = np.exp(blk - mx)
        p = (e / e.sum(-1, keepdims=True)).mean(0)                                # [c, nb]
        return p / np.maximum(p.sum(-1, keepdims=True), 1e-9)


def aux_kl(pstar, bsc, cand):
    """attention.py:531-537: -mean over (batch, KV head, query with a
    candidate) of sum_blocks pstar * log_softmax(bsc) (terms with pstar = 0
    dropped).  pstar, bsc: [B, Hkv, n, nb]; cand: [n, nb]."""
    vq = np.asarray(cand).any(-1)
    if not vq.any():
        return 0.0
    bv = np.asarray(bsc, np.float64)[:, :, vq]
    pv = np.asarray(pstar, np.float64)[:, :, vq]
    mx = bv.max(-1, keepdims=True)
    logp = bv - mx - np.log(np.exp(bv - mx).sum(-1, keepdims=True))
    term = np.where(pv > 0, pv * np.where(np.isfinite(logp), logp, 0.0), 0.0)
    return float(-term.sum(-1).mean())
