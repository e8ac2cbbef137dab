"""Helpers shared by the GPU parity tests: run the CUDA path through the
C-ABI wrappers, run the oracle on the exact stored bf16 values, compare."""

import math

import numpy as np
import torch

from hba_b200 import HBADecodeCache, hba_attention_b200, synth
from hba_b200.config import HBAConfig
from hba_b200.ops import build_super_b200, qknorm_b200, summarize_b200
from oracle import hba_oracle as orc

OUT_TOL = 2e-2    # max |out - oracle| in bf16
LSE_TOL = 1e-3    # max |lse - oracle| (natural log)
TIE = 1e-6        # selection picks may differ only inside a 1e-6-logit tie
# With trained QKNorm gains the routing scores reach the hundreds, where one
# float32 ulp is ~1e-5: the kernels' fp32 sums (exact bf16 products) and the
# oracle's float64 sums then resolve near-ties differently below ~1e-6
# relative, so those tests widen the tie by 1e-6 of the score's magnitude.
TIE_REL_TRAINED = 1e-6


def np32(t):
    return t.detach().float().cpu().numpy()


def cfg_of(**kw):
    base = dict(n_heads=14, n_kv=2, head_dim=64, block=64, window=1024, sinks=4, k_blocks=16, slots=4, fanout=16,
                beam=4, native_ctx=32768, qknorm=True, content_scale_mode="inv_d", temp_c=0.1, n_cal=None)
    base.update(kw)
    return HBAConfig(**base)


def oracle_cfg(cfg):
    return dict(block=cfg.block, window=cfg.window, sinks=cfg.sinks, k_blocks=cfg.k_blocks, fanout=cfg.fanout,
                beam=cfg.beam, qknorm=cfg.qknorm, content_scale_mode=cfg.content_scale_mode, temp_c=cfg.temp_c,
                n_cal=cfg.n_cal, native_ctx=cfg.native_ctx)


def scale_of(cfg, n):
    return orc.union_scale(cfg.qknorm, cfg.content_scale_mode, cfg.temp_c, cfg.n_cal, cfg.native_ctx, cfg.head_dim, n)


def compare_selection(k_idx, k_sc, o_idx, o_val, o_ok, where, tie_rel=0.0):
    ok, why = orc.selection_parity(k_idx, k_sc, k_idx >= 0, o_idx, o_val, o_ok, tie=TIE, tie_rel=tie_rel)
    assert ok, f"{where}: {why}; kernel {list(k_idx)} oracle {list(o_idx[o_ok])}"
    common = [i for i in k_idx if i >= 0 and i in set(o_idx[o_ok].tolist())]
    kd = {int(i): float(s) for i, s in zip(k_idx, k_sc) if i >= 0}
    od = {int(i): float(s) for i, s, o in zip(o_idx, o_val, o_ok) if o}
    for i in common:
        assert abs(kd[i] - od[i]) <= 1e-5 * max(1.0, abs(od[i])), (where, i, kd[i], od[i])


def assert_picks_agree(si_a, ss_a, si_b, ss_b, tie=TIE, tie_rel=1e-6, score_rel=1e-5):
    """Two kernels' pick lists [..., k] (e.g. the tensor-core selection GEMM
    against the CUDA-core scan, whose fp32 summation orders differ): the same
    sets except inside a tie, and the common picks' scores within score_rel."""
    a_i, a_s = si_a.reshape(-1, si_a.shape[-1]).cpu().numpy(), np32(ss_a).reshape(-1, ss_a.shape[-1])
    b_i, b_s = si_b.reshape(-1, si_b.shape[-1]).cpu().numpy(), np32(ss_b).reshape(-1, ss_b.shape[-1])
    for r in range(a_i.shape[0]):
        ok, why = orc.selection_parity(a_i[r], a_s[r], a_i[r] >= 0, b_i[r], b_s[r], b_i[r] >= 0, tie=tie,
                                       tie_rel=tie_rel)
        assert ok, f"row {r}: {why}"
        da = {int(i): float(x) for i, x in zip(a_i[r], a_s[r]) if i >= 0}
        for i, x in zip(b_i[r], b_s[r]):
            if i >= 0 and int(i) in da:
                assert abs(da[int(i)] - float(x)) <= score_rel * max(1.0, abs(float(x))), (r, i, da[int(i)], x)


def build_cache(cfg, B, n, hier, seed, gains=True, planted=8):
    summ, qkn = synth.make_weights(cfg, "cuda", seed=seed, gains=gains)
    n_cap = -(-n // cfg.block) * cfg.block
    cos, sin = synth.rope_tables(max(n_cap, 1), cfg.head_dim, 1e6)
    wl = synth.decode_workload(cfg, B, n, hier=hier, seed=seed, qkn=qkn, planted=planted)
    cache = HBADecodeCache(cfg, B, n_cap, summ, qkn, cos, sin, hier=hier)
    cache.append(wl["k"], wl["v"])
    return cache, wl, summ, qkn, cos, sin


def check_decode(cache, q, cfg, hier, qkn, cos, sin, rows=None, lens=None, tie_rel=0.0):
    """Decode through the C-ABI and compare every sequence in `rows` with the
    oracle on the cache's stored values.  Returns (max out err, max lse err)."""
    out, lse, (si, ss) = cache.attend(q, return_lse=True, return_selection=True)
    torch.cuda.synchronize()
    qc = np32(qknorm_b200(q, qkn.q.gain)) if cfg.qknorm else np32(q)
    lens = cache.lens_host if lens is None else lens
    rows = range(cache.B) if rows is None else rows
    cosn, sinn = np32(cos), np32(sin)
    out_n, lse_n, si_n, ss_n = np32(out), np32(lse), si.cpu().numpy(), np32(ss)
    worst_o = worst_l = 0.0
    for b in rows:
        n_b = int(lens[b])
        nb = n_b // cfg.block
        kc = np32(cache.tokens("k")[b:b + 1, :n_b])
        v = np32(cache.tokens("v")[b:b + 1, :n_b])
        S0 = np32(cache.summaries[b:b + 1, :, :nb])
        S1 = np32(cache.supers[b:b + 1, :, :-(-nb // cfg.fanout)]) if hier else None
        res = orc.decode(qc[b:b + 1], kc, v, cosn, sinn, S0, S1, oracle_cfg(cfg), scale_of(cfg, n_b), None,
                         hier=hier, bf16=True, qknorm_q=False)
        for g in range(cfg.n_kv):
            compare_selection(si_n[b, g], ss_n[b, g], res["idx"][0, g], res["val"][0, g], res["ok"][0, g],
                              f"b={b} g={g} n={n_b}", tie_rel=tie_rel)
        worst_o = max(worst_o, float(np.abs(out_n[b] - res["out"][0]).max()))
        worst_l = max(worst_l, float(np.abs(lse_n[b] - res["lse"][0]).max()))
    assert worst_o <= OUT_TOL, worst_o
    assert worst_l <= LSE_TOL, worst_l
    assert cache.device_status() == 0  # no bounded wait expired
    assert np.isfinite(out_n).all() and np.isfinite(lse_n).all()
    return worst_o, worst_l, (si, ss)


def check_prefill(cfg, B, n, hier, seed, rows, gains=True, qkv=None, tie_rel=0.0):
    summ, qkn = synth.make_weights(cfg, "cuda", seed=seed, gains=gains)
    cos, sin = synth.rope_tables(n, cfg.head_dim, 1e6)
    if qkv is None:
        wl = synth.prefill_workload(cfg, B, n, seed=seed)
        q, k, v = wl["q"], wl["k"], wl["v"]
    else:
        q, k, v = qkv
    with torch.no_grad():
        out, lse, (si, ss) = hba_attention_b200(q, k, v, cos, sin, cfg, summ, qkn, hier=hier, return_lse=True,
                                                return_selection=True)
        if cfg.qknorm:
            qc, kc = qknorm_b200(q, qkn.q.gain), qknorm_b200(k, qkn.k.gain)
        else:
            qc, kc = q, k
        S0 = summarize_b200(kc, summ.probes, summ.proj, cfg)
        S1 = build_super_b200(S0, cfg)[0] if hier else None
    torch.cuda.synchronize()
    rows = np.asarray(rows)
    res = orc.eval_forward(np32(q), np32(k), np32(v), np32(cos), np32(sin), oracle_cfg(cfg), np32(summ.probes),
                           np32(summ.proj), np32(qkn.q.gain), np32(qkn.k.gain), hier=hier, bf16=True, rows=rows,
                           summaries=np32(S0), supers=None if S1 is None else np32(S1), kc=np32(kc), qc=np32(qc))
    si_n, ss_n = si.cpu().numpy(), np32(ss)
    for b in range(B):
        for g in range(cfg.n_kv):
            for r, row in enumerate(rows):
                compare_selection(si_n[b, g, row], ss_n[b, g, row], res["idx"][b, g, r], res["val"][b, g, r],
                                  res["ok"][b, g, r], f"b={b} g={g} row={row}", tie_rel=tie_rel)
    assert np.isfinite(np32(out)).all() and np.isfinite(np32(lse)[:, :, rows]).all()
    eo = float(np.abs(np32(out)[:, rows] - res["out"]).max())
    el = float(np.abs(np32(lse)[:, :, rows] - res["lse"]).max())
    assert eo <= OUT_TOL, eo
    assert el <= LSE_TOL, el
    return eo, el, out, lse, (si, ss)


def sample_rows(n, count, seed=0):
    r = np.random.default_rng(seed)
    fixed = [0, 1, 2, 3, min(n - 1, 1023), min(n - 1, 1024), min(n - 1, 1200), n - 1]
    return np.unique(np.concatenate([fixed, r.choice(n, size=min(n, count), replace=False)]))
