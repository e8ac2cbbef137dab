"""Generate the golden vectors under tests/golden/ by running the REFERENCE
implementation (nealxpatel/hierarchical-block-attention, ``src/hba``) on the
seeded inputs defined in ``cases.py``.

Run it where the reference source is importable:

    HBA_REFERENCE_SRC=/path/to/hierarchical-block-attention/src python tests/golden/make_golden.py

It writes only ``tests/golden/*.npz``.  The test suite never imports the
reference; it checks the numpy oracle (``oracle/hba_oracle.py``) against these
files.
"""

import math
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.join(HERE, "..", ".."))

import cases  # noqa: E402
from oracle import hba_oracle as orc  # noqa: E402  (only for the shared rope tables)

REF_SRC = os.environ.get("HBA_REFERENCE_SRC")
if not REF_SRC or not os.path.isdir(REF_SRC):
    sys.exit("set HBA_REFERENCE_SRC to the reference's src/ directory")
# the reference's config module creates results/data/logs under these paths at import
_tmp = tempfile.mkdtemp(prefix="hba-golden-")
for _k in ("HBA_RESULTS_DIR", "HBA_DATA_DIR", "HBA_LOGS_DIR"):
    os.environ.setdefault(_k, _tmp)
sys.path.insert(0, REF_SRC)

import torch  # noqa: E402

from hba import attention as ref_attn  # noqa: E402
from hba import summarizer as ref_summ  # noqa: E402
from hba.config import HBAConfig  # noqa: E402

torch.set_num_threads(max(1, os.cpu_count() or 1))


def T(a):
    return torch.from_numpy(np.ascontiguousarray(a))


def ref_cfg(c, qknorm, n_layers=1):
    return HBAConfig(n_layers=n_layers, n_heads=c["n_heads"], n_kv=c["n_kv"], head_dim=c["head_dim"],
                     hidden=c["n_heads"] * c["head_dim"], rope_theta=c["rope_theta"],
                     native_ctx=c["native_ctx"], block=c["block"], window=c["window"], sinks=c["sinks"],
                     k_blocks=c["k_blocks"], slots=c["slots"], fanout=c["fanout"], beam=c["beam"],
                     qknorm=qknorm, content_scale_mode=c["content_scale_mode"], temp_c=c["temp_c"],
                     n_cal=c["n_cal"], mem_elem_cap=2e7, attn_backend="naive", aux_w=0.0)


def ref_modules(cfg, inp):
    summ = ref_summ.SlotSummarizer(cfg)
    summ.probes.data.copy_(T(inp["probes"]))
    summ.proj.data.copy_(T(inp["proj"]))
    qkn = ref_attn.QKNorm(cfg)
    qkn.q.gain.data.copy_(T(inp["q_gain"]))
    qkn.k.gain.data.copy_(T(inp["k_gain"]))
    return summ, qkn


def ref_dense_lse(q, k, v, cos, sin, cfg, summ, qkn):
    """Natural-log LSE of the union softmax built from the reference's own
    pieces, following hba_attention_dense (attention.py:324-355) step for step
    (the reference returns no LSE from its dense or eval paths)."""
    B, n, Hq, dh = q.shape
    G = cfg.G
    qc, kc, scale = ref_attn._content_qk(q, k, cfg, qkn, n)
    qr = ref_attn.apply_rope(qc, cos, sin).transpose(1, 2)
    kr = ref_attn.apply_rope(kc, cos, sin).transpose(1, 2).repeat_interleave(G, dim=1)
    nb = n // cfg.block
    qn = qc.transpose(1, 2)
    kn = kc.transpose(1, 2).repeat_interleave(G, dim=1)
    m_sink, m_win, cand = ref_attn._causal_bucket_masks(n, cfg.sinks, cfg.window, nb, cfg.block, q.device)
    sel, _ = ref_attn.route_topk(qc, kc, cfg, summ, cand)
    m_rout = sel.repeat_interleave(G, dim=1).repeat_interleave(cfg.block, dim=-1)
    s_nope = torch.matmul(qn, kn.transpose(-1, -2)) * scale
    s_rope = torch.matmul(qr, kr.transpose(-1, -2)) * scale
    sc = torch.where(m_win[None, None], s_rope, s_nope)
    sc = sc.masked_fill(~(m_rout | (m_sink | m_win)[None, None]), float("-inf"))
    return torch.logsumexp(sc, -1)                                   # [B, Hq, n]


def out(name, **arrays):
    path = os.path.join(HERE, f"{name}.npz")
    np.savez_compressed(path, **arrays)
    print("wrote", path, {k: v.shape for k, v in arrays.items()})


@torch.no_grad()
def main():
    # ---- QKNorm (attention.py:88-94) ----
    r = cases.rng(1)
    x = cases.randn(r, 3, 17, 4, 8, scale=5.0) + 2.0
    gain = r.uniform(0.3, 2.0, 4).astype(np.float32)
    hn = ref_attn._HeadRMSNorm(4)
    hn.gain.data.copy_(T(gain))
    y = hn(T(x)).numpy()
    xb = torch.from_numpy(x).to(torch.bfloat16)
    yb = hn(xb).float().numpy()
    out("qknorm", y=y, y_bf16=yb)

    # ---- scalars (attention.py:123-198) ----
    rows = []
    for mode in ("inv_d", "inv_sqrt_d"):
        for temp_c in (0.0, 0.1, 0.5):
            for n_cal in (None, 4096):
                for native in (8192, 32768):
                    for n in (1, 4096, 8192, 32768, 65536, 131072):
                        for qk in (False, True):
                            c = dict(cases.TINY, content_scale_mode=mode, temp_c=temp_c, n_cal=n_cal,
                                     native_ctx=native, head_dim=64)
                            cfg = ref_cfg(c, qk)
                            tau = ref_attn.log_len_tau(cfg, n)
                            qq = torch.zeros(1, 1, 4, 64)
                            kq = torch.zeros(1, 1, 2, 64)
                            _, _, s = ref_attn._content_qk(qq, kq, cfg, ref_attn.QKNorm(cfg), n)
                            rows.append([["inv_d", "inv_sqrt_d"].index(mode), temp_c, n_cal or 0, native, n,
                                         int(qk), tau, s])
    out("scales", table=np.array(rows, dtype=np.float64))

    # ---- RoPE tables (attention.py:27-32) ----
    c16, s16 = ref_attn.rope_tables(300, 16, 1e6, "cpu")
    c64, s64 = ref_attn.rope_tables(4096, 64, 1e6, "cpu")
    pick = np.array([0, 1, 2, 63, 64, 1000, 2047, 4095])
    out("rope", cos16=c16.numpy(), sin16=s16.numpy(), cos64=c64.numpy()[pick], sin64=s64.numpy()[pick],
        pick64=pick)

    # ---- summaries + supers + selection (summarizer.py:34-54, attention.py:202-246) ----
    c = dict(cases.TINY, head_dim=16)
    cfg = ref_cfg(c, True)
    r = cases.rng(2)
    kc = cases.randn(r, 2, 176, 2, 16)
    probes, proj = cases.summarizer_params(r, 2, 2, 16)
    summ = ref_summ.SlotSummarizer(cfg)
    summ.probes.data.copy_(T(probes))
    summ.proj.data.copy_(T(proj))
    S = summ.summarize(T(kc), 16)                                   # [2,2,11,2,16]
    S0 = S[:, 0]                                                    # [2,11,2,16]
    S1, ns = ref_attn.build_super(S0, 4)
    qn = cases.randn(r, 2, 5, 16)
    pos = np.array([100, 130, 150, 175, 60], dtype=np.int64)
    cand = ref_attn._route_candidates(176, 64, 11, 16, "cpu")[torch.from_numpy(pos)]
    scale = 1.0 / 16
    hidx, hval, ncmp = ref_attn.hier_select(T(qn), S0, S1, 4, 2, 4, cand, scale)
    bsc = ref_summ.slot_block_scores(T(qn)[:, None], S0[:, None], scale)[:, 0]   # [2,5,11]
    bsc = bsc.masked_fill(~cand[None], float("-inf"))
    ftk = bsc.topk(4, dim=-1)
    qfull = cases.randn(r, 2, 7, 8, 16)
    qg = ref_summ.grouped_query(T(qfull), ref_cfg(dict(c, n_heads=8), True)).numpy()
    out("summaries", kc=kc, probes=probes, proj=proj, S=S.numpy(), S1=S1.numpy(), qn=qn, pos=pos,
        hidx=hidx.numpy(), hval=hval.numpy(), ncmp=np.array(ncmp), fidx=ftk.indices.numpy(),
        fval=ftk.values.numpy(), qfull=qfull, qg=qg)

    # ---- full eval forwards (attention.py:610-713) + LSE from the dense path ----
    for case in cases.EVAL_CASES:
        name, c, n, seed, qk, hier, _ = case
        inp = cases.eval_case_inputs(c, n, seed)
        cfg = ref_cfg(c, qk)
        summ, qkn = ref_modules(cfg, inp)
        cos, sin = orc.rope_tables(n, c["head_dim"], c["rope_theta"])
        q, k, v = T(inp["q"]), T(inp["k"]), T(inp["v"])
        o = ref_attn.hba_attention_eval(q, k, v, T(cos), T(sin), cfg, summ, qkn, cfg.mem_elem_cap, hier=hier)
        rws = cases.rows_for(case)
        arrays = dict(out=o.numpy()[:, rws], rows=rws)
        if not hier:
            lse = ref_dense_lse(q, k, v, T(cos), T(sin), cfg, summ, qkn)
            arrays["lse"] = lse.numpy()[:, :, rws]
            od, _ = ref_attn.hba_attention_dense(q, k, v, T(cos), T(sin), cfg, summ, qkn)
            arrays["out_dense"] = od.numpy()[:, rws]
        out(f"eval_{name}", **arrays)


@torch.enable_grad()
def backward_cases():
    """Gradients of sum(out * dout) w.r.t. q, k, v and the QKNorm gains
    through the reference's dense training path (attention.py:306-389),
    fp32 autograd; the selection is a top-k (no gradient)."""
    for name, c, n, seed, qk in cases.BWD_CASES:
        inp = cases.bwd_case_inputs(c, n, seed)
        cfg = ref_cfg(c, qk)
        summ, qkn = ref_modules(cfg, inp)
        cos, sin = orc.rope_tables(n, c["head_dim"], c["rope_theta"])
        q, k, v = (T(inp[x]).clone().requires_grad_(True) for x in ("q", "k", "v"))
        o, _ = ref_attn.hba_attention_dense(q, k, v, T(cos), T(sin), cfg, summ, qkn)
        (o * T(inp["dout"])).sum().backward()
        qrows, krows = cases.bwd_rows(n, seed)
        out(f"bwd_{name}", qrows=qrows, krows=krows, out=o.detach().numpy()[:, qrows], dq=q.grad.numpy()[:, qrows],
            dk=k.grad.numpy()[:, krows], dv=v.grad.numpy()[:, krows],
            dq_gain=qkn.q.gain.grad.numpy() if qk else np.zeros(c["n_heads"], np.float32),
            dk_gain=qkn.k.gain.grad.numpy() if qk else np.zeros(c["n_kv"], np.float32))


def aux_cases():
    """The summarizer's aux-KL pieces from the reference, fp32: the teacher
    pstar as _aux_kl_chunked computes it (attention.py:501-529, calling
    _teacher_chunk :476-490), the block scores route_topk gives the loss
    (:272-303), and hba_attention_dense's aux with its gradients w.r.t. the
    summarizer's probes and proj (aux_w = 1)."""
    for name, c, n, seed, qk in cases.AUX_CASES:
        inp = cases.bwd_case_inputs(c, n, seed)
        cfg = ref_cfg(c, qk)
        cfg.aux_w = 1.0
        summ, qkn = ref_modules(cfg, inp)
        cos, sin = orc.rope_tables(n, c["head_dim"], c["rope_theta"])
        q, k, v = T(inp["q"]), T(inp["k"]), T(inp["v"])
        B, Hq, Hkv, dh, Bk = 1, c["n_heads"], c["n_kv"], c["head_dim"], c["block"]
        G = Hq // Hkv
        nb = n // Bk
        with torch.no_grad():
            qc, kc, _ = ref_attn._content_qk(q, k, cfg, qkn, n)
            scale = (ref_attn.content_scale(cfg, dh) * ref_attn.log_len_tau(cfg, n)) if qk else dh ** -0.5
            cand = ref_attn._route_candidates(n, c["window"], nb, Bk, "cpu")
            qn = qc.view(B, n, Hkv, G, dh).permute(0, 2, 3, 1, 4).contiguous()
            kt = kc.permute(0, 2, 3, 1).unsqueeze(2).contiguous()
            pstar = ref_attn._teacher_chunk(qn, kt, cand, scale, Bk)
            _, bsc = ref_attn.route_topk(qc, kc, cfg, summ, cand)
        with torch.enable_grad():
            _, aux = ref_attn.hba_attention_dense(q, k, v, T(cos), T(sin), cfg, summ, qkn)
            aux.backward()
        out(f"aux_{name}", pstar=pstar.numpy(), bsc=bsc.numpy(), aux=np.array(float(aux)),
            dprobes=summ.probes.grad.numpy(), dproj=summ.proj.grad.numpy())


if __name__ == "__main__":
    main()
    backward_cases()
    aux_cases()
