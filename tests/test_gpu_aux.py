"""The summarizer's aux-KL on the GPU: the teacher kernel
(hba_b200_aux_teacher) against the oracle's teacher (oracle/hba_oracle.py
``aux_teacher``, pinned to the reference's _teacher_chunk by
tests/test_oracle_golden.py) on the bf16 QKNorm'd operands the kernel reads,
and the whole loss of ``hba_attention_b200_fused`` (aux_w = 1) with its
gradients w.r.t. the summarizer's probes and proj against the reference's
own (tests/golden/aux_*.npz: hba_attention_dense's aux, fp32 autograd).

Tolerances: pstar within 1e-4 + 1e-3 relative (fp32 logits of exact bf16
products; the kernel's sums run in another order); the replayed loss within
1e-2 relative and its gradients within 3e-2 in relative norm (the reference
keeps QKNorm's outputs in fp32 where the device path rounds them to bf16)."""

import os

import numpy as np
import pytest
import torch

import cases
import gpu_helpers as H
from hba_b200 import hba_attention_b200_fused, synth
from hba_b200.attention import aux_teacher_b200, union_scale
from hba_b200.ops import qknorm_b200
from oracle import hba_oracle as orc

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

CASES = [
    # name, config, batch, n
    ("g4_d64", dict(n_heads=8, n_kv=2, head_dim=64, window=256), 1, 1024),
    ("g4_d128", dict(n_heads=16, n_kv=4, head_dim=128, window=256), 2, 1024),
    ("g7_d64_rows126", dict(n_heads=14, n_kv=2, head_dim=64, window=512), 1, 1024),
    ("g1_d64_qt128", dict(n_heads=2, n_kv=2, head_dim=64, window=128), 1, 512),
    ("noqk_d64", dict(n_heads=8, n_kv=2, head_dim=64, window=256, qknorm=False), 1, 1024),
    ("short_no_candidates", dict(n_heads=8, n_kv=2, head_dim=64, window=1024), 1, 512),
    # trained-scale gains: the logits exceed the bound, the kernel takes its two passes
    ("trained_gains_d64", dict(n_heads=8, n_kv=2, head_dim=64, window=256), 1, 1024),
]


@pytest.mark.parametrize("name,kw,B,n", CASES, ids=[c[0] for c in CASES])
def test_aux_teacher_matches_oracle(name, kw, B, n):
    """One pass (QKNorm, bounded logits) and two passes (no QKNorm, trained
    gains) against the oracle on every row."""
    cfg = H.cfg_of(**kw)
    summ, qkn = synth.make_weights(cfg, "cuda", seed=70, gains="trained" if "trained" in name else True)
    cos, sin = synth.rope_tables(n, cfg.head_dim, 1e6)
    wl = synth.prefill_workload(cfg, B, n, seed=70)
    pstar = aux_teacher_b200(wl["q"], wl["k"], cos, sin, cfg, qkn)
    from hba_b200 import _lib
    assert b"aux_teacher_kernel" in _lib.load().hba_b200_last_kernels()
    with torch.no_grad():
        if cfg.qknorm:
            qc, kc = qknorm_b200(wl["q"], qkn.q.gain), qknorm_b200(wl["k"], qkn.k.gain)
        else:
            qc, kc = wl["q"], wl["k"]
    torch.cuda.synchronize()
    ref = orc.aux_teacher(H.np32(qc), H.np32(kc), H.oracle_cfg(cfg), union_scale(cfg, cfg.head_dim, n))
    got = H.np32(pstar)
    cand = orc.route_candidates(np.arange(n), cfg.window, n // cfg.block, cfg.block)
    rows = cand.any(-1)
    assert np.isfinite(got).all()
    assert (got[:, :, ~rows] == 0).all()                     # queries without a candidate: 0 (the reference: NaN)
    assert (got[:, :, :, 0] == 0).all()                      # block 0 is never a candidate
    if rows.any():
        np.testing.assert_allclose(got[:, :, rows], ref[:, :, rows], rtol=1e-3, atol=1e-4)
        np.testing.assert_allclose(got[:, :, rows].sum(-1), 1.0, atol=1e-4)


@pytest.mark.parametrize("name", ["g4d64_qk", "g4d64_noqk"])
def test_aux_kl_replays_reference(name):
    """hba_attention_b200_fused's aux (aux_w = 1) and its gradients w.r.t.
    the summarizer's probes / proj against the reference's dense path."""
    _, c, n, seed, qk = [x for x in cases.AUX_CASES if x[0] == name][0]
    g = np.load(os.path.join(GOLD, f"aux_{name}.npz"))
    inp = cases.bwd_case_inputs(c, n, seed)
    cfg = H.cfg_of(**{k_: c[k_] for k_ in ("n_heads", "n_kv", "head_dim", "block", "window", "sinks", "k_blocks",
                                           "slots", "fanout", "beam", "native_ctx", "content_scale_mode", "temp_c",
                                           "n_cal")}, qknorm=qk, aux_w=1.0)
    dev = "cuda"
    t = lambda a, dt=torch.bfloat16: torch.from_numpy(np.ascontiguousarray(a)).to(dev, dt)  # noqa: E731
    q, k, v = (t(inp[x]) for x in ("q", "k", "v"))
    probes = t(inp["probes"], torch.float32).requires_grad_(True)
    proj = t(inp["proj"], torch.float32).requires_grad_(True)
    summ = type("S", (), {"probes": probes, "proj": proj})()
    qkn = type("Q", (), {})()
    qkn.q = type("G", (), {"gain": t(inp["q_gain"], torch.float32)})()
    qkn.k = type("G", (), {"gain": t(inp["k_gain"], torch.float32)})()
    cos, sin = orc.rope_tables(n, c["head_dim"], c["rope_theta"])
    _, aux = hba_attention_b200_fused(q, k, v, t(cos, torch.float32), t(sin, torch.float32), cfg, summ, qkn)
    aux.backward()
    torch.cuda.synchronize()
    ref = float(g["aux"])
    a = float(aux.detach())
    assert abs(a - ref) <= 1e-2 * abs(ref), (a, ref)
    for key, got in (("dprobes", probes.grad), ("dproj", proj.grad)):
        gv, rv = H.np32(got).astype(np.float64), g[key].astype(np.float64)
        assert np.isfinite(gv).all()
        assert np.linalg.norm(gv - rv) <= 3e-2 * np.linalg.norm(rv), (key, np.linalg.norm(gv - rv), np.linalg.norm(rv))


def test_aux_teacher_sliced_long_sequence():
    """A 32K sequence at 32/8 heads, dh 128: the single pass's block masses
    ([queries, blocks, heads] fp32) exceed the kernel's scratch, so the
    queries run in slices; sampled rows on both sides of the slice boundary
    and at the end against the oracle's rows."""
    cfg = H.cfg_of(n_heads=32, n_kv=8, head_dim=128)
    n = 32768
    summ, qkn = synth.make_weights(cfg, "cuda", seed=71, gains=True)
    cos, sin = synth.rope_tables(n, 128, 1e6)
    wl = synth.prefill_workload(cfg, 1, n, seed=71)
    pstar = aux_teacher_b200(wl["q"], wl["k"], cos, sin, cfg, qkn)
    with torch.no_grad():
        qc, kc = qknorm_b200(wl["q"], qkn.q.gain), qknorm_b200(wl["k"], qkn.k.gain)
    torch.cuda.synchronize()
    rows = np.array([1200, 8191, 16383, 16384, 16385, 20000, 24575, 24576, 32766, 32767])
    G = 4
    scale = union_scale(cfg, 128, n)
    qcn, kcn, got = H.np32(qc), H.np32(kc), H.np32(pstar)
    for g in (0, 7):
        ref = orc.aux_teacher_rows(rows, qcn[0, rows, g * G:(g + 1) * G], kcn[0, :, g], H.oracle_cfg(cfg), scale)
        np.testing.assert_allclose(got[0, g, rows], ref, rtol=1e-3, atol=1e-4)
