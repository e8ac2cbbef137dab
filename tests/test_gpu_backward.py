"""Backward of the prefill union softmax on the GPU (hba_b200_prefill_backward,
through ``hba_attention_b200_fused`` and torch autograd) against the
oracle's backward (oracle/hba_oracle.py ``eval_backward``, pinned to the
reference's dense-path autograd by tests/test_oracle_golden.py), fed the
GPU's own block selection and the bf16 operands the kernels consume.

Tolerance (bf16 storage: P and dS enter the MMAs as bf16, D comes from the
bf16 output): per gradient tensor, max |gpu - oracle| <= 3e-2 max |oracle|
and ||gpu - oracle|| <= 1.5e-2 ||oracle||; the QKNorm gains' gradients
within 2e-2 relative."""

import numpy as np
import pytest
import torch

import gpu_helpers as H
from hba_b200 import hba_attention_b200_fused, synth
from oracle import hba_oracle as orc

pytestmark = pytest.mark.gpu

MAX_REL = 3e-2
NORM_REL = 1.5e-2
GAIN_REL = 2e-2


def _close(name, got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert np.isfinite(got).all(), f"{name}: non-finite values"
    scale = max(np.abs(ref).max(), 1e-12)
    err = np.abs(got - ref).max()
    nrm = np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-12)
    assert err <= MAX_REL * scale, f"{name}: max err {err:.3e} vs max |ref| {scale:.3e}"
    assert nrm <= NORM_REL, f"{name}: relative norm err {nrm:.3e}"


def run_backward(cfg, B, n, seed, gains=True):
    cfg.aux_w = 0.0  # the attention's gradients alone (the aux-KL has its own tests)
    summ, qkn = synth.make_weights(cfg, "cuda", seed=seed, gains=gains)
    cos, sin = synth.rope_tables(n, cfg.head_dim, 1e6)
    wl = synth.prefill_workload(cfg, B, n, seed=seed)
    q = wl["q"].clone().requires_grad_(True)
    k = wl["k"].clone().requires_grad_(True)
    v = wl["v"].clone().requires_grad_(True)
    qg = qkn.q.gain.clone().requires_grad_(True)
    kg = qkn.k.gain.clone().requires_grad_(True)

    class _QKN:
        pass

    qk = _QKN()
    qk.q = type("G", (), {"gain": qg})()
    qk.k = type("G", (), {"gain": kg})()
    out, aux = hba_attention_b200_fused(q, k, v, cos, sin, cfg, summ, qk)
    assert float(aux) == 0.0
    g = torch.Generator(device="cpu").manual_seed(seed + 7)
    dout = torch.randn(out.shape, generator=g).to(out.device, out.dtype)
    out.backward(dout)
    torch.cuda.synchronize()
    from hba_b200 import _lib
    assert b"prefill_bwd_kernel" in _lib.load().hba_b200_last_kernels()
    # the forward's picks, for the oracle to follow
    with torch.no_grad():
        from hba_b200 import hba_attention_b200
        _, _, (si, _) = hba_attention_b200(wl["q"], wl["k"], wl["v"], cos, sin, cfg, summ, qkn, return_lse=True,
                                           return_selection=True)
    sel = si.cpu().numpy()
    ref = orc.eval_backward(H.np32(wl["q"]), H.np32(wl["k"]), H.np32(wl["v"]), H.np32(cos), H.np32(sin),
                            H.oracle_cfg(cfg), H.np32(summ.probes), H.np32(summ.proj), H.np32(qkn.q.gain),
                            H.np32(qkn.k.gain), H.np32(dout), bf16=True, sel=(np.maximum(sel, 0), sel >= 0))
    return dict(dq=H.np32(q.grad), dk=H.np32(k.grad), dv=H.np32(v.grad), dqg=H.np32(qg.grad) if cfg.qknorm else None,
                dkg=H.np32(kg.grad) if cfg.qknorm else None, out=H.np32(out)), ref


CASES = [
    # name, config, batch, n
    ("g4_d64", dict(n_heads=8, n_kv=2, head_dim=64, window=256, k_blocks=4), 1, 1024),
    ("g4_d128", dict(n_heads=16, n_kv=4, head_dim=128, window=256, k_blocks=8), 2, 1024),
    ("g7_d64_rows126", dict(n_heads=14, n_kv=2, head_dim=64, window=512, k_blocks=8), 1, 1024),
    ("g8_d128", dict(n_heads=16, n_kv=2, head_dim=128, window=128, k_blocks=4), 1, 768),
    ("noqk_d64", dict(n_heads=8, n_kv=2, head_dim=64, window=256, k_blocks=4, qknorm=False), 1, 1024),
]


@pytest.mark.parametrize("name,kw,B,n", CASES, ids=[c[0] for c in CASES])
def test_backward_matches_oracle(name, kw, B, n):
    cfg = H.cfg_of(**kw)
    got, ref = run_backward(cfg, B, n, seed=40 + len(name))
    assert np.abs(got["out"] - ref["out"]).max() <= H.OUT_TOL
    for key in ("dq", "dk", "dv"):
        _close(f"{name} {key}", got[key], ref[key])
    if cfg.qknorm:
        np.testing.assert_allclose(got["dqg"], ref["dq_gain"], rtol=GAIN_REL, atol=GAIN_REL * np.abs(ref["dq_gain"]).max())
        np.testing.assert_allclose(got["dkg"], ref["dk_gain"], rtol=GAIN_REL, atol=GAIN_REL * np.abs(ref["dk_gain"]).max())


def test_backward_short_sequence_no_routed():
    """n < W: sinks and window only (no routed candidates), one NoPE chunk per tile."""
    cfg = H.cfg_of(n_heads=8, n_kv=2, head_dim=64, window=1024, k_blocks=4)
    got, ref = run_backward(cfg, 1, 512, seed=61)
    for key in ("dq", "dk", "dv"):
        _close(f"short {key}", got[key], ref[key])


def test_backward_replays_reference_fixture():
    """The reference's own gradients (fp32 autograd through its dense
    training path, tests/golden/bwd_g4d64_qk.npz) against the GPU backward on
    the same (bf16-valued) inputs.  The GPU keeps QKNorm's outputs in bf16
    where the reference's fp32 run does not, so the bound is wider than
    against the bf16 oracle: max err <= 5e-2 max |ref|, norm err <= 3e-2,
    gains 3e-2.  The fixture's picks are the same under bf16 and fp32
    (checked on the CPU when the fixture was made)."""
    import os
    import cases
    name, c, n, seed, qk = [x for x in cases.BWD_CASES if x[0] == "g4d64_qk"][0]
    gold = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", f"bwd_{name}.npz"))
    inp = cases.bwd_case_inputs(c, n, seed)
    cfg = H.cfg_of(**{k_: c[k_] for k_ in ("n_heads", "n_kv", "head_dim", "block", "window", "sinks", "k_blocks",
                                           "slots", "fanout", "beam", "native_ctx", "content_scale_mode", "temp_c",
                                           "n_cal")}, qknorm=qk, aux_w=0.0)
    dev = "cuda"
    t = lambda a, dt=torch.bfloat16: torch.from_numpy(np.ascontiguousarray(a)).to(dev, dt)  # noqa: E731
    q, k, v = (t(inp[x]).requires_grad_(True) for x in ("q", "k", "v"))
    qg, kg = (t(inp[x], torch.float32).requires_grad_(True) for x in ("q_gain", "k_gain"))
    summ = type("S", (), {"probes": t(inp["probes"], torch.float32), "proj": t(inp["proj"], torch.float32)})()
    qkn = type("Q", (), {})()
    qkn.q = type("G", (), {"gain": qg})()
    qkn.k = type("G", (), {"gain": kg})()
    cos, sin = orc.rope_tables(n, c["head_dim"], c["rope_theta"])
    out, _ = hba_attention_b200_fused(q, k, v, t(cos, torch.float32), t(sin, torch.float32), cfg, summ, qkn)
    out.backward(t(inp["dout"]))
    torch.cuda.synchronize()
    qr, kr = gold["qrows"], gold["krows"]
    for key, got, rows in (("dq", q.grad, qr), ("dk", k.grad, kr), ("dv", v.grad, kr)):
        g_ = H.np32(got)[:, rows].astype(np.float64)
        ref = gold[key].astype(np.float64)
        scale = np.abs(ref).max()
        assert np.isfinite(g_).all()
        assert np.abs(g_ - ref).max() <= 5e-2 * scale, (key, np.abs(g_ - ref).max(), scale)
        assert np.linalg.norm(g_ - ref) <= 3e-2 * np.linalg.norm(ref), key
    for key, got in (("dq_gain", qg.grad), ("dk_gain", kg.grad)):
        ref = gold[key].astype(np.float64)
        np.testing.assert_allclose(H.np32(got), ref, rtol=3e-2, atol=3e-2 * np.abs(ref).max())


def _gain_bound(x, dqc, rel):
    """Per head, rel x sum over rows and columns of |dy u| (u = x / rms): the
    error bound of a sum whose terms cancel.  With trained gains the gains'
    gradients are such sums: on the model layer below the terms' magnitudes
    add up to ~2500 per head against results of ~3, and one bf16 rounding of
    the forward output (through D) moves the results by up to 0.4."""
    xf = np.asarray(x, np.float64)
    u = xf / np.sqrt(np.maximum((xf * xf).mean(-1, keepdims=True), 1e-6))
    return rel * np.abs(dqc * u).sum(axis=-1).reshape(-1, xf.shape[-2]).sum(axis=0)


def test_backward_reference_model_layer_trained_gains():
    """Layer 0 of the reference's own HBAModel (tests/golden/model_layer.npz:
    the q / k / v its block_fn hands to the attention, QKNorm gains from the
    reference's init_qknorm_gains, gain_q * gain_k ~ 81, so the union softmax
    is sharply peaked): the GPU backward against the oracle's (the GPU's
    picks, D from the bf16 output as the kernels compute it).  dq / dk / dv
    within the tolerances above; the gains' gradients within 1e-3 of the sum
    of their terms' magnitudes (``_gain_bound``; errors of ~2e-4 of it were
    seen)."""
    import model_fixture as M
    d = M.load()
    c = d["cfg"]
    cfg = H.cfg_of(**{k_: c[k_] for k_ in ("n_heads", "n_kv", "head_dim", "block", "window", "sinks", "k_blocks",
                                           "slots", "fanout", "beam", "native_ctx", "qknorm", "content_scale_mode",
                                           "temp_c", "n_cal")}, aux_w=0.0)
    n = d["q"].shape[1]
    dev = "cuda"
    t = lambda a, dt=torch.bfloat16: torch.from_numpy(np.ascontiguousarray(a)).to(dev, dt)  # noqa: E731
    q, k, v = (t(d[x]).requires_grad_(True) for x in ("q", "k", "v"))
    qg, kg = (t(d[x], torch.float32).requires_grad_(True) for x in ("q_gain", "k_gain"))
    summ = type("S", (), {"probes": t(d["probes"], torch.float32), "proj": t(d["proj"], torch.float32)})()
    qkn = type("Q", (), {})()
    qkn.q = type("G", (), {"gain": qg})()
    qkn.k = type("G", (), {"gain": kg})()
    cos, sin = synth.rope_tables(n, cfg.head_dim, c["rope_theta"])
    out, _ = hba_attention_b200_fused(q, k, v, cos, sin, cfg, summ, qkn)
    g = torch.Generator(device="cpu").manual_seed(77)
    dout = torch.randn(out.shape, generator=g).to(dev, out.dtype)
    out.backward(dout)
    torch.cuda.synchronize()
    with torch.no_grad():
        from hba_b200 import hba_attention_b200
        _, _, (si, _) = hba_attention_b200(q.detach(), k.detach(), v.detach(), cos, sin, cfg, summ, qkn,
                                           return_lse=True, return_selection=True)
    sel = si.cpu().numpy()
    ref = orc.eval_backward(d["q"], d["k"], d["v"], H.np32(cos), H.np32(sin), M.oracle_cfg(c), d["probes"],
                            d["proj"], d["q_gain"], d["k_gain"], H.np32(dout), bf16=True,
                            sel=(np.maximum(sel, 0), sel >= 0), d_from_bf16_out=True)
    for key, got in (("dq", q.grad), ("dk", k.grad), ("dv", v.grad)):
        _close(f"model layer {key}", H.np32(got), ref[key])
    for key, got, x, dy in (("dq_gain", qg.grad, d["q"], ref["dqc"]), ("dk_gain", kg.grad, d["k"], ref["dkc"])):
        err = np.abs(H.np32(got) - ref[key])
        bound = _gain_bound(x, dy, 1e-3)
        assert (err <= bound).all(), (key, H.np32(got), ref[key], bound)
