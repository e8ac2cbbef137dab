"""Pin the numpy oracle to the reference: every function the CUDA path is
checked against is first checked here against vectors that the reference
implementation itself produced (tests/golden/make_golden.py)."""

import math
import os

import numpy as np
import pytest

import cases
from oracle import hba_oracle as orc

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    return np.load(os.path.join(GOLD, f"{name}.npz"))


def test_qknorm_matches_reference_fp32_and_bf16():
    g = load("qknorm")
    r = cases.rng(1)
    x = cases.randn(r, 3, 17, 4, 8, scale=5.0) + 2.0
    gain = r.uniform(0.3, 2.0, 4).astype(np.float32)
    y = orc.head_rmsnorm(x, gain)
    np.testing.assert_allclose(y, g["y"], rtol=2e-6, atol=2e-6)
    xb = orc.round_bf16(x)
    yb = orc.head_rmsnorm(xb, gain, bf16=True)
    # the reference rounds to bf16 exactly once; allow a 1-ulp flip on ties of the fp32 sum order
    ulp = np.abs(g["y_bf16"]) * 2.0 ** -7
    assert (np.abs(yb - g["y_bf16"]) <= ulp + 1e-30).all()
    assert (yb == g["y_bf16"]).mean() > 0.99


def test_qknorm_rms_equals_gain():
    """Reference tests/test_qknorm.py:67-78: after QKNorm the per-head RMS is the gain."""
    r = cases.rng(7)
    x = cases.randn(r, 3, 17, 4, 8, scale=5.0) + 2.0
    gain = r.uniform(0.3, 2.0, 4).astype(np.float32)
    y = orc.head_rmsnorm(x, gain)
    rms = np.sqrt((y.astype(np.float64) ** 2).mean(-1))
    np.testing.assert_allclose(rms, np.broadcast_to(gain, rms.shape), atol=1e-5)


def test_scales_and_temperature_match_reference():
    t = load("scales")["table"]
    for mode_i, temp_c, n_cal, native, n, qk, tau, s in t:
        mode = ["inv_d", "inv_sqrt_d"][int(mode_i)]
        n_cal = int(n_cal) or None
        assert orc.log_len_tau(temp_c, n_cal, int(native), int(n)) == pytest.approx(tau, rel=1e-12)
        assert orc.union_scale(bool(qk), mode, temp_c, n_cal, int(native), 64, int(n)) == pytest.approx(s, rel=1e-12)


def test_tau_closed_forms():
    """Reference tests/test_qknorm.py:123-165."""
    assert orc.log_len_tau(0.1, 32768, 32768, 32768) == 1.0
    assert orc.log_len_tau(0.1, 32768, 32768, 65536) == pytest.approx(1 + 0.1 * math.log(2))
    assert orc.union_scale(True, "inv_d", 0.1, None, 32768, 128, 131072) == pytest.approx(
        (1 / 128) * (1 + 0.1 * math.log(4)))
    assert orc.log_len_tau(0.0, 1, 1, 10 ** 9) == 1.0
    with pytest.raises(ValueError):
        orc.content_scale("bogus", 64)


def test_rope_tables_match_reference():
    g = load("rope")
    c16, s16 = orc.rope_tables(300, 16, 1e6)
    np.testing.assert_allclose(c16, g["cos16"], atol=2e-6)
    np.testing.assert_allclose(s16, g["sin16"], atol=2e-6)
    c64, s64 = orc.rope_tables(4096, 64, 1e6)
    # numpy's float32 pow may differ from torch's by an ulp in theta^(-2i/d); the
    # angle error grows with position (the CUDA path takes the tables as inputs)
    np.testing.assert_allclose(c64[g["pick64"]], g["cos64"], atol=2e-5)
    np.testing.assert_allclose(s64[g["pick64"]], g["sin64"], atol=2e-5)


def test_summaries_supers_and_selection_match_reference():
    g = load("summaries")
    S = orc.summarize(g["kc"], g["probes"], g["proj"], 16)
    np.testing.assert_allclose(S, g["S"], rtol=1e-5, atol=1e-5)
    S1, ns = orc.build_super(g["S"][:, 0], 4)
    assert ns == 3
    np.testing.assert_allclose(S1, g["S1"], rtol=1e-6, atol=1e-6)
    cand = orc.route_candidates(g["pos"], 64, 11, 16)
    scale = 1.0 / 16
    for b in range(2):
        hidx, hval, ncmp = orc.hier_select(g["qn"][b], g["S"][b, 0], g["S1"][b], 4, 2, 4, cand, scale)
        assert ncmp == int(g["ncmp"])
        fidx, fval = orc.flat_select(g["qn"][b], g["S"][b, 0], cand, 4, scale)
        for c in range(5):
            for (ia, va, ib, vb) in ((hidx[c], hval[c], g["hidx"][b, c], g["hval"][b, c]),
                                     (fidx[c], fval[c], g["fidx"][b, c], g["fval"][b, c])):
                ok, why = orc.selection_parity(ia, va, np.isfinite(va), ib, vb, np.isfinite(vb))
                assert ok, why
                np.testing.assert_allclose(np.sort(va[np.isfinite(va)]), np.sort(vb[np.isfinite(vb)]),
                                           rtol=1e-5, atol=1e-6)
    qg = orc.grouped_query(g["qfull"], 2)
    np.testing.assert_allclose(qg, g["qg"], rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("case", cases.EVAL_CASES, ids=[c[0] for c in cases.EVAL_CASES])
def test_eval_forward_matches_reference(case):
    name, c, n, seed, qk, hier, _ = case
    g = load(f"eval_{name}")
    inp = cases.eval_case_inputs(c, n, seed)
    cos, sin = orc.rope_tables(n, c["head_dim"], c["rope_theta"])
    res = orc.eval_forward(inp["q"], inp["k"], inp["v"], cos, sin, cases.cfg_dict(c, qk), inp["probes"],
                           inp["proj"], inp["q_gain"], inp["k_gain"], hier=hier, rows=g["rows"])
    np.testing.assert_allclose(res["out"], g["out"], atol=2e-5, rtol=1e-4)
    if "lse" in g:
        np.testing.assert_allclose(res["lse"], g["lse"], atol=2e-5, rtol=1e-5)
        np.testing.assert_allclose(res["out"], g["out_dense"], atol=2e-5, rtol=1e-4)


def test_selection_parity_tie_rule():
    ok, _ = orc.selection_parity([1, 2, 3], [3.0, 2.0, 1.0], [1, 1, 1], [1, 2, 4], [3.0, 2.0, 1.0 + 5e-7], [1, 1, 1])
    assert ok
    ok, _ = orc.selection_parity([1, 2, 3], [3.0, 2.0, 1.0], [1, 1, 1], [1, 2, 4], [3.0, 2.0, 0.5], [1, 1, 1])
    assert not ok


def test_round_bf16_matches_torch():
    import torch
    r = cases.rng(5)
    x = np.concatenate([cases.randn(r, 4096, scale=3.0), np.array([0.0, -0.0, np.inf, -np.inf, 3.4e38,
                                                                     1e-40], np.float32)])
    ref = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(orc.round_bf16(x), ref)


@pytest.mark.parametrize("hier", [False, True])
def test_oracle_matches_reference_model_layer(hier):
    """The oracle (fp32 mode) against layer 0 of the reference's own HBAModel
    at trained-donor QKNorm gains (gain_q * gain_k ~ 81, logits in the tens):
    the reference's hba_attention_eval outputs on the same bf16 q/k/v."""
    import model_fixture as MF
    f = MF.load()
    cfg = f["cfg"]
    n = f["q"].shape[1]
    cos, sin = orc.rope_tables(n, cfg["head_dim"], cfg["rope_theta"])
    res = orc.eval_forward(f["q"], f["k"], f["v"], cos, sin, MF.oracle_cfg(cfg), f["probes"], f["proj"],
                           f["q_gain"], f["k_gain"], hier=hier, rows=f["rows"])
    ref = f["out_eval_hier"] if hier else f["out_eval"]
    assert np.abs(res["out"] - ref).max() < 1e-4
    # the gains are in the regime the fixed-maximum softmax could not hold
    assert float(np.outer(f["q_gain"], f["k_gain"]).min()) > 50


@pytest.mark.parametrize("name,c,n,seed,qk", cases.BWD_CASES, ids=[x[0] for x in cases.BWD_CASES])
def test_backward_matches_reference_autograd(name, c, n, seed, qk):
    """The oracle's union-softmax backward (selection fixed) against fp32
    autograd through the reference's dense training path
    (attention.py:306-389): gradients of q, k, v and both QKNorm gains."""
    g = load(f"bwd_{name}")
    inp = cases.bwd_case_inputs(c, n, seed)
    cfg = cases.cfg_dict(c, qk)
    cos, sin = orc.rope_tables(n, c["head_dim"], c["rope_theta"])
    res = orc.eval_backward(inp["q"], inp["k"], inp["v"], cos, sin, cfg, inp["probes"], inp["proj"], inp["q_gain"],
                            inp["k_gain"], inp["dout"])
    qr, kr = g["qrows"], g["krows"]
    np.testing.assert_allclose(res["out"][:, qr], g["out"], rtol=1e-4, atol=1e-5)
    for key, rows in (("dq", qr), ("dk", kr), ("dv", kr)):
        ref = g[key]
        err = np.abs(res[key][:, rows] - ref).max()
        assert err <= 1e-4 * max(1.0, np.abs(ref).max()), (key, err)
    np.testing.assert_allclose(res["dq_gain"], g["dq_gain"], rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(res["dk_gain"], g["dk_gain"], rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("name,c,n,seed,qk", cases.AUX_CASES, ids=[x[0] for x in cases.AUX_CASES])
def test_aux_teacher_and_kl_match_reference(name, c, n, seed, qk):
    """The oracle's aux-KL teacher (pstar) and loss against the reference's
    own (_teacher_chunk as _aux_kl_chunked calls it; hba_attention_dense's
    aux with route_topk's block scores), fp32."""
    g = load(f"aux_{name}")
    inp = cases.bwd_case_inputs(c, n, seed)
    cfg = cases.cfg_dict(c, qk)
    dh = c["head_dim"]
    if qk:
        qc = orc.head_rmsnorm(inp["q"], inp["q_gain"])
        kc = orc.head_rmsnorm(inp["k"], inp["k_gain"])
    else:
        qc, kc = inp["q"], inp["k"]
    scale = orc.union_scale(qk, c["content_scale_mode"], c["temp_c"], c["n_cal"], c["native_ctx"], dh, n)
    pstar = orc.aux_teacher(qc, kc, cfg, scale)
    cand = orc.route_candidates(np.arange(n), c["window"], n // c["block"], c["block"])
    rows = cand.any(-1)
    assert rows.any()
    np.testing.assert_allclose(pstar[:, :, rows], g["pstar"][:, :, rows], rtol=1e-4, atol=1e-6)
    assert abs(orc.aux_kl(pstar, g["bsc"], cand) - float(g["aux"])) <= 1e-5 * max(1.0, abs(float(g["aux"])))
