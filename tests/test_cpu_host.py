"""CPU checks of the host-side logic: scalar math against the oracle, the
model patch hook, the synthetic generators, and that the product path refuses
CPU tensors instead of falling back."""

import math
import types

import numpy as np
import pytest
import torch

import hba_b200
from hba_b200 import HBAConfig, attention, synth
from oracle import hba_oracle as orc


@pytest.mark.parametrize("mode", ["inv_d", "inv_sqrt_d"])
@pytest.mark.parametrize("qk", [False, True])
@pytest.mark.parametrize("n", [1, 4096, 32768, 65536, 131072])
def test_union_scale_matches_oracle(mode, qk, n):
    cfg = HBAConfig(qknorm=qk, content_scale_mode=mode, temp_c=0.1, n_cal=None, native_ctx=32768)
    for dh in (64, 128):
        assert attention.union_scale(cfg, dh, n) == pytest.approx(
            orc.union_scale(qk, mode, 0.1, None, 32768, dh, n), rel=1e-15)


def test_scale_edge_cases():
    cfg = HBAConfig(content_scale_mode="bogus")
    with pytest.raises(ValueError):
        attention.content_scale(cfg, 64)
    assert attention.log_len_tau(HBAConfig(temp_c=0.0, n_cal=1), 10 ** 9) == 1.0
    assert attention.union_scale(HBAConfig(), 128, 131072) == pytest.approx((1 / 128) * (1 + 0.1 * math.log(4)))


def test_c_config_mirrors_reference_fields():
    cfg = HBAConfig(n_heads=32, n_kv=8, head_dim=128, fanout=16, beam=8)
    c = attention.c_config(cfg, True)
    assert (c.n_heads, c.n_kv, c.head_dim, c.block, c.window, c.sinks, c.k_blocks, c.slots, c.fanout, c.beam,
            c.hier, c.qknorm) == (32, 8, 128, 64, 1024, 4, 16, 4, 16, 8, 1, 1)


def test_product_path_refuses_cpu_tensors():
    cfg = HBAConfig()
    q = torch.zeros(1, 64, 14, 64)
    k = torch.zeros(1, 64, 2, 64)
    summ, qkn = synth.make_weights(cfg, "cpu")
    with pytest.raises(RuntimeError, match="CUDA"):
        hba_b200.hba_attention_b200(q, k, k, torch.zeros(64, 64), torch.zeros(64, 64), cfg, summ, qkn)


def test_install_rebinds_and_restores_model_module():
    def e(*a, **k):
        return "eval"

    def f(*a, **k):
        return "fused"

    def d(*a, **k):
        return "dense"

    mod = types.SimpleNamespace(hba_attention_eval=e, hba_attention_fused=f, hba_attention_dense=d)
    restore = hba_b200.install(mod)
    assert mod.hba_attention_eval is not e and mod.hba_attention_fused is hba_b200.hba_attention_b200_fused
    # equiv mode (dense, not the HBA path) stays on the module's own function
    assert mod.hba_attention_eval(None, None, None, None, None, None, None, None, None, equiv=True) == "eval"
    restore()
    assert mod.hba_attention_eval is e and mod.hba_attention_fused is f and mod.hba_attention_dense is d


def test_decode_workload_plants_candidate_blocks():
    cfg = HBAConfig()
    wl = synth.decode_workload(cfg, 2, 4096, hier=False, seed=3, device="cpu")
    pl = wl["planted"].numpy()
    bmax = (4096 - 1024) // 64 - 1
    assert ((pl >= 1) & (pl <= bmax)).all()
    assert all(len(set(pl[b, g])) == 8 for b in range(2) for g in range(2))
    # planted keys have cosine 0.8 with the normalised grouped query
    q = wl["q"].float()
    qc = q / q.pow(2).mean(-1, keepdim=True).sqrt()
    qhat = qc.to(torch.bfloat16).float().view(2, 2, 7, 64).sum(2)
    qhat = qhat / qhat.norm(dim=-1, keepdim=True)
    b, g, blk = 1, 0, int(pl[1, 0, 0])
    keys = wl["k"][b, blk * 64:(blk + 1) * 64, g].float()
    cosv = (keys / keys.norm(dim=-1, keepdim=True)) @ qhat[b, g]
    assert torch.allclose(cosv, torch.full_like(cosv, 0.8), atol=0.02)


def test_hier_planting_uses_distinct_supers():
    cfg = HBAConfig(n_heads=8, n_kv=2, head_dim=128, fanout=16, beam=8)
    wl = synth.decode_workload(cfg, 2, 16384, hier=True, seed=4, device="cpu")
    pl = wl["planted"].numpy()
    assert all(len(set((pl[b, g] // 16).tolist())) == 8 for b in range(2) for g in range(2))


def test_baseline_configs():
    cfg, B, n, hier = hba_b200.baseline_config("cfg3")
    assert (B, n, hier, cfg.n_heads, cfg.n_kv, cfg.head_dim, cfg.beam, cfg.fanout) == (32, 131072, True, 32, 8, 128,
                                                                                      8, 16)
    assert attention.log_len_tau(cfg, n) == pytest.approx(1.138629, abs=1e-6)


def _aux_case(name):
    import cases
    from hba_b200.config import HBAConfig
    c = [x for x in cases.AUX_CASES if x[0] == name][0]
    _, cc, n, seed, qk = c
    inp = cases.bwd_case_inputs(cc, n, seed)
    cfg = HBAConfig(n_heads=cc["n_heads"], n_kv=cc["n_kv"], head_dim=cc["head_dim"], block=cc["block"],
                    window=cc["window"], sinks=cc["sinks"], k_blocks=cc["k_blocks"], slots=cc["slots"],
                    fanout=cc["fanout"], beam=cc["beam"], native_ctx=cc["native_ctx"], qknorm=qk,
                    content_scale_mode=cc["content_scale_mode"], temp_c=cc["temp_c"], n_cal=cc["n_cal"], aux_w=1.0)
    return cfg, inp, n, qk


@pytest.mark.parametrize("name", ["tiny_qk", "g4d64_qk", "g4d64_noqk"])
def test_aux_kl_torch_part_matches_reference(name):
    """The aux-KL's torch part (route_topk's block scores and the KL, the
    part the summarizer's gradient flows through) on the CPU against the
    reference's own bsc, aux and probes / proj gradients
    (tests/golden/aux_*.npz), fed the reference's teacher pstar."""
    import os
    import numpy as np
    import torch
    from hba_b200.attention import aux_kl_from_teacher, route_block_scores
    from oracle import hba_oracle as orc
    cfg, inp, n, qk = _aux_case(name)
    g = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", f"aux_{name}.npz"))
    if qk:
        qc = orc.head_rmsnorm(inp["q"], inp["q_gain"])
        kc = orc.head_rmsnorm(inp["k"], inp["k_gain"])
    else:
        qc, kc = inp["q"], inp["k"]
    probes = torch.tensor(inp["probes"], requires_grad=True)
    proj = torch.tensor(inp["proj"], requires_grad=True)
    summ = type("S", (), {"probes": probes, "proj": proj})()
    bsc = route_block_scores(torch.tensor(qc), torch.tensor(kc), cfg, summ)
    ref_bsc = g["bsc"]
    fin = np.isfinite(ref_bsc)
    assert (np.isfinite(bsc.detach().numpy()) == fin).all()
    np.testing.assert_allclose(bsc.detach().numpy()[fin], ref_bsc[fin], rtol=1e-4, atol=1e-5)
    aux = aux_kl_from_teacher(torch.tensor(np.nan_to_num(g["pstar"])), bsc, cfg)
    assert abs(float(aux.detach()) - float(g["aux"])) <= 1e-4 * max(1.0, abs(float(g["aux"])))
    aux.backward()
    for key, got in (("dprobes", probes.grad), ("dproj", proj.grad)):
        np.testing.assert_allclose(got.numpy(), g[key], rtol=1e-3, atol=1e-3 * np.abs(g[key]).max())
