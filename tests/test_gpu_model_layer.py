"""A layer of the reference's own HBAModel, replayed through ``install()``.

``install(model_module)`` rebinds the names ``HBAModel.forward`` calls
(src/hba/model.py:119-141).  The reference package is not importable on the
GPU box, so a stand-in module namespace carries those names; the patched
functions are then called exactly as ``block_fn`` calls them, with layer 0's
q/k/v, summarizer and QKNorm gains from ``tests/golden/model_layer.npz``
(produced by running the reference's HBAModel; gain_q * gain_k ~ 81, the
trained-donor regime).

Two comparisons per mode (eval, eval_hier):
* strict parity against the oracle on the same stored bf16 operands: picks
  index-exact (ties within 1e-6 of the score magnitude), output <= 2e-2,
  LSE <= 1e-3;
* against the reference's own fp32 ``hba_attention_eval`` output: the B200
  path stores the QKNorm'd q/k and the RoPE'd window operands in bf16 (as the
  reference's bf16 path does), which at these gains moves this fixture's
  outputs by up to 0.025 (the oracle's bf16-operand mode shows the same gap
  on CPU), so that bound is 5e-2.
"""

import types

import numpy as np
import pytest
import torch

import gpu_helpers as H
import model_fixture as MF
from hba_b200 import synth
from hba_b200.config import HBAConfig
from hba_b200.ops import qknorm_b200, summarize_b200
from hba_b200.patch import install
from oracle import hba_oracle as orc

pytestmark = pytest.mark.gpu

REF_TOL = 5e-2


def _setup():
    f = MF.load()
    c = f["cfg"]
    cfg = HBAConfig(**{k: v for k, v in c.items() if k in HBAConfig.__dataclass_fields__})
    dev = "cuda"
    q = torch.from_numpy(f["q"]).to(dev, torch.bfloat16)
    k = torch.from_numpy(f["k"]).to(dev, torch.bfloat16)
    v = torch.from_numpy(f["v"]).to(dev, torch.bfloat16)
    summ = synth.SummarizerWeights(torch.from_numpy(f["probes"]).to(dev), torch.from_numpy(f["proj"]).to(dev))
    qkn = synth.QKNormGains(torch.from_numpy(f["q_gain"]).to(dev), torch.from_numpy(f["k_gain"]).to(dev))
    cos, sin = synth.rope_tables(q.shape[1], cfg.head_dim, cfg.rope_theta)
    return f, cfg, q, k, v, summ, qkn, cos, sin


def _stand_in_module():
    def never(*a, **kw):
        raise AssertionError("the reference's own function was called instead of the B200 path")
    return types.SimpleNamespace(hba_attention_eval=never, hba_attention_fused=never, hba_attention_dense=never)


@pytest.mark.parametrize("hier", [False, True])
def test_reference_model_layer_through_install(hier):
    f, cfg, q, k, v, summ, qkn, cos, sin = _setup()
    mod = _stand_in_module()
    orig = dict(vars(mod))
    restore = install(mod)
    try:
        with torch.no_grad():
            # the call of block_fn for mode "eval" / "eval_hier" (src/hba/model.py:137-140)
            out = mod.hba_attention_eval(q, k, v, cos, sin, cfg, summ, qkn, cfg.mem_elem_cap, hier=hier)
            o2, aux = mod.hba_attention_fused(q, k, v, cos, sin, cfg, summ, qkn)  # the train-forward contract
    finally:
        restore()
    assert dict(vars(mod)) == orig
    torch.cuda.synchronize()
    rows = f["rows"]
    got = H.np32(out)[:, rows]
    ref = f["out_eval_hier"] if hier else f["out_eval"]
    assert np.isfinite(got).all()
    assert np.abs(got - ref).max() <= REF_TOL, np.abs(got - ref).max()
    if not hier:
        assert torch.equal(o2, out) and float(aux) == 0.0

    # strict parity on the same stored operands (the kernel's own QKNorm'd q/k and summaries)
    with torch.no_grad():
        from hba_b200 import hba_attention_b200
        out3, lse, (si, ss) = hba_attention_b200(q, k, v, cos, sin, cfg, summ, qkn, hier=hier, return_lse=True,
                                                 return_selection=True)
        qc, kc = qknorm_b200(q, qkn.q.gain), qknorm_b200(k, qkn.k.gain)
        S0 = summarize_b200(kc, summ.probes, summ.proj, cfg)
        S1 = None
        if hier:
            from hba_b200.ops import build_super_b200
            S1 = build_super_b200(S0, cfg)[0]
    torch.cuda.synchronize()
    assert torch.equal(out3, out)
    res = orc.eval_forward(f["q"], f["k"], f["v"], H.np32(cos), H.np32(sin), MF.oracle_cfg(f["cfg"]), f["probes"],
                           f["proj"], f["q_gain"], f["k_gain"], hier=hier, bf16=True, rows=rows,
                           summaries=H.np32(S0), supers=None if S1 is None else H.np32(S1), kc=H.np32(kc),
                           qc=H.np32(qc))
    si_n, ss_n = si.cpu().numpy(), H.np32(ss)
    for g in range(cfg.n_kv):
        for r, row in enumerate(rows):
            H.compare_selection(si_n[0, g, row], ss_n[0, g, row], res["idx"][0, g, r], res["val"][0, g, r],
                                res["ok"][0, g, r], f"g={g} row={row}", tie_rel=H.TIE_REL_TRAINED)
    assert np.abs(got - res["out"]).max() <= H.OUT_TOL
    assert np.abs(H.np32(lse)[:, :, rows] - res["lse"]).max() <= H.LSE_TOL


def test_reference_model_layer_decode_matches_prefill_last_row():
    """The decode cache over the same layer: the newest token attends over the
    n cached tokens with the same tau(n) and must give prefill's last row."""
    from hba_b200 import HBADecodeCache, hba_attention_b200
    f, cfg, q, k, v, summ, qkn, cos, sin = _setup()
    n = q.shape[1]
    with torch.no_grad():
        out, lse, (si, ss) = hba_attention_b200(q, k, v, cos, sin, cfg, summ, qkn, return_lse=True,
                                                return_selection=True)
    cache = HBADecodeCache(cfg, 1, n, summ, qkn, cos, sin)
    cache.append(k, v)
    o2, l2, (si2, ss2) = cache.attend(q[:, n - 1], return_lse=True, return_selection=True)
    H.assert_picks_agree(si[:, :, n - 1], ss[:, :, n - 1], si2, ss2)
    assert (out[:, n - 1].float() - o2.float()).abs().max().item() < 2e-2
    assert (lse[:, :, n - 1] - l2).abs().max().item() < 1e-3
    ref = f["out_eval"][:, list(f["rows"]).index(n - 1)]
    assert np.abs(H.np32(o2) - ref).max() <= REF_TOL
