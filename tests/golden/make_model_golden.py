"""Generate ``tests/golden/model_layer.npz``: one layer of the REFERENCE
``HBAModel`` (nealxpatel/hierarchical-block-attention, ``src/hba``), run on
CPU here, in the regime a trained donor puts its attention in.

Run it where the reference source is importable:

    HBA_REFERENCE_SRC=/path/to/hierarchical-block-attention/src python tests/golden/make_model_golden.py

What it does:

* builds a tiny random-init Qwen2 donor and wraps it in the reference's own
  ``HBAModel`` -- the pattern of the reference's CPU tests
  (tests/test_qknorm.py:24-53) -- at a geometry the B200 kernels cover
  (head_dim 64, block 64, G = 4 query heads per KV head);
* scales the donor's q/k projections up, as a trained donor's q/k RMS are
  large, then calibrates the QKNorm gains with the reference's own
  ``init_qknorm_gains`` (src/hba/model.py:197-253): gain_q * gain_k =
  sqrt(dh) * rms_q * rms_k, which lands in the tens to hundreds;
* runs ``HBAModel.forward`` in modes "eval" and "eval_hier" with hooks that
  capture layer 0's q/k/v projections (the arguments ``block_fn`` hands to
  ``hba_attention_eval``, src/hba/model.py:121-140) and the attention output
  that goes into ``o_proj``;
* rounds q/k/v to bf16 (what the B200 path consumes) and runs the
  reference's ``hba_attention_eval`` on those exact values (fp32), flat and
  hierarchical -- these outputs are the fixture's reference answers.

The tests read only the .npz: q/k/v as raw bf16 bits, the layer's
summarizer weights and QKNorm gains, the config, and the outputs at sampled
rows.
"""

import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

REF_SRC = os.environ.get("HBA_REFERENCE_SRC")
if not REF_SRC or not os.path.isdir(REF_SRC):
    sys.exit("set HBA_REFERENCE_SRC to the reference's src/ directory")
_tmp = tempfile.mkdtemp(prefix="hba-golden-")
os.chdir(_tmp)  # the reference's config module creates results/data/logs in the CWD
sys.path.insert(0, REF_SRC)

import torch  # noqa: E402

from hba import attention as ref_attn  # noqa: E402
from hba.config import HBAConfig  # noqa: E402
from hba.model import HBAModel, init_qknorm_gains  # noqa: E402

N_TOK = 1024
LAYER = 0
QK_SCALE = 10.0  # q/k projection scale-up: per-head q/k RMS of ~4 instead of ~0.45

GEOM = dict(n_layers=2, n_heads=4, n_kv=1, head_dim=64, hidden=256, rope_theta=1_000_000.0, native_ctx=512,
            vocab_size=300, block=64, window=256, sinks=4, k_blocks=4, slots=4, fanout=4, beam=2, hier_from=512,
            heal_ctx=256, mem_elem_cap=2e7, attn_backend="naive", qknorm=True, content_scale_mode="inv_d",
            temp_c=0.1, n_cal=None, aux_w=0.0)


def bf16_bits(x):
    return x.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


@torch.no_grad()
def main():
    from transformers import Qwen2Config, Qwen2ForCausalLM

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    qcfg = Qwen2Config(vocab_size=GEOM["vocab_size"], hidden_size=GEOM["hidden"], intermediate_size=512,
                       num_hidden_layers=GEOM["n_layers"], num_attention_heads=GEOM["n_heads"],
                       num_key_value_heads=GEOM["n_kv"], max_position_embeddings=8192,
                       rope_theta=GEOM["rope_theta"], tie_word_embeddings=True)
    torch.manual_seed(0)
    donor = Qwen2ForCausalLM(qcfg).eval()
    for lyr in donor.model.layers:
        for lin in (lyr.self_attn.q_proj, lyr.self_attn.k_proj):
            lin.weight.mul_(QK_SCALE)
            if lin.bias is not None:
                lin.bias.mul_(QK_SCALE)
    cfg = HBAConfig(**GEOM)
    model = HBAModel(donor, cfg).eval()
    init_qknorm_gains(model, cfg)

    g = torch.Generator().manual_seed(20261202)
    ids = torch.randint(0, cfg.vocab_size, (1, N_TOK), generator=g)
    cos, sin = ref_attn.rope_tables(N_TOK, cfg.head_dim, cfg.rope_theta, "cpu")
    lyr = model.core.layers[LAYER]
    cap = {}
    hooks = [lyr.self_attn.q_proj.register_forward_hook(lambda m, i, o: cap.__setitem__("q", o.detach())),
             lyr.self_attn.k_proj.register_forward_hook(lambda m, i, o: cap.__setitem__("k", o.detach())),
             lyr.self_attn.v_proj.register_forward_hook(lambda m, i, o: cap.__setitem__("v", o.detach())),
             lyr.self_attn.o_proj.register_forward_pre_hook(lambda m, i: cap.__setitem__("o", i[0].detach()))]
    model_out = {}
    qkv = None
    for mode in ("eval", "eval_hier"):
        model(ids, cos, sin, cfg.mem_elem_cap, mode=mode, tail=1)
        model_out[mode] = cap["o"].clone()
        qkv = (cap["q"].clone(), cap["k"].clone(), cap["v"].clone())  # layer 0: the same in both modes
    for h in hooks:
        h.remove()

    B, n, Hq, Hkv, dh = 1, N_TOK, cfg.n_heads, cfg.n_kv, cfg.head_dim
    q = qkv[0].view(B, n, Hq, dh)
    k = qkv[1].view(B, n, Hkv, dh)
    v = qkv[2].view(B, n, Hkv, dh)
    qb, kb, vb = (t.to(torch.bfloat16).float() for t in (q, k, v))
    summ, qkn = model.summarizers[LAYER], model.qknorms[LAYER]
    outs = {}
    for name, hier in (("eval", False), ("eval_hier", True)):
        o = ref_attn.hba_attention_eval(qb, kb, vb, cos, sin, cfg, summ, qkn, cfg.mem_elem_cap, hier=hier)
        outs[name] = o
        # the model's own call (unrounded inputs) agrees to bf16-input precision
        d = (o.reshape(B, n, -1) - model_out[name]).abs().max().item()
        print(f"{name}: |ref(bf16 inputs) - model layer output| max {d:.3g}")
    gq = qkn.q.gain.detach().numpy().astype(np.float32)
    gk = qkn.k.gain.detach().numpy().astype(np.float32)
    print("gain_q", gq, "gain_k", gk, "products", np.outer(gq, gk).ravel())
    r = np.random.default_rng(7)
    rows = np.array(sorted({0, 1, 2, 3, 4, 255, 256, 257, 511, 512, n // 2, n - 2, n - 1} |
                           set(r.choice(n, size=48, replace=False).tolist())), dtype=np.int64)
    path = os.path.join(HERE, "model_layer.npz")
    np.savez_compressed(
        path, cfg=np.array(json.dumps({k: GEOM[k] for k in GEOM})), layer=np.array(LAYER),
        q_bits=bf16_bits(q), k_bits=bf16_bits(k), v_bits=bf16_bits(v),
        probes=summ.probes.detach().numpy().astype(np.float32), proj=summ.proj.detach().numpy().astype(np.float32),
        q_gain=gq, k_gain=gk, rows=rows, out_eval=outs["eval"].numpy()[:, rows],
        out_eval_hier=outs["eval_hier"].numpy()[:, rows])
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
