"""Model-level incremental decode (HBAModelDecoder) against the model's own
prefill.  The stand-in model has the reference HBAModel's attribute layout
around a tiny random-init Hugging Face Qwen2 donor (the reference's CPU
tests build theirs the same way, tests/test_qknorm.py:24-53), at a geometry
the B200 kernels cover.  Decoding token n after a prefill of n tokens must
give the logits that a prefill over the longer sequence gives at row n
(same temperature: both lengths within native_ctx)."""

import types

import pytest
import torch

from hba_b200 import synth
from hba_b200.config import HBAConfig
from hba_b200.decoder import HBAModelDecoder

pytestmark = pytest.mark.gpu


def _model(seed=0, n_layers=2):
    from transformers import Qwen2Config, Qwen2ForCausalLM
    cfg = HBAConfig(n_layers=n_layers, n_heads=8, n_kv=2, head_dim=64, hidden=512, rope_theta=1e6, native_ctx=4096,
                    vocab_size=512, block=64, window=256, sinks=4, k_blocks=4, slots=4, fanout=4, beam=2)
    qcfg = Qwen2Config(vocab_size=cfg.vocab_size, hidden_size=cfg.hidden, intermediate_size=1024,
                       num_hidden_layers=n_layers, num_attention_heads=cfg.n_heads, num_key_value_heads=cfg.n_kv,
                       max_position_embeddings=8192, rope_theta=cfg.rope_theta, tie_word_embeddings=True)
    torch.manual_seed(seed)
    donor = Qwen2ForCausalLM(qcfg).to("cuda", torch.bfloat16).eval()
    summ, qkn = [], []
    for i in range(n_layers):
        s, q = synth.make_weights(cfg, "cuda", seed=seed + i, gains=True)
        summ.append(s)
        qkn.append(q)
    return types.SimpleNamespace(cfg=cfg, core=donor.model, lm_head=donor.lm_head, summarizers=summ, qknorms=qkn)


@pytest.mark.parametrize("hier", [False, True])
def test_decode_steps_match_prefill_rows(hier):
    m = _model()
    B, n0, extra = 2, 1024, 4
    g = torch.Generator().manual_seed(3)
    ids = torch.randint(0, m.cfg.vocab_size, (B, n0 + 64), generator=g).cuda()
    dec = HBAModelDecoder(m, B, n0 + 64, hier=hier)
    last = dec.prefill(ids[:, :n0])
    steps = [dec.step(ids[:, n0 + j]) for j in range(extra)]
    ref = HBAModelDecoder(m, B, n0 + 64, hier=hier).prefill(ids, all_logits=True)   # [B, n0 + 64, V]
    rows = [ref[:, n0 - 1]] + [ref[:, n0 + j] for j in range(extra)]
    got = [last] + steps
    for r, (a, b) in enumerate(zip(got, rows)):
        a, b = a.float(), b.float()
        err = (a - b).abs().max().item()
        scale = b.abs().max().item()
        cos = torch.nn.functional.cosine_similarity(a, b, dim=-1).min().item()
        assert torch.isfinite(a).all()
        assert cos > 0.999 and err <= 0.05 * scale + 0.05, (r, err, scale, cos)
    assert dec.n == n0 + extra
