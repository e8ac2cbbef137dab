"""Sequence-sharded model prefill + decode (HBAShardedModelDecoder) on two
GPUs against the one-GPU HBAModelDecoder on the same model: the logits of
the prompt's last position and of four decode steps must agree.  The stand-in
model has the reference HBAModel's layout around a tiny random-init Qwen2
donor (built identically on every rank from a seed).  Needs 2 GPUs."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

B, N0, EXTRA, CAP = 2, 1024, 4, 1088


def _model(dev):
    import types
    from transformers import Qwen2Config, Qwen2ForCausalLM
    from hba_b200 import synth
    from hba_b200.config import HBAConfig
    cfg = HBAConfig(n_layers=2, n_heads=8, n_kv=2, head_dim=64, hidden=512, rope_theta=1e6, native_ctx=4096,
                    vocab_size=512, block=64, window=256, sinks=4, k_blocks=4, slots=4, fanout=4, beam=2)
    qcfg = Qwen2Config(vocab_size=512, hidden_size=512, intermediate_size=1024, num_hidden_layers=2,
                       num_attention_heads=8, num_key_value_heads=2, max_position_embeddings=8192, rope_theta=1e6,
                       tie_word_embeddings=True)
    torch.manual_seed(0)
    donor = Qwen2ForCausalLM(qcfg).to(dev, torch.bfloat16).eval()
    summ, qkn = zip(*[synth.make_weights(cfg, dev, seed=10 + i, gains=True) for i in range(2)])
    return types.SimpleNamespace(cfg=cfg, core=donor.model, lm_head=donor.lm_head, summarizers=list(summ),
                                 qknorms=list(qkn))


def _ids():
    g = torch.Generator().manual_seed(5)
    return torch.randint(0, 512, (B, N0 + EXTRA), generator=g)


def _rank(rank, world, port, outdir):
    import datetime
    from hba_b200.sharded_model import HBAShardedModelDecoder
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    dec = None
    try:
        m = _model(dev)
        ids = _ids().to(dev)
        dec = HBAShardedModelDecoder(m, B, CAP, dev)
        outs = [dec.prefill(ids[:, :N0]).float().cpu().numpy()]
        for j in range(EXTRA):
            outs.append(dec.step(ids[:, N0 + j]).float().cpu().numpy())
        torch.cuda.synchronize()
        np.save(os.path.join(outdir, f"r{rank}.npy"), np.stack(outs))
    finally:
        if dec is not None:
            dec.close()
        dist.destroy_process_group()


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_model_matches_one_gpu(tmp_path, world):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    mp.spawn(_rank, args=(world, _port(), str(tmp_path)), nprocs=world, join=True)
    from hba_b200.decoder import HBAModelDecoder
    m = _model("cuda")
    ids = _ids().cuda()
    dec = HBAModelDecoder(m, B, CAP)
    ref = [dec.prefill(ids[:, :N0]).float()] + [dec.step(ids[:, N0 + j]).float() for j in range(EXTRA)]
    ref = torch.stack(ref).cpu().numpy()
    for r in range(world):
        got = np.load(tmp_path / f"r{r}.npy")
        assert np.isfinite(got).all()
        err = np.abs(got - ref).max()
        assert err <= 0.05 * np.abs(ref).max() + 0.05, (r, err)
        cos = (got * ref).sum(-1) / (np.linalg.norm(got, axis=-1) * np.linalg.norm(ref, axis=-1))
        assert cos.min() > 0.999, (r, cos.min())
