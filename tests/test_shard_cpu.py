"""KV-range sharded decode on CPU: two gloo ranks run `HBAShardedDecode`
(its collectives and list merges) with the oracle-built CPU stand-ins for the
shard kernels, and must reproduce the oracle's one-device decode (picks,
output and LSE) for flat and hierarchical selection."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from hba_b200 import attention
from hba_b200.config import HBAConfig
from hba_b200.sharded import HBAShardedDecode, shard_range
from oracle import hba_oracle as orc
from shard_cpu_ops import CpuShard, CpuShardOps

B, N, DH = 2, 2048, 64


def _cfg():
    return HBAConfig(n_heads=8, n_kv=2, head_dim=DH, block=64, window=128, sinks=4, k_blocks=4, slots=4, fanout=4,
                     beam=2, native_ctx=2048, qknorm=True, content_scale_mode="inv_d", temp_c=0.1, n_cal=None)


def _data(hier):
    cfg = _cfg()
    rng = np.random.default_rng(11)
    Hq, Hkv, m = cfg.n_heads, cfg.n_kv, cfg.slots
    q = orc.round_bf16(rng.standard_normal((B, Hq, DH)))
    k = orc.round_bf16(rng.standard_normal((B, N, Hkv, DH)))
    v = orc.round_bf16(rng.standard_normal((B, N, Hkv, DH)))
    # a few planted blocks so that the top-k is well separated from the noise
    qg_dir = q.reshape(B, Hkv, Hq // Hkv, DH).sum(2)
    for b in range(B):
        for g in range(Hkv):
            for blk in rng.choice(np.arange(1, N // 64 - 4), 3, replace=False):
                k[b, blk * 64:(blk + 1) * 64, g] += 0.8 * qg_dir[b, g] / np.linalg.norm(qg_dir[b, g]) * np.sqrt(DH)
    k = orc.round_bf16(k)
    q_gain = (1 + 0.1 * rng.standard_normal(Hq)).astype(np.float32)
    k_gain = (1 + 0.1 * rng.standard_normal(Hkv)).astype(np.float32)
    probes = rng.standard_normal((Hkv, m, DH)) / np.sqrt(DH)
    proj = np.eye(DH)[None].repeat(Hkv, 0) + 0.02 * rng.standard_normal((Hkv, DH, DH))
    kc = orc.head_rmsnorm(k, k_gain, bf16=True)
    S0 = orc.round_bf16(orc.summarize(kc, probes, proj, cfg.block))
    S1 = orc.round_bf16(orc.build_super(S0, cfg.fanout)[0]) if hier else None
    cos, sin = orc.rope_tables(N, DH, 1e6)
    return cfg, q, kc, v, S0, S1, q_gain, k_gain, cos, sin


def _rank(rank, world, port, hier, outdir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg, q, kc, v, S0, S1, q_gain, k_gain, cos, sin = _data(hier)
        tok_lo, n_loc, _ = shard_range(cfg, N, rank, world, hier)
        local = CpuShard(kc, v, S0, S1, q_gain, k_gain, tok_lo, n_loc, cfg.block, cfg.fanout)
        sh = HBAShardedDecode(cfg, B, N, None, None, torch.as_tensor(cos), torch.as_tensor(sin), device="cpu",
                              hier=hier, ops=CpuShardOps(cfg, cos, sin), local=local)
        sh._set_lengths(N)
        out = torch.empty(B, cfg.n_heads, DH, dtype=torch.float32)
        lse = torch.empty(B, cfg.n_heads, dtype=torch.float32)
        sel = torch.full((B, cfg.n_kv, cfg.k_blocks), -2, dtype=torch.int32)
        sel_sc = torch.empty(B, cfg.n_kv, cfg.k_blocks, dtype=torch.float32)
        sh.decode_into(torch.as_tensor(q, dtype=torch.bfloat16), out, lse, sel, sel_sc)
        ocfg = dict(block=cfg.block, window=cfg.window, sinks=cfg.sinks, k_blocks=cfg.k_blocks, fanout=cfg.fanout,
                    beam=cfg.beam)
        scale = attention.union_scale(cfg, DH, N)
        ref = orc.decode(q, kc, v, cos, sin, S0, S1, ocfg, scale, q_gain, hier=hier, bf16=True)
        np.savez(os.path.join(outdir, f"r{rank}.npz"), out=out.numpy(), lse=lse.numpy(), sel=sel.numpy(),
                 ref_out=ref["out"], ref_lse=ref["lse"], ref_idx=ref["idx"], ref_ok=ref["ok"])
    finally:
        dist.destroy_process_group()


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("hier", [False, True])
def test_sharded_decode_matches_one_device(hier, tmp_path):
    world = 2
    mp.spawn(_rank, args=(world, _port(), hier, str(tmp_path)), nprocs=world, join=True)
    results = [np.load(tmp_path / f"r{r}.npz") for r in range(world)]
    for r in results:
        # every rank ends with the whole answer
        np.testing.assert_allclose(r["out"], r["ref_out"], atol=1e-5, rtol=1e-5)
        np.testing.assert_allclose(r["lse"], r["ref_lse"], atol=1e-5)
        for b in range(B):
            for g in range(r["sel"].shape[1]):
                picks = sorted(int(i) for i in r["sel"][b, g] if i >= 0)
                want = sorted(int(i) for i, ok in zip(r["ref_idx"][b, g], r["ref_ok"][b, g]) if ok)
                assert picks == want, (b, g, picks, want)
    np.testing.assert_array_equal(results[0]["out"], results[1]["out"])


def test_shard_range_alignment():
    cfg = _cfg()
    for world in (1, 2, 4, 8):
        spans = [shard_range(cfg, 5000, r, world, True)[:2] for r in range(world)]
        n_total = shard_range(cfg, 5000, 0, world, True)[2]
        assert n_total >= 5000 and n_total % (cfg.block * cfg.fanout * world) == 0
        assert spans[0][0] == 0 and all(lo % (cfg.block * cfg.fanout) == 0 for lo, _ in spans)
        assert sum(n for _, n in spans) == n_total
        assert all(spans[i][0] + spans[i][1] == spans[i + 1][0] for i in range(world - 1))
