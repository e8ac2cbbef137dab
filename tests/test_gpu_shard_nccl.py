"""KV-range sharded decode over NCCL (the split path): two processes, one GPU
each, run `HBAShardedDecode(fused=False)` -- the shard kernels with
torch.distributed collectives in between; every rank's output must match the
one-GPU decode of the same context.  Needs 2 GPUs."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from gpu_helpers import LSE_TOL, OUT_TOL, cfg_of

pytestmark = pytest.mark.gpu

B, N = 4, 16384


def _cfg():
    return cfg_of(n_heads=32, n_kv=8, head_dim=128, fanout=16, beam=8, k_blocks=16)


def _rank(rank, world, port, outdir):
    import datetime
    from hba_b200 import synth
    from hba_b200.sharded import HBAShardedDecode
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        cfg = _cfg()
        dev = torch.device("cuda", rank)
        summ, qkn = synth.make_weights(cfg, dev, seed=3, gains=True)
        cos, sin = synth.rope_tables(N, cfg.head_dim, 1e6)
        wl = synth.decode_workload(cfg, B, N, hier=True, seed=3, device=dev, qkn=qkn, planted=8)
        sh = HBAShardedDecode(cfg, B, N, summ, qkn, cos, sin, device=dev, hier=True, fused=False)
        sh.fill(wl["k"], wl["v"])
        q = wl["q"].contiguous()
        out = torch.empty_like(q)
        lse = torch.empty(B, cfg.n_heads, dtype=torch.float32, device=dev)
        si = torch.empty(B, cfg.n_kv, cfg.k_blocks, dtype=torch.int32, device=dev)
        ss = torch.empty(B, cfg.n_kv, cfg.k_blocks, dtype=torch.float32, device=dev)
        for _ in range(3):  # repeated steps reuse the buffers
            sh.decode_into(q, out, lse, si, ss)
        torch.cuda.synchronize()
        out_e = out.clone()
        sh.capture(q, out, lse, si, ss)  # the step as one CUDA graph, collectives included
        out.zero_()
        sh.replay()
        torch.cuda.synchronize()
        sh.release()
        assert torch.equal(out, out_e)
        np.savez(os.path.join(outdir, f"r{rank}.npz"), out=out.float().cpu().numpy(), lse=lse.cpu().numpy(),
                 si=si.cpu().numpy(), ss=ss.cpu().numpy(), status=sh.status.cpu().numpy())
    finally:
        dist.destroy_process_group()


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_shard_nccl_world2(tmp_path):
    from hba_b200 import HBADecodeCache, synth
    world = 2
    mp.spawn(_rank, args=(world, _port(), str(tmp_path)), nprocs=world, join=True)
    cfg = _cfg()
    summ, qkn = synth.make_weights(cfg, "cuda", seed=3, gains=True)
    cos, sin = synth.rope_tables(N, cfg.head_dim, 1e6)
    wl = synth.decode_workload(cfg, B, N, hier=True, seed=3, qkn=qkn, planted=8)
    one = HBADecodeCache(cfg, B, N, summ, qkn, cos, sin, hier=True)
    one.append(wl["k"], wl["v"])
    out1, lse1, (si1, ss1) = one.attend(wl["q"].contiguous(), return_lse=True, return_selection=True)
    for r in range(world):
        res = np.load(tmp_path / f"r{r}.npz")
        assert int(res["status"][0]) == 0
        np.testing.assert_array_equal(res["si"], si1.cpu().numpy())
        np.testing.assert_array_equal(res["ss"], ss1.cpu().numpy())
        assert np.abs(res["out"] - out1.float().cpu().numpy()).max() <= OUT_TOL
        assert np.abs(res["lse"] - lse1.cpu().numpy()).max() <= LSE_TOL
