"""Fused KV-range sharded decode over NVLink: two processes, one GPU each,
run `HBAShardedDecode` on its default GPU path -- one
`hba_b200_decode_shard_fused` launch per step, the lists and the (O, l)
partials exchanged through the ranks' IPC-mapped buffers inside the kernel.
Every rank's picks must equal the one-GPU decode's exactly and its output /
LSE must agree within the parity tolerances, over several steps (eager, then
as a replayed CUDA graph) and across an append.  Needs 2 (and, for the 4-rank cases, 4) GPUs."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from gpu_helpers import LSE_TOL, OUT_TOL, cfg_of

pytestmark = pytest.mark.gpu

B, CAP = 4, 16384


def _cfg(hier):
    if hier:
        return cfg_of(n_heads=32, n_kv=8, head_dim=128, fanout=16, beam=8, k_blocks=16)
    return cfg_of(n_heads=14, n_kv=2, head_dim=64, k_blocks=16)


def _workload(cfg, hier, n, dev, gains=True):
    from hba_b200 import synth
    summ, qkn = synth.make_weights(cfg, dev, seed=7, gains=gains)
    cos, sin = synth.rope_tables(CAP, cfg.head_dim, 1e6)
    wl = synth.decode_workload(cfg, B, n + 1, hier=hier, seed=7, device=dev, qkn=qkn, planted=8)
    return summ, qkn, cos, sin, wl


def _rank(rank, world, port, outdir, hier, n, gains=True):
    import datetime
    from hba_b200.sharded import HBAShardedDecode
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    sh = None
    try:
        cfg = _cfg(hier)
        dev = torch.device("cuda", rank)
        summ, qkn, cos, sin, wl = _workload(cfg, hier, n, dev, gains)
        sh = HBAShardedDecode(cfg, B, CAP, summ, qkn, cos, sin, device=dev, hier=hier)
        assert sh.fused
        sh.fill(wl["k"][:, :n], wl["v"][:, :n])
        q = wl["q"].contiguous()
        out = torch.empty_like(q)
        lse = torch.empty(B, cfg.n_heads, dtype=torch.float32, device=dev)
        si = torch.empty(B, cfg.n_kv, cfg.k_blocks, dtype=torch.int32, device=dev)
        ss = torch.empty(B, cfg.n_kv, cfg.k_blocks, dtype=torch.float32, device=dev)
        for _ in range(3):  # repeated steps: the epochs advance
            sh.decode_into(q, out, lse, si, ss)
        torch.cuda.synchronize()
        res = dict(out=out.float().cpu().numpy(), lse=lse.cpu().numpy(), si=si.cpu().numpy(),
                   ss=ss.cpu().numpy())
        out_e = out.clone()
        sh.capture(q, out, lse, si, ss)  # the step as a CUDA graph: epoch bump + the fused kernel
        for _ in range(2):
            out.zero_()
            sh.replay()
        torch.cuda.synchronize()
        sh.release()
        assert torch.equal(out, out_e)
        sh.append(wl["k"][:, n:n + 1], wl["v"][:, n:n + 1])  # one more token; decode again
        sh.decode_into(q, out, lse, si, ss)
        torch.cuda.synchronize()
        res.update(out2=out.float().cpu().numpy(), lse2=lse.cpu().numpy(), si2=si.cpu().numpy(),
                   status=sh.status.cpu().numpy())
        np.savez(os.path.join(outdir, f"r{rank}.npz"), **res)
    finally:
        if sh is not None:
            sh.close()
        dist.destroy_process_group()


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _one_gpu(cfg, hier, n, wl, summ, qkn, cos, sin):
    from hba_b200 import HBADecodeCache
    one = HBADecodeCache(cfg, B, CAP, summ, qkn, cos, sin, hier=hier)
    one.append(wl["k"][:, :n], wl["v"][:, :n])
    a = one.attend(wl["q"].contiguous(), return_lse=True, return_selection=True)
    one.append(wl["k"][:, n:n + 1], wl["v"][:, n:n + 1])
    b = one.attend(wl["q"].contiguous(), return_lse=True, return_selection=True)
    return a, b


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("hier,n", [(False, CAP - 64), (False, CAP // 2 + 512), (True, CAP - 1024),
                                    (True, CAP // 2 + 512)])
def test_shard_fused(tmp_path, hier, n, world):
    # n = CAP // 2 + 512: the 1024-token window straddles two ranks
    _check(tmp_path, hier, n, world, True)


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("hier,n", [(False, CAP // 2 + 512), (True, CAP - 1024)])
def test_shard_fused_trained_gains(tmp_path, hier, n, world):
    # trained QKNorm gains: each rank's partial carries its own running
    # maximum and the in-kernel merge rescales them
    _check(tmp_path, hier, n, world, "trained")


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("hier", [False, True])
def test_shard_fused_empty_ranks(tmp_path, hier, world):
    # the context ends where a rank's range begins: the later ranks own no
    # token (no window, no candidate) until the append gives the first of
    # them one; they still take part in every exchange
    _check(tmp_path, hier, CAP // 2, world, True)


def _check(tmp_path, hier, n, world, gains):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    mp.spawn(_rank, args=(world, _port(), str(tmp_path), hier, n, gains), nprocs=world, join=True)
    cfg = _cfg(hier)
    summ, qkn, cos, sin, wl = _workload(cfg, hier, n, "cuda", gains)
    (o1, l1, (si1, ss1)), (o2, l2, (si2, _)) = _one_gpu(cfg, hier, n, wl, summ, qkn, cos, sin)
    for r in range(world):
        res = np.load(tmp_path / f"r{r}.npz")
        assert int(res["status"][0]) == 0
        np.testing.assert_array_equal(res["si"], si1.cpu().numpy())
        np.testing.assert_array_equal(res["ss"], ss1.cpu().numpy())
        assert np.abs(res["out"] - o1.float().cpu().numpy()).max() <= OUT_TOL
        assert np.abs(res["lse"] - l1.cpu().numpy()).max() <= LSE_TOL
        np.testing.assert_array_equal(res["si2"], si2.cpu().numpy())
        assert np.abs(res["out2"] - o2.float().cpu().numpy()).max() <= OUT_TOL
        assert np.abs(res["lse2"] - l2.cpu().numpy()).max() <= LSE_TOL
