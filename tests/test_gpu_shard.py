"""KV-range sharded decode on one GPU: P ranks run as threads of one process,
each with its own shard caches and the real `hba_b200_decode_shard_*`
kernels, exchanging lists and partials through an in-process stand-in for the
collectives (no kernel waits on another rank, so their launches may
interleave on one device).  The sharded picks must equal the one-GPU decode's
picks exactly, and output / LSE must agree within the parity tolerances."""

import threading

import numpy as np
import pytest
import torch

from gpu_helpers import LSE_TOL, OUT_TOL, cfg_of
from hba_b200 import HBADecodeCache, synth
from hba_b200.sharded import HBAShardedDecode, shard_range

pytestmark = pytest.mark.gpu


class _Shared:
    def __init__(self, world):
        self.bar = threading.Barrier(world, timeout=120)
        self.slots = [None] * world


class ThreadComm:
    """all_gather among the threads of one process."""

    def __init__(self, rank, world, shared):
        self.rank, self.world, self.s = rank, world, shared

    def all_gather(self, t):
        self.s.bar.wait()
        self.s.slots[self.rank] = t.clone()
        self.s.bar.wait()
        out = torch.stack(self.s.slots)
        self.s.bar.wait()
        return out


def _run(cfg, B, n, hier, world, seed=5, cap=None, gains=True):
    """n context tokens in a sharded capacity of `cap` (default n)."""
    cap = cap or n
    summ, qkn = synth.make_weights(cfg, "cuda", seed=seed, gains=gains)
    cos, sin = synth.rope_tables(cap, cfg.head_dim, 1e6)
    wl = synth.decode_workload(cfg, B, n, hier=hier, seed=seed, qkn=qkn, planted=8)
    q = wl["q"].contiguous()
    one = HBADecodeCache(cfg, B, n, summ, qkn, cos, sin, hier=hier)
    one.append(wl["k"], wl["v"])
    out1, lse1, (si1, ss1) = one.attend(q, return_lse=True, return_selection=True)
    torch.cuda.synchronize()

    shared = _Shared(world)
    results, errors = [None] * world, []

    def rank_main(r):
        try:
            sh = HBAShardedDecode(cfg, B, cap, summ, qkn, cos, sin, hier=hier, comm=ThreadComm(r, world, shared))
            sh.fill(wl["k"], wl["v"])
            out = torch.empty_like(q)
            lse = torch.empty(B, cfg.n_heads, dtype=torch.float32, device="cuda")
            si = torch.empty(B, cfg.n_kv, cfg.k_blocks, dtype=torch.int32, device="cuda")
            ss = torch.empty(B, cfg.n_kv, cfg.k_blocks, dtype=torch.float32, device="cuda")
            sh.decode_into(q, out, lse, si, ss)
            torch.cuda.synchronize()
            assert int(sh.status.item()) == 0
            results[r] = (out, lse, si, ss)
        except BaseException as e:  # surfaced below; the barrier breaks the other threads
            errors.append(e)
            shared.bar.abort()

    threads = [threading.Thread(target=rank_main, args=(r,)) for r in range(world)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    if errors:
        raise errors[0]
    for out, lse, si, ss in results:
        np.testing.assert_array_equal(si.cpu().numpy(), si1.cpu().numpy())
        np.testing.assert_array_equal(ss.cpu().numpy(), ss1.cpu().numpy())
        assert (out.float() - out1.float()).abs().max().item() <= OUT_TOL
        assert (lse - lse1).abs().max().item() <= LSE_TOL
    return results


@pytest.mark.parametrize("world", [2, 4])
def test_shard_flat_dh64(world):
    cfg = cfg_of(n_heads=14, n_kv=2, head_dim=64, k_blocks=16)
    _run(cfg, B=4, n=8192, hier=False, world=world)


@pytest.mark.parametrize("world", [2, 4])
def test_shard_hier_dh128(world):
    cfg = cfg_of(n_heads=32, n_kv=8, head_dim=128, fanout=16, beam=8, k_blocks=16)
    _run(cfg, B=2, n=16384, hier=True, world=world)


def test_shard_window_straddles_ranks():
    # a context that ends 192 tokens past the last shard bound of an 8192-token
    # capacity: the window spans two ranks and the last rank holds few tokens
    cfg = cfg_of(n_heads=14, n_kv=2, head_dim=64, k_blocks=16)
    tok_lo, n_loc, n_total = shard_range(cfg, 8192, 3, 4, False)
    assert n_total == 8192 and tok_lo == 6144
    _run(cfg, B=2, n=tok_lo + 64 * 3, hier=False, world=4, cap=8192)


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("hier", [False, True])
def test_shard_trained_gains(world, hier):
    # trained QKNorm gains: every rank keeps a running maximum of its own
    # logits, so the partials carry different maxima and the finish merge
    # has to rescale them (the max-rescaled merge, not a plain sum)
    if hier:
        cfg = cfg_of(n_heads=32, n_kv=8, head_dim=128, fanout=16, beam=8, k_blocks=16)
        _run(cfg, B=2, n=16384, hier=True, world=world, seed=6, gains="trained")
    else:
        cfg = cfg_of(n_heads=14, n_kv=2, head_dim=64, k_blocks=16)
        _run(cfg, B=4, n=8192, hier=False, world=world, seed=6, gains="trained")
