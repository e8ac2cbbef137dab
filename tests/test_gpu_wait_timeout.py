"""The bounded device waits turn a missing peer into a status, not a hang.

One GPU runs the fused sharded decode kernel as rank 0 of a world of 2 whose
rank 1 never launches: rank 1's slots in rank 0's exchange buffer stay zero,
so the first wait on them (the list exchange) gives up after the kernels'
limit for waits on another rank (2 s of the global timer), sets the status
word to 1, and the launch waits no more: the kernel returns.  The host reads HBA_B200_ERR_DEVICE_TIMEOUT
through hba_b200_device_status, and the context stays usable: a normal decode
afterwards gives the oracle's result.  No kernel waits on another launch: the
flag the wait polls is simply never written."""

import ctypes
import time

import pytest
import torch

import gpu_helpers as H
from hba_b200 import HBADecodeCache, _lib, synth
from hba_b200.attention import ptr, stream_of

pytestmark = pytest.mark.gpu


def test_missing_peer_expires_into_device_timeout_status():
    cfg = H.cfg_of()
    B, n_loc, n_glob = 2, 2048, 4096
    summ, qkn = synth.make_weights(cfg, "cuda", seed=71, gains=True)
    cos, sin = synth.rope_tables(n_glob, cfg.head_dim, 1e6)
    wl = synth.decode_workload(cfg, B, n_glob, seed=71, qkn=qkn)
    loc = HBADecodeCache(cfg, B, n_loc, summ, qkn, cos, sin)   # rank 0's tokens [0, 2048)
    loc.append(wl["k"][:, :n_loc], wl["v"][:, :n_loc])
    L = _lib.load()
    xbytes = L.hba_b200_shard_xbuf_bytes(ctypes.byref(loc.c), B, 2)
    assert xbytes > 0
    own = torch.zeros(xbytes, dtype=torch.uint8, device="cuda")
    absent = torch.zeros(xbytes, dtype=torch.uint8, device="cuda")  # stands in for the peer's buffer
    xbufs = (ctypes.c_void_p * 2)(own.data_ptr(), absent.data_ptr())
    epoch = torch.zeros(1, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    glens = torch.full((B,), n_glob, dtype=torch.int32, device="cuda")
    scales = torch.full((B,), H.scale_of(cfg, n_glob), dtype=torch.float32, device="cuda")
    q = wl["q"].contiguous()
    out = torch.empty_like(q)
    lse = torch.empty(B, cfg.n_heads, dtype=torch.float32, device="cuda")
    gcos = cos.float().contiguous()
    gsin = sin.float().contiguous()
    torch.cuda.synchronize()
    t0 = time.time()
    st = L.hba_b200_decode_shard_fused(
        ctypes.byref(loc.c), B, n_loc, 0, 2, 0, xbufs, ptr(epoch), ptr(glens), ptr(scales), ptr(q),
        ptr(loc.q_gain), ptr(loc.k_gain), ptr(loc.summaries), ptr(loc.supers), ptr(loc.k), ptr(loc.kr),
        ptr(loc.v), ptr(gcos), ptr(gsin), ptr(out), ptr(lse), None, None, ptr(status), stream_of(loc.device))
    assert st == _lib.OK                      # the launch itself is fine
    dst = L.hba_b200_device_status(ptr(status), 0, stream_of(loc.device))
    elapsed = time.time() - t0
    assert dst == _lib.ERR_DEVICE_TIMEOUT, _lib.status_string(dst)
    assert int(status.item()) == 1
    assert elapsed < 30, elapsed              # bounded: one expired 2 s wait, not a hang
    # the clear flag zeroes the word; the context is still usable
    assert L.hba_b200_device_status(ptr(status), 1, stream_of(loc.device)) == _lib.ERR_DEVICE_TIMEOUT
    assert L.hba_b200_device_status(ptr(status), 0, stream_of(loc.device)) == _lib.OK
    full, wl2, _, qkn2, cos2, sin2 = H.build_cache(cfg, B, 4096, False, seed=72)
    H.check_decode(full, wl2["q"], cfg, False, qkn2, cos2, sin2)


def test_python_layer_raises_on_a_timed_out_status():
    # the decode cache's status check maps a set word to HBAError(ERR_DEVICE_TIMEOUT)
    cfg = H.cfg_of()
    cache, wl, *_ = H.build_cache(cfg, 2, 2048, False, seed=73)
    cache.workspace[:4].view(torch.int32).fill_(1)   # as a kernel whose wait expired leaves it
    with pytest.raises(_lib.HBAError) as e:
        cache.attend(wl["q"])
    assert e.value.status == _lib.ERR_DEVICE_TIMEOUT
    assert cache.device_status(clear=True) == 1
    cache.attend(wl["q"])                            # cleared: the next step checks clean
