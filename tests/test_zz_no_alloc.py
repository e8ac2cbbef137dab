"""The allocation-free decode entry point (hba_b200_decode_noalloc), for
callers that cannot allocate device memory when they decode.  It must give the
same result as hba_b200_decode with a caller workspace, on consecutive calls
that share its fixed scratch array.  Collected last on purpose: a failure here
leaves every other test already run."""

import ctypes

import numpy as np
import pytest
import torch

import gpu_helpers as H
from hba_b200 import _lib
from hba_b200.attention import ptr, stream_of

pytestmark = pytest.mark.gpu


def _noalloc(cache, q, out, lse, si, ss):
    st = _lib.load().hba_b200_decode_noalloc(
        ctypes.byref(cache.c), cache.B, cache.n_cap, ptr(cache.lens), ptr(cache.scales), ptr(q), ptr(cache.q_gain),
        ptr(cache.k_gain), ptr(cache.k), ptr(cache.kr), ptr(cache.v), ptr(cache.summaries), ptr(cache.supers), ptr(cache.cos),
        ptr(cache.sin),
        ptr(out), ptr(lse), ptr(si), ptr(ss), stream_of(cache.device))
    _lib.check(st, "hba_b200_decode_noalloc")


@pytest.mark.parametrize("path", ["split", "fused", "tc"])
@pytest.mark.parametrize("hier", [False, True])
def test_noalloc_decode_matches_workspace_decode_on_two_calls(hier, path, monkeypatch):
    # every decode path, forced (the library reads the variable on each call):
    # the small batch here would otherwise always take the tensor-core path
    monkeypatch.setenv("HBA_B200_DECODE_PATH", path)
    cfg = H.cfg_of(n_heads=8, n_kv=2, head_dim=128, fanout=8, beam=4) if hier else H.cfg_of()
    cache, wl, summ, qkn, cos, sin = H.build_cache(cfg, 4, 4096, hier, seed=41)
    ref_out, ref_lse, (ref_si, ref_ss) = cache.attend(wl["q"], return_lse=True, return_selection=True)
    q2 = torch.randn(wl["q"].shape, device="cuda").to(torch.bfloat16)      # a different second query
    ref2 = cache.attend(q2, return_lse=True, return_selection=True)
    for q, (ro, rl, (rsi, rss)) in ((wl["q"], (ref_out, ref_lse, (ref_si, ref_ss))), (q2, ref2)):
        out = torch.empty_like(q)
        lse = torch.empty(cache.B, cfg.n_heads, dtype=torch.float32, device="cuda")
        si = torch.empty(cache.B, cfg.n_kv, cfg.k_blocks, dtype=torch.int32, device="cuda")
        ss = torch.empty_like(si, dtype=torch.float32)
        _noalloc(cache, q.contiguous(), out, lse, si, ss)
        torch.cuda.synchronize()
        assert torch.equal(si, rsi)
        assert (out.float() - ro.float()).abs().max().item() <= H.OUT_TOL
        assert (lse - rl).abs().max().item() <= H.LSE_TOL
    # the status word inside the scratch array, read through its own entry point
    L = _lib.load()
    assert L.hba_b200_decode_noalloc_status(0, stream_of(cache.device)) == _lib.OK


def test_noalloc_rejects_requests_beyond_its_scratch():
    cfg = H.cfg_of(n_heads=32, n_kv=8, head_dim=128)
    c = _lib.Config(n_heads=32, n_kv=8, head_dim=128, block=64, window=1024, sinks=4, k_blocks=16, slots=4,
                    fanout=16, beam=4, hier=0, qknorm=1, eps=1e-6)
    L = _lib.load()
    big_batch = 4096
    assert L.hba_b200_decode_workspace_size(ctypes.byref(c), big_batch, 131072) > (8 << 20)
    one = ctypes.c_void_p(16)
    st = L.hba_b200_decode_noalloc(ctypes.byref(c), big_batch, 131072, one, one, one, one, one, one, one, one, one,
                                   None, one, one, one, None, None, None, None)
    assert st == _lib.ERR_WORKSPACE
    del cfg
