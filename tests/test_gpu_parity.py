"""GPU parity: the CUDA path (through the C-ABI) against the oracle on the
same seeded inputs.  Selection must be index-exact (ties within 1e-6 logit
excepted), outputs within 2e-2 max-abs (bf16), LSE within 1e-3."""

import numpy as np
import pytest
import torch

import gpu_helpers as H
from hba_b200 import HBADecodeCache, hba_attention_b200, synth
from hba_b200.ops import build_super_b200, qknorm_b200, summarize_b200
from oracle import hba_oracle as orc

pytestmark = pytest.mark.gpu


# ------------------------------------------------------------ components ----
@pytest.mark.parametrize("dh", [64, 128])
def test_qknorm_kernel_matches_oracle(dh):
    g = torch.Generator(device="cuda").manual_seed(1)
    x = (torch.randn(37, 5, dh, generator=g, device="cuda") * 3 + 1).to(torch.bfloat16)
    gain = torch.rand(5, generator=g, device="cuda") + 0.5
    y = H.np32(qknorm_b200(x, gain))
    ref = orc.head_rmsnorm(H.np32(x), H.np32(gain), bf16=True)
    ulp = np.abs(ref) * 2.0 ** -7 + 1e-30
    assert (np.abs(y - ref) <= ulp).all()
    assert (y == ref).mean() > 0.99
    rms = np.sqrt((H.np32(qknorm_b200(x, gain)).astype(np.float64) ** 2).mean(-1))
    np.testing.assert_allclose(rms, np.broadcast_to(H.np32(gain), rms.shape), rtol=1e-2)


@pytest.mark.parametrize("dh,Bk,m", [(64, 64, 4), (128, 64, 4), (64, 32, 2), (128, 16, 8)])
def test_summaries_and_supers_match_oracle(dh, Bk, m):
    cfg = H.cfg_of(head_dim=dh, block=Bk, slots=m, n_heads=4, n_kv=2, fanout=4)
    g = torch.Generator(device="cuda").manual_seed(2)
    kc = torch.randn(2, 11 * Bk, 2, dh, generator=g, device="cuda").to(torch.bfloat16)
    summ, _ = synth.make_weights(cfg, "cuda", seed=3)
    S = summarize_b200(kc, summ.probes, summ.proj, cfg)
    ref = orc.summarize(H.np32(kc), H.np32(summ.probes), H.np32(summ.proj), Bk)
    err = np.abs(H.np32(S) - ref)
    assert (err <= np.abs(ref) * 2.0 ** -7 + 2e-3).all(), err.max()
    S1, ns = build_super_b200(S, cfg)
    assert ns == 3                                     # 11 blocks, fanout 4: partial last group
    ref1, _ = orc.build_super(H.np32(S), 4)
    err1 = np.abs(H.np32(S1) - ref1)
    assert (err1 <= np.abs(ref1) * 2.0 ** -7 + 1e-6).all(), err1.max()


# ---------------------------------------------------------------- decode ----
# hba_b200_decode has three paths: "tc" (one CTA per sequence and kv head,
# attention on tcgen05/TMEM, QKNorm only), "fused" (same shape on mma.sync) and
# "split" (selection kernels + stream-K attention); the library picks by batch
# size and config, HBA_B200_DECODE_PATH forces one so all are checked.
PATHS = ["split", "fused", "tc"]


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("hier", [False, True])
def test_decode_small_matches_oracle(hier, path, monkeypatch):
    monkeypatch.setenv("HBA_B200_DECODE_PATH", path)
    cfg = H.cfg_of(n_heads=8, n_kv=2, head_dim=128, fanout=8, beam=3) if hier else H.cfg_of()
    cache, wl, summ, qkn, cos, sin = H.build_cache(cfg, 3, 4096, hier, seed=11)
    H.check_decode(cache, wl["q"], cfg, hier, qkn, cos, sin)


def test_decode_paths_agree():
    """Both paths select the same blocks and agree on out/LSE (same scores)."""
    import os
    cfg = H.cfg_of(n_heads=32, n_kv=8, head_dim=128, fanout=16, beam=4)
    cache, wl, summ, qkn, cos, sin = H.build_cache(cfg, 4, 16384, True, seed=15)
    res = {}
    for path in PATHS:
        os.environ["HBA_B200_DECODE_PATH"] = path
        try:
            res[path] = cache.attend(wl["q"], return_lse=True, return_selection=True)
        finally:
            del os.environ["HBA_B200_DECODE_PATH"]
    o1, l1, (s1, _) = res["split"]
    for other in ("fused", "tc"):
        o2, l2, (s2, _) = res[other]
        assert torch.equal(s1, s2), other
        assert (o1.float() - o2.float()).abs().max().item() < 1e-2, other
        assert (l1 - l2).abs().max().item() < 1e-3, other


def test_decode_planted_blocks_are_selected():
    cfg = H.cfg_of()
    cache, wl, summ, qkn, cos, sin = H.build_cache(cfg, 4, 8192, False, seed=12, gains=False)
    _, _, (si, _) = H.check_decode(cache, wl["q"], cfg, False, qkn, cos, sin)
    sel = si.cpu().numpy()
    pl = wl["planted"].cpu().numpy()
    for b in range(4):
        for g in range(2):
            assert set(pl[b, g].tolist()) <= set(sel[b, g].tolist())


@pytest.mark.parametrize("path", PATHS)
def test_decode_ragged_lengths_and_edges(path, monkeypatch):
    """Ragged batch: a sequence shorter than the window (no candidates), one
    with fewer candidates than k, one shorter than the sink count, a full one."""
    monkeypatch.setenv("HBA_B200_DECODE_PATH", path)
    cfg = H.cfg_of()
    cache, wl, summ, qkn, cos, sin = H.build_cache(cfg, 5, 4096, False, seed=13)
    lens = np.array([4096, 300, 1024 + 64 * 5 + 7, 2, 1], dtype=np.int64)
    cache.lens.copy_(torch.tensor(lens, dtype=torch.int32))
    cache.lens_host = lens.copy()
    cache._refresh_scales()
    H.check_decode(cache, wl["q"], cfg, False, qkn, cos, sin)


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("variant", ["noqk", "inv_sqrt_d", "tau"])
def test_decode_scale_variants(variant, path, monkeypatch):
    monkeypatch.setenv("HBA_B200_DECODE_PATH", path)
    if variant == "noqk":
        cfg = H.cfg_of(qknorm=False)
    elif variant == "inv_sqrt_d":
        cfg = H.cfg_of(content_scale_mode="inv_sqrt_d")
    else:
        cfg = H.cfg_of(native_ctx=1024, n_heads=8, n_kv=2, head_dim=128)      # tau(4096) = 1 + 0.1 ln 4
    cache, wl, summ, qkn, cos, sin = H.build_cache(cfg, 2, 4096, False, seed=14)
    H.check_decode(cache, wl["q"], cfg, False, qkn, cos, sin)
    if path == "tc":  # without QKNorm too: the tensor-core kernel (running maximum from the first chunk)
        from hba_b200 import _lib
        cache.attend(wl["q"])
        assert b"decode_tc_kernel" in _lib.load().hba_b200_last_kernels()


def test_cache_incremental_append_matches_bulk():
    cfg = H.cfg_of(n_heads=8, n_kv=2, head_dim=128, fanout=4, beam=2)
    n = 640
    summ, qkn = synth.make_weights(cfg, "cuda", seed=5, gains=True)
    cos, sin = synth.rope_tables(n, 128, 1e6)
    wl = synth.decode_workload(cfg, 2, n, hier=True, seed=5, qkn=qkn)
    bulk = HBADecodeCache(cfg, 2, n, summ, qkn, cos, sin, hier=True)
    bulk.append(wl["k"], wl["v"])
    inc = HBADecodeCache(cfg, 2, n, summ, qkn, cos, sin, hier=True)
    for t0 in range(0, n, 37):
        t1 = min(n, t0 + 37)
        inc.append(wl["k"][:, t0:t1], wl["v"][:, t0:t1])
    torch.cuda.synchronize()
    for name in ("k", "kr", "v", "summaries", "supers"):
        assert torch.equal(getattr(bulk, name), getattr(inc, name)), name
    a = bulk.attend(wl["q"])
    b = inc.attend(wl["q"])
    assert torch.equal(a, b)


# --------------------------------------------------------------- prefill ----
# hba_b200_prefill runs the union softmax on the tcgen05 tensor cores ("tc")
# or with the per-query gather kernel ("gather"); HBA_B200_PREFILL_PATH
# selects one so both are checked (configurations outside the tensor-core
# envelope -- no QKNorm, block != 64, G < 4 -- always gather).
PREFILL_PATHS = ["gather", "tc"]


@pytest.mark.parametrize("path", PREFILL_PATHS)
@pytest.mark.parametrize("hier", [False, True])
def test_prefill_cfg0_shape_matches_oracle(hier, path, monkeypatch):
    monkeypatch.setenv("HBA_B200_PREFILL_PATH", path)
    cfg = H.cfg_of(fanout=8, beam=4) if hier else H.cfg_of()
    rows = H.sample_rows(2048, 48, seed=1)
    H.check_prefill(cfg, 1, 2048, hier, seed=21, rows=rows)


@pytest.mark.parametrize("path", PREFILL_PATHS)
def test_prefill_dh128_gqa4_matches_oracle(path, monkeypatch):
    monkeypatch.setenv("HBA_B200_PREFILL_PATH", path)
    cfg = H.cfg_of(n_heads=32, n_kv=8, head_dim=128)
    rows = H.sample_rows(2048, 24, seed=2)
    H.check_prefill(cfg, 2, 2048, False, seed=22, rows=rows)


@pytest.mark.parametrize("path", PREFILL_PATHS)
def test_prefill_without_qknorm(path, monkeypatch):
    # no QKNorm: no logit bound, so the tensor-core union keeps a running maximum from the first chunk
    monkeypatch.setenv("HBA_B200_PREFILL_PATH", path)
    cfg = H.cfg_of(qknorm=False)
    rows = H.sample_rows(2048, 48, seed=3)
    H.check_prefill(cfg, 1, 2048, False, seed=24, rows=rows)
    if path == "tc":
        from hba_b200 import _lib
        assert b"prefill_tc_kernel" in _lib.load().hba_b200_last_kernels()


@pytest.mark.parametrize("path", PREFILL_PATHS)
def test_prefill_short_sequence_no_candidates(path, monkeypatch):
    monkeypatch.setenv("HBA_B200_PREFILL_PATH", path)
    cfg = H.cfg_of()
    H.check_prefill(cfg, 1, 512, False, seed=23, rows=np.arange(512))


def test_prefill_paths_agree_on_every_row():
    """Tensor-core and gather paths: same selection, outputs within bf16 noise, all rows."""
    import os
    cfg = H.cfg_of(n_heads=32, n_kv=8, head_dim=128)
    n = 4096
    summ, qkn = synth.make_weights(cfg, "cuda", seed=25, gains=True)
    cos, sin = synth.rope_tables(n, 128, 1e6)
    wl = synth.prefill_workload(cfg, 2, n, seed=25)
    res = {}
    for path in PREFILL_PATHS:
        os.environ["HBA_B200_PREFILL_PATH"] = path
        try:
            with torch.no_grad():
                res[path] = hba_attention_b200(wl["q"], wl["k"], wl["v"], cos, sin, cfg, summ, qkn,
                                               return_lse=True, return_selection=True)
        finally:
            del os.environ["HBA_B200_PREFILL_PATH"]
    (o1, l1, (s1, _)), (o2, l2, (s2, _)) = res["gather"], res["tc"]
    assert torch.equal(s1, s2)
    assert (o1.float() - o2.float()).abs().max().item() < 2e-2
    assert (l1 - l2).abs().max().item() < 1e-3


@pytest.mark.parametrize("dh,heads,slots,n,block,window", [(128, (32, 8), 4, 4096, 64, 1024),
                                                             (64, (14, 2), 4, 3072, 64, 1024),
                                                             (64, (8, 2), 8, 2048, 64, 1024),
                                                             (128, (16, 4), 2, 1536, 64, 1024),
                                                             (64, (4, 2), 4, 400, 16, 64)])
def test_prefill_selection_paths_agree_on_every_row(dh, heads, slots, n, block, window):
    """The three prefill selections on every row: the query-tiled CUDA-core
    kernel equals the per-query scan bit for bit (same fp32 fma order); the
    tcgen05 selection GEMM (the default) sums the same exact bf16 products in
    the tensor core's order, so its picks equal the scan's up to the 1e-6 tie
    rule and its scores agree to 1e-5 relative (the block-16 case leaves a
    partial last tile)."""
    import os
    from hba_b200 import _lib
    cfg = H.cfg_of(n_heads=heads[0], n_kv=heads[1], head_dim=dh, slots=slots, block=block, window=window,
                   sinks=min(4, block))
    summ, qkn = synth.make_weights(cfg, "cuda", seed=31, gains=True)
    cos, sin = synth.rope_tables(n, dh, 1e6)
    wl = synth.prefill_workload(cfg, 2, n, seed=31)
    res, kern = {}, {}
    for path in ("scan", "tile", "tc"):
        if path != "tc":
            os.environ["HBA_B200_SELECT_PATH"] = path
        try:
            with torch.no_grad():
                res[path] = hba_attention_b200(wl["q"], wl["k"], wl["v"], cos, sin, cfg, summ, qkn,
                                               return_lse=True, return_selection=True)
            kern[path] = _lib.load().hba_b200_last_kernels().decode()
        finally:
            os.environ.pop("HBA_B200_SELECT_PATH", None)
    assert "select_tc_kernel" in kern["tc"] and "select_tile_kernel" in kern["tile"]
    (_, _, (i1, s1)), (_, _, (i2, s2)), (_, _, (i3, s3)) = res["scan"], res["tile"], res["tc"]
    assert torch.equal(i1, i2)
    assert torch.equal(s1, s2)
    H.assert_picks_agree(i1, s1, i3, s3)


@pytest.mark.parametrize("dh,heads,n,fanout,beam", [(64, (14, 2), 4096, 16, 4), (128, (32, 8), 8192, 16, 8),
                                                     (64, (8, 2), 2048, 1, 4)])
def test_prefill_hier_selection_tc_matches_scan(dh, heads, n, fanout, beam):
    """Hierarchical prefill selection: the two tensor-core passes (supers, then
    the beam's children) against the per-query CUDA-core kernels: the same
    picks up to the 1e-6 tie rule, scores within 1e-5 (fanout 1: super 0 is
    block 0 alone, never a candidate)."""
    import os
    from hba_b200 import _lib
    cfg = H.cfg_of(n_heads=heads[0], n_kv=heads[1], head_dim=dh, fanout=fanout, beam=beam)
    summ, qkn = synth.make_weights(cfg, "cuda", seed=33, gains=True)
    cos, sin = synth.rope_tables(n, dh, 1e6)
    wl = synth.prefill_workload(cfg, 2, n, seed=33)
    res, kern = {}, {}
    for path in ("scan", "tc"):
        if path != "tc":
            os.environ["HBA_B200_SELECT_PATH"] = path
        try:
            with torch.no_grad():
                res[path] = hba_attention_b200(wl["q"], wl["k"], wl["v"], cos, sin, cfg, summ, qkn, hier=True,
                                               return_lse=True, return_selection=True)
            kern[path] = _lib.load().hba_b200_last_kernels().decode()
        finally:
            os.environ.pop("HBA_B200_SELECT_PATH", None)
    assert "select_tc_kernel+select_tc_kernel" in kern["tc"] and "select_tc" not in kern["scan"]
    (o1, l1, (i1, s1)), (o2, l2, (i2, s2)) = res["scan"], res["tc"]
    H.assert_picks_agree(i1, s1, i2, s2)
    if torch.equal(i1, i2):
        assert (o1.float() - o2.float()).abs().max().item() < 2e-2


def test_prefill_tiny_blocks_and_knobs():
    """Block 16, window 64, 2 sinks, k 4, 2 slots (the reference's test knobs)."""
    cfg = H.cfg_of(block=16, window=64, sinks=2, k_blocks=4, slots=2, fanout=4, beam=2, n_heads=4, n_kv=2)
    for hier in (False, True):
        H.check_prefill(cfg, 2, 384, hier, seed=24, rows=np.arange(384))


def test_prefill_rejects_non_block_multiple():
    cfg = H.cfg_of()
    summ, qkn = synth.make_weights(cfg, "cuda")
    q = torch.zeros(1, 100, 14, 64, device="cuda", dtype=torch.bfloat16)
    k = torch.zeros(1, 100, 2, 64, device="cuda", dtype=torch.bfloat16)
    cos, sin = synth.rope_tables(100, 64, 1e6)
    with pytest.raises(AssertionError):
        hba_attention_b200(q, k, k, cos, sin, cfg, summ, qkn)


def test_prefill_causality():
    """Outputs at positions <= t must not change when tokens > t change
    (reference gate_causality, gates.py:101-126), flat selection."""
    cfg = H.cfg_of()
    n, t = 2048, 1500
    summ, qkn = synth.make_weights(cfg, "cuda", seed=7, gains=True)
    cos, sin = synth.rope_tables(n, 64, 1e6)
    wl = synth.prefill_workload(cfg, 1, n, seed=7)
    q, k, v = wl["q"], wl["k"], wl["v"]
    g = torch.Generator(device="cuda").manual_seed(8)
    q2, k2, v2 = q.clone(), k.clone(), v.clone()
    q2[:, t + 1:] = torch.randn(q2[:, t + 1:].shape, generator=g, device="cuda").to(q.dtype)
    k2[:, t + 1:] = torch.randn(k2[:, t + 1:].shape, generator=g, device="cuda").to(k.dtype)
    v2[:, t + 1:] = torch.randn(v2[:, t + 1:].shape, generator=g, device="cuda").to(v.dtype)
    with torch.no_grad():
        o1 = hba_attention_b200(q, k, v, cos, sin, cfg, summ, qkn)
        o2 = hba_attention_b200(q2, k2, v2, cos, sin, cfg, summ, qkn)
    assert torch.equal(o1[:, :t + 1], o2[:, :t + 1])
    assert not torch.equal(o1[:, t + 1:], o2[:, t + 1:])


def test_decode_equals_prefill_last_row():
    cfg = H.cfg_of(n_heads=8, n_kv=2, head_dim=128)
    n = 3072
    summ, qkn = synth.make_weights(cfg, "cuda", seed=9, gains=True)
    cos, sin = synth.rope_tables(n, 128, 1e6)
    wl = synth.prefill_workload(cfg, 2, n, seed=9)
    with torch.no_grad():
        out, lse, (si, ss) = hba_attention_b200(wl["q"], wl["k"], wl["v"], cos, sin, cfg, summ, qkn,
                                                return_lse=True, return_selection=True)
    cache = HBADecodeCache(cfg, 2, n, summ, qkn, cos, sin)
    cache.append(wl["k"], wl["v"])
    o2, l2, (si2, ss2) = cache.attend(wl["q"][:, -1], return_lse=True, return_selection=True)
    H.assert_picks_agree(si[:, :, -1], ss[:, :, -1], si2, ss2)   # tensor-core vs CUDA-core scores
    assert (out[:, -1].float() - o2.float()).abs().max().item() < 1e-2
    assert (lse[:, :, -1] - l2).abs().max().item() < 1e-4


# ------------------------------------------------- BASELINE full sizes ------
def test_baseline_cfg1_decode_full_size():
    """B64 x 32K context, 14/2 heads, dh 64, flat top-16: every sequence's 8
    planted blocks selected; 16 sampled sequences checked against the oracle."""
    cfg = H.cfg_of()
    cache, wl, summ, qkn, cos, sin = H.build_cache(cfg, 64, 32768, False, seed=31, gains=False)
    out, (si, _) = cache.attend(wl["q"], return_selection=True)
    assert torch.isfinite(out.float()).all()
    sel = si.cpu().numpy()
    pl = wl["planted"].cpu().numpy()
    assert all(set(pl[b, g]) <= set(sel[b, g]) for b in range(64) for g in range(2))
    H.check_decode(cache, wl["q"], cfg, False, qkn, cos, sin, rows=range(0, 64, 4))


def test_baseline_cfg3_hier_decode_full_size():
    """B32 x 128K context, 32/8 heads, dh 128, beam 8 over 128 supers, tau active."""
    cfg = H.cfg_of(n_heads=32, n_kv=8, head_dim=128, fanout=16, beam=8)
    cache, wl, summ, qkn, cos, sin = H.build_cache(cfg, 32, 131072, True, seed=33, gains=False)
    out, (si, _) = cache.attend(wl["q"], return_selection=True)
    assert torch.isfinite(out.float()).all()
    sel = si.cpu().numpy()
    pl = wl["planted"].cpu().numpy()
    assert all(set(pl[b, g]) <= set(sel[b, g]) for b in range(32) for g in range(8))
    H.check_decode(cache, wl["q"], cfg, True, qkn, cos, sin, rows=[0, 13, 31])


def test_baseline_cfg2_prefill_full_size_sampled_rows():
    """B4 x 32K, 32/8 heads, dh 128: 24 sampled query rows per sequence against
    the oracle; all outputs finite."""
    cfg = H.cfg_of(n_heads=32, n_kv=8, head_dim=128)
    rows = H.sample_rows(32768, 16, seed=3)
    eo, el, out, lse, _ = H.check_prefill(cfg, 4, 32768, False, seed=32, rows=rows, gains=False)
    assert torch.isfinite(out.float()).all() and torch.isfinite(lse).all()


@pytest.mark.parametrize("hier", [False, True])
def test_decode_zero_copy_host_io(hier):
    # q read from, out / lse written to mapped pinned host memory by the
    # decode kernel itself: the same bytes as the device-buffer decode
    from hba_b200.hostio import MappedHostBuffer
    cfg = H.cfg_of(n_heads=14, n_kv=2, head_dim=64) if not hier else \
        H.cfg_of(n_heads=32, n_kv=8, head_dim=128, fanout=16, beam=8)
    B, n = 8, 4096 + 37
    summ, qkn = synth.make_weights(cfg, "cuda", seed=11, gains=True)
    cos, sin = synth.rope_tables(n + cfg.block, cfg.head_dim, 1e6)  # the cache rounds its capacity up to a block
    wl = synth.decode_workload(cfg, B, n, hier=hier, seed=11, qkn=qkn, planted=8)
    cache = HBADecodeCache(cfg, B, n, summ, qkn, cos, sin, hier=hier)
    cache.append(wl["k"], wl["v"])
    q = wl["q"].contiguous()
    out_d, lse_d = cache.attend(q, return_lse=True)
    qb, ob, lb = q.numel() * 2, q.numel() * 2, B * cfg.n_heads * 4
    buf = MappedHostBuffer(qb + ob + lb)
    try:
        buf.host_view(torch.bfloat16, q.shape).copy_(q.cpu())
        out_h = buf.host_view(torch.bfloat16, q.shape, offset=qb)
        lse_h = buf.host_view(torch.float32, (B, cfg.n_heads), offset=qb + ob)
        out_h.zero_()
        lse_h.zero_()
        cache.decode_into(buf.device_view(0), buf.device_view(qb), buf.device_view(qb + ob))
        torch.cuda.synchronize()
        assert torch.equal(out_h, out_d.cpu())
        assert torch.equal(lse_h, lse_d.cpu())
        assert cache.device_status() == 0
    finally:
        buf.close()
