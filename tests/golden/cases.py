"""Seeded golden cases for the HBA hot path.

The inputs of every case are regenerated from a numpy PCG64 seed (stable
across numpy versions and machines), so only the reference's OUTPUTS are
committed (``*.npz`` beside this file, written by ``make_golden.py``, which
runs the reference implementation itself).  Both the generator and the tests
import this module, so the two sides always see identical inputs.
"""

import numpy as np


def rng(seed):
    return np.random.default_rng(seed)


def randn(r, *shape, scale=1.0):
    return (r.standard_normal(shape, dtype=np.float32) * np.float32(scale)).astype(np.float32)


# Tiny config: the reference's own unit-test knobs (tests/test_qknorm.py:28-35).
TINY = dict(n_heads=4, n_kv=2, head_dim=8, block=16, window=64, sinks=2, k_blocks=4, slots=2,
            fanout=4, beam=2, native_ctx=8192, rope_theta=1_000_000.0, content_scale_mode="inv_d",
            temp_c=0.1, n_cal=None)

# BASELINE config 0 geometry (CPU naive-oracle case): 14/2 heads, dh 64, block 64,
# window 1024, sinks 4, top-16, 4 slots.
CFG0 = dict(n_heads=14, n_kv=2, head_dim=64, block=64, window=1024, sinks=4, k_blocks=16, slots=4,
            fanout=16, beam=4, native_ctx=32768, rope_theta=1_000_000.0, content_scale_mode="inv_d",
            temp_c=0.1, n_cal=None)


def summarizer_params(r, Hkv, m, dh):
    """Reference init distribution (summarizer.py:25,31-32): probes ~ N(0, 1/dh),
    proj = I + 0.02 N(0,1)."""
    probes = randn(r, Hkv, m, dh, scale=dh ** -0.5)
    proj = (np.eye(dh, dtype=np.float32)[None] + randn(r, Hkv, dh, dh, scale=0.02)).astype(np.float32)
    return probes, proj


def eval_case_inputs(cfg, n, seed, B=1):
    r = rng(seed)
    Hq, Hkv, dh = cfg["n_heads"], cfg["n_kv"], cfg["head_dim"]
    q = randn(r, B, n, Hq, dh)
    k = randn(r, B, n, Hkv, dh)
    v = randn(r, B, n, Hkv, dh)
    probes, proj = summarizer_params(r, Hkv, cfg["slots"], dh)
    q_gain = r.uniform(0.6, 1.6, Hq).astype(np.float32)
    k_gain = r.uniform(0.6, 1.6, Hkv).astype(np.float32)
    return dict(q=q, k=k, v=v, probes=probes, proj=proj, q_gain=q_gain, k_gain=k_gain)


# (name, cfg, n, seed, qknorm, hier, rows) -- rows=None: store all rows.
EVAL_CASES = [
    ("tiny_flat_qk", TINY, 256, 11, True, False, None),
    ("tiny_flat_noqk", TINY, 256, 12, False, False, None),
    ("tiny_hier_qk", TINY, 384, 13, True, True, None),
    ("tiny_short_qk", TINY, 48, 14, True, False, None),          # n < W: zero routed candidates
    ("cfg0_flat_2048", CFG0, 2048, 21, True, False, "sample"),
    ("cfg0_hier_2048", CFG0, 2048, 22, True, True, "sample"),
]


def sample_rows(n, count=48, seed=0):
    """Deterministic row sample: the first and last few positions plus a spread."""
    r = rng(1000 + seed)
    fixed = {0, 1, 2, 3, 4, n // 2, n - 2, n - 1}
    extra = set(r.choice(n, size=min(n, count), replace=False).tolist())
    return np.array(sorted(fixed | extra), dtype=np.int64)


def rows_for(case):
    name, cfg, n, seed, qk, hier, rows = case
    if rows is None:
        return np.arange(n, dtype=np.int64)
    return sample_rows(n, seed=seed)


def cfg_dict(cfg, qknorm):
    d = dict(cfg)
    d["qknorm"] = qknorm
    return d


# Backward cases: gradients of sum(out * dout) through the reference's dense
# training path (attention.py:306-389), fp32 autograd.  BWD64 has the
# tensor-core kernels' geometry (block 64, dh 64, G = 4) at a size the dense
# path runs on a CPU in seconds.
BWD64 = dict(n_heads=8, n_kv=2, head_dim=64, block=64, window=256, sinks=4, k_blocks=4, slots=4,
             fanout=16, beam=4, native_ctx=32768, rope_theta=1_000_000.0, content_scale_mode="inv_d",
             temp_c=0.1, n_cal=None)

# (name, cfg, n, seed, qknorm)
BWD_CASES = [
    ("tiny_qk", TINY, 256, 31, True),
    ("tiny_noqk", TINY, 256, 32, False),
    ("g4d64_qk", BWD64, 512, 33, True),
]


def bwd_rows(n, seed):
    """The query and key rows a backward fixture stores (all of a tiny case;
    a sample, sinks and the last rows included, of a larger one)."""
    if n <= 256:
        a = np.arange(n, dtype=np.int64)
        return a, a
    return sample_rows(n, count=64, seed=seed), sample_rows(n, count=96, seed=seed + 1)


def bwd_case_inputs(cfg, n, seed, B=1):
    """Forward inputs as ``eval_case_inputs``, rounded to bf16 values (so a
    bf16 device path consumes the same numbers), plus the output gradient."""
    inp = eval_case_inputs(cfg, n, seed, B)
    for k in ("q", "k", "v"):
        inp[k] = _bf16_values(inp[k])
    r = rng(seed + 500)
    inp["dout"] = _bf16_values(randn(r, B, n, cfg["n_heads"], cfg["head_dim"]))
    return inp


def _bf16_values(a):
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    lsb = (u >> np.uint64(16)) & np.uint64(1)
    return ((u + np.uint64(0x7FFF) + lsb) & np.uint64(0xFFFF0000)).astype(np.uint32).view(np.float32).reshape(
        np.shape(a))


# Aux-KL cases (teacher pstar, route_topk's block scores, the dense path's
# aux and its summarizer gradients): (name, cfg, n, seed, qknorm)
AUX_CASES = [
    ("tiny_qk", TINY, 256, 41, True),
    ("g4d64_qk", BWD64, 512, 42, True),
    ("g4d64_noqk", BWD64, 512, 43, False),
]
