"""The decode cache's chunk-tiled K / RoPE'd K / V layout (CPU).

Element (token t, dim d) of a (sequence, kv head) sits at
    ((t // 64) * (dh // 64) + d // 64) * 4096 + (t % 64) * 64
    + (((d % 64) // 8) ^ (t % 8)) * 8 + d % 8
of that head's [n_cap/64, dh/64, 64, 64] run: the 8 KB image a
128-byte-swizzled TMA box leaves in shared memory (the device helper
tiled_offset, which the append kernel writes and the decode kernels read).
HBADecodeCache.tokens() must invert it exactly."""

import types

import numpy as np
import torch

from hba_b200.cache import HBADecodeCache


def _tiled_offset(t, d, dh):
    return ((t // 64) * (dh // 64) + d // 64) * 4096 + (t % 64) * 64 + (((d % 64) // 8) ^ (t % 8)) * 8 + d % 8


def test_tokens_inverts_the_tiled_layout():
    rng = np.random.default_rng(0)
    for dh in (64, 128):
        B, Hkv, n = 2, 3, 192
        tok = rng.standard_normal((B, n, Hkv, dh)).astype(np.float32)
        flat = np.zeros(B * Hkv * n * dh, dtype=np.float32)
        t, d = np.meshgrid(np.arange(n), np.arange(dh), indexing="ij")
        off = _tiled_offset(t, d, dh)
        for b in range(B):
            for g in range(Hkv):
                base = (b * Hkv + g) * n * dh
                flat[base + off] = tok[b, :, g, :]
        tiled = torch.from_numpy(flat).view(B, Hkv, n // 64, dh // 64, 64, 64)
        got = HBADecodeCache.tokens(types.SimpleNamespace(k=tiled), "k").numpy()
        np.testing.assert_array_equal(got, tok)


def test_a_block_group_is_one_contiguous_8kb_tile():
    # rows of one 64-token block and 64-dim group cover exactly 4096 consecutive elements
    t, d = np.meshgrid(np.arange(64, 128), np.arange(64, 128), indexing="ij")
    off = _tiled_offset(t, d, 128)
    assert off.min() == (1 * 2 + 1) * 4096 and off.max() == (1 * 2 + 1) * 4096 + 4095
    assert len(np.unique(off)) == 4096
