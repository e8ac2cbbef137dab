"""KV / summary cache and the incremental decode API.

The reference has no KV cache: every ``HBAModel.forward`` recomputes QKNorm
and every block summary over the whole sequence (src/hba/attention.py:631,
:659).  ``HBADecodeCache`` keeps, per layer, the state that call rebuilds and
updates it incrementally, so one decode step reads only what the union
softmax needs (~2.1K keys + the candidate summaries):

* ``k``        QKNorm'd NoPE keys, chunk-tiled: [B, Hkv, n_cap/64, dh/64, 64, 64]
                 bf16, per 64-token block and 64-dim group the 8 KB image a
                 128-byte-swizzled TMA box leaves in shared memory (16-byte
                 unit u of row r at unit u ^ (r % 8)), so the decode kernel
                 moves a block with one 1-D bulk copy; ``tokens("k")`` gives
                 the token-major [B, n_cap, Hkv, dh] view
* ``kr``       the same keys RoPE'd at their positions (written once at
                 append time, read for the window), same layout
* ``v``        the values, same layout
* ``summaries``[B, Hkv, n_cap/block, m, dh] bf16 -- slot summaries of complete blocks
* ``supers``   [B, Hkv, ceil(nb/F), m, dh] bf16 -- hierarchical mode only
* ``lens``     [B] int32 -- tokens held per sequence (ragged batches allowed)

Decoding the token at position n-1 of a length-n context gives the last row
of ``hba_attention_eval`` at length n (with that call's tau(n)).
"""

import ctypes

import numpy as np
import torch

from . import _lib
from .attention import (as_bf16, as_f32, c_config, gains, ptr, stream_of, summarizer_weights, union_scale)

BF16 = torch.bfloat16


class HBADecodeCache:
    """`pos_offset`: global position of cache row 0 (a KV-range shard holding
    tokens [pos_offset, pos_offset + max_len) of every sequence; its keys are
    RoPE'd at their global positions)."""

    def __init__(self, cfg, batch, max_len, summ, qkn, cos, sin, device="cuda", hier=False, pos_offset=0):
        self.cfg = cfg
        self.hier = bool(hier)
        self.B = int(batch)
        Bk = cfg.block
        unit = Bk * 64 // np.gcd(Bk, 64)  # whole blocks and whole 64-token cache tiles
        self.n_cap = -(-int(max_len) // unit) * unit
        self.nb_cap = self.n_cap // Bk
        self.ns_cap = -(-self.nb_cap // cfg.fanout) if self.hier else 0
        self.device = torch.device(device)
        H, Hkv, dh, m = cfg.n_heads, cfg.n_kv, cfg.head_dim, cfg.slots
        self.pos_offset = int(pos_offset)
        if cos.shape[0] < self.pos_offset + self.n_cap:
            raise ValueError(f"RoPE tables cover {cos.shape[0]} positions < cache end "
                             f"{self.pos_offset + self.n_cap}")
        dev = self.device
        self.c = c_config(cfg, self.hier)
        self.k = torch.zeros(self.B, Hkv, self.n_cap // 64, dh // 64, 64, 64, dtype=BF16, device=dev)
        self.kr = torch.zeros_like(self.k)
        self.v = torch.zeros_like(self.k)
        self.summaries = torch.zeros(self.B, Hkv, self.nb_cap, m, dh, dtype=BF16, device=dev)
        self.supers = (torch.zeros(self.B, Hkv, max(1, self.ns_cap), m, dh, dtype=BF16, device=dev)
                       if self.hier else None)
        self.cos = as_f32(cos[self.pos_offset: self.pos_offset + self.n_cap], dev)
        self.sin = as_f32(sin[self.pos_offset: self.pos_offset + self.n_cap], dev)
        self.q_gain, self.k_gain = gains(qkn, dev)
        self.probes, self.proj = summarizer_weights(summ, dev)
        self.lens = torch.zeros(self.B, dtype=torch.int32, device=dev)
        self.lens_host = np.zeros(self.B, dtype=np.int64)
        self.scales = torch.zeros(self.B, dtype=torch.float32, device=dev)
        L = _lib.load()
        self.ws_bytes = L.hba_b200_decode_workspace_size(ctypes.byref(self.c), self.B, self.n_cap)
        if self.ws_bytes == 0:
            _lib.check(_lib.ERR_UNSUPPORTED, "hba_b200_decode_workspace_size")
        self.workspace = torch.empty(self.ws_bytes, dtype=torch.uint8, device=dev)
        self.workspace[:256].zero_()  # sticky device status word (see device_status)

    # ---------------------------------------------------------------- state --

    def tokens(self, name):
        """The cache tensor `name` ("k", "kr" or "v") un-tiled: a token-major
        [B, n_cap, Hkv, dh] copy (for inspection and tests)."""
        t = getattr(self, name)
        B, Hkv, nblk, groups, R, C = t.shape
        x = t.reshape(B, Hkv, nblk, groups, R, 8, 8)
        r = torch.arange(R, device=t.device)
        u = torch.arange(8, device=t.device)
        phys = u[None, :] ^ (r[:, None] & 7)  # where logical unit u of row r sits
        idx = phys[None, None, None, None, :, :, None].expand(B, Hkv, nblk, groups, R, 8, 8)
        x = torch.gather(x, 5, idx).reshape(B, Hkv, nblk, groups, R, C)
        return x.permute(0, 2, 4, 1, 3, 5).reshape(B, nblk * R, Hkv, groups * C)
    def _refresh_scales(self):
        dh = self.cfg.head_dim
        s = [union_scale(self.cfg, dh, max(1, int(n))) for n in self.lens_host]
        self.scales.copy_(torch.tensor(s, dtype=torch.float32), non_blocking=False)

    def append(self, k_new, v_new):
        """Append t tokens to every sequence: k_new, v_new [B, t, Hkv, dh] raw
        projections.  QKNorm'd keys and values are written at each sequence's
        current length; summaries (and supers) of blocks that complete are rebuilt."""
        B, t = k_new.shape[:2]
        if B != self.B:
            raise ValueError("batch mismatch")
        if (self.lens_host + t > self.n_cap).any():
            raise ValueError(f"cache capacity {self.n_cap} exceeded")
        with torch.cuda.device(self.device):
            kb, vb = as_bf16(k_new), as_bf16(v_new)
            st = _lib.load().hba_b200_append_kv(
                ctypes.byref(self.c), self.B, self.n_cap, int(t), ptr(self.lens), ptr(kb), ptr(vb), ptr(self.k_gain),
                ptr(self.cos), ptr(self.sin), ptr(self.probes), ptr(self.proj), ptr(self.k), ptr(self.kr),
                ptr(self.v), ptr(self.summaries), ptr(self.supers), stream_of(self.device))
            _lib.check(st, "hba_b200_append_kv")
            self.lens += t
        self.lens_host += t
        self._refresh_scales()

    def attend(self, q, return_lse=False, return_selection=False, check_status=True):
        """Decode attention for the newest token of every sequence.
        q: [B, Hq, dh] (or [B, 1, Hq, dh]) raw query.  Returns out [B, Hq, dh]
        (q's dtype), plus lse [B, Hq] and (idx, score) [B, Hkv, k] on request.
        With ``check_status`` (default) it waits for the step and raises
        HBAError if a bounded device wait expired; ``decode_into`` (the
        graph-capturable path) leaves that to ``check_status()``."""
        if q.dim() == 4:
            q = q[:, 0]
        if (self.lens_host < 1).any():
            raise ValueError("every sequence needs at least one cached token")
        cfg = self.cfg
        dev = self.device
        with torch.cuda.device(dev):
            qb = as_bf16(q)
            out = torch.empty_like(qb)
            lse = torch.empty(self.B, cfg.n_heads, dtype=torch.float32, device=dev) if return_lse else None
            si = ss = None
            if return_selection:
                si = torch.empty(self.B, cfg.n_kv, cfg.k_blocks, dtype=torch.int32, device=dev)
                ss = torch.empty(self.B, cfg.n_kv, cfg.k_blocks, dtype=torch.float32, device=dev)
            self.decode_into(qb, out, lse, si, ss)
            if check_status:
                self.check_status()
        res = (out.to(q.dtype),)
        if return_lse:
            res += (lse,)
        if return_selection:
            res += ((si, ss),)
        return res[0] if len(res) == 1 else res

    def device_status(self, clear=False):
        """The decode's sticky device status word (0 = ok, 1 = a bounded device
        wait timed out); synchronises with the device.  `clear` resets it to 0."""
        st = int(self.workspace[:4].view(torch.int32).item())
        if clear:
            self.workspace[:4].zero_()
        return st

    def check_status(self, clear=False):
        """Raise HBAError (ERR_DEVICE_TIMEOUT) if a decode since the last clear
        met an expired bounded device wait; waits for the current stream."""
        _lib.check_device(ptr(self.workspace), stream_of(self.device), "hba_b200_decode (device status)", clear)

    def decode_into(self, qb, out, lse=None, sel_idx=None, sel_score=None, stream=None):
        """Allocation-free decode on preallocated bf16 q/out (graph-capturable)."""
        st = _lib.load().hba_b200_decode(
            ctypes.byref(self.c), self.B, self.n_cap, ptr(self.lens), ptr(self.scales), ptr(qb), ptr(self.q_gain),
            ptr(self.k_gain), ptr(self.k), ptr(self.kr), ptr(self.v), ptr(self.summaries), ptr(self.supers), ptr(self.cos),
            ptr(self.sin), ptr(out),
            ptr(lse), ptr(sel_idx), ptr(sel_score), ptr(self.workspace), self.ws_bytes,
            stream if stream is not None else stream_of(self.device))
        _lib.check(st, "hba_b200_decode")

    def step(self, q, k_new, v_new, **kw):
        """One decode step for a new token: append its k/v, then attend with its q."""
        if k_new.dim() == 3:
            k_new, v_new = k_new[:, None], v_new[:, None]
        self.append(k_new, v_new)
        return self.attend(q, **kw)
