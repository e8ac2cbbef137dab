"""KV-range sharded decode: one long context split across ranks (one process
per GPU), for contexts whose caches outgrow one GPU or whose decode should
use several GPUs' HBM bandwidth at once.

Rank r of P keeps global tokens [r*n_loc, (r+1)*n_loc) of every sequence:
its K / RoPE'd-K / V caches, the summaries of its blocks and (hierarchical
mode) the supers of its super-blocks; shard bounds fall on block (super)
multiples, so no block or super straddles two ranks.  One decode step:

  flat  local top-k over the owned candidate blocks (exact scores)
        -> all-gather the lists -> every rank merges them into the same
           global top-k (score desc, block asc) = the one-device picks
  hier  local top-beam supers -> all-gather -> global beam; each rank scores
        the children it owns -> local top-k -> all-gather -> global top-k
  then  each rank runs the union softmax over the tokens it owns (its part of
        the window, the sinks on rank 0, its picks) and keeps it as an
        unnormalised partial (O, l) scaled by its own reference maximum m2
        (log2 units: the QKNorm logit bound while it is small, else the
        running maximum of the owned logits); one all-gather of the
        (m2, l, O) triples, then the max-rescaled merge: M = max m2_r,
        w_r = 2^(m2_r - M), out = sum w_r O_r / sum w_r l_r,
        lse = (M + log2 sum w_r l_r) ln 2.

The reference runs on one device and has no equivalent; the result is its
decode (src/hba/attention.py:663-711 at cs = n-1) over the whole context.

Two implementations of the step:
  fused (default on GPUs)  one `hba_b200_decode_shard_fused` launch per step:
        the kernel's CTA for (sequence, kv head) exchanges its lists and its
        partial with the same CTA of every other rank through NVLink peer
        memory (`PeerExchange`: each rank's buffer, IPC-mapped by the others),
        with epoch flags and bounded waits -- no collective library call.
  split  the `hba_b200_decode_shard_select / _attend / _finish` kernels with
        the collectives in between through `TorchComm` (torch.distributed:
        NCCL on GPUs, gloo in the CPU tests, which also swap the kernels for a
        CPU stand-in via `ops`).
"""

import ctypes

import numpy as np
import torch
import torch.distributed as dist

from . import _lib
from .attention import as_bf16, as_f32, c_config, gains, ptr, stream_of, union_scale
from .cache import HBADecodeCache


def shard_range(cfg, max_len, rank, world, hier):
    """(tok_lo, n_loc, n_total): this rank's first global token and token
    count, and the total capacity (a multiple of world * block * F)."""
    unit = cfg.block * (cfg.fanout if hier else 1) * world
    n_total = -(-int(max_len) // unit) * unit
    n_loc = n_total // world
    return rank * n_loc, n_loc, n_total


class TorchComm:
    """The collective of a step (an all-gather) over a torch.distributed process group."""

    def __init__(self, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)

    def all_gather(self, t):
        """[*shape] -> [world, *shape] (rank order)."""
        parts = [torch.empty_like(t) for _ in range(self.world)]
        dist.all_gather(parts, t.contiguous(), group=self.group)
        return torch.stack(parts)


class PeerExchange:
    """The exchange buffers of the fused sharded decode: this rank's (cudaMalloc
    by the library, zeroed) and every other rank's, mapped into this process
    through CUDA IPC handles shared over the process group, plus the device
    epoch counter the fused call bumps each step.  `close()` unmaps and frees
    (collective: every rank calls it)."""

    def __init__(self, cfg, batch, hier, device, group=None):
        L = _lib.load()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = torch.device(device)
        nbytes = L.hba_b200_shard_xbuf_bytes(ctypes.byref(c_config(cfg, hier)), int(batch), self.world)
        if nbytes <= 0:
            raise ValueError(f"fused sharded decode: unsupported world size {self.world}")
        handle = ctypes.create_string_buffer(64)
        own = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _lib.check(L.hba_b200_peer_alloc(int(nbytes), ctypes.byref(own), handle), "hba_b200_peer_alloc")
        self.own = own.value
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle.raw), group=group)
        ptrs, self.mapped = [], []
        with torch.cuda.device(self.device):
            for r, h in enumerate(handles):
                if r == self.rank:
                    ptrs.append(self.own)
                    continue
                pr = ctypes.c_void_p()
                _lib.check(L.hba_b200_peer_open(ctypes.create_string_buffer(h, 64), ctypes.byref(pr)),
                           "hba_b200_peer_open")
                ptrs.append(pr.value)
                self.mapped.append(pr.value)
        self.ptrs = (ctypes.c_void_p * self.world)(*ptrs)
        self.epoch = torch.zeros(1, dtype=torch.int32, device=self.device)

    def close(self):
        if self.own is None:
            return
        L = _lib.load()
        torch.cuda.synchronize(self.device)
        with torch.cuda.device(self.device):
            for pr in self.mapped:
                L.hba_b200_peer_close(ctypes.c_void_p(pr))
        self.mapped = []
        dist.barrier(group=self.group)  # nobody maps our buffer any more
        with torch.cuda.device(self.device):
            L.hba_b200_peer_free(ctypes.c_void_p(self.own))
        self.own = None


class CudaShardOps:
    """The product path: the library's shard kernels on the rank's GPU."""

    def select(self, sh, level, in_idx, in_score, n_in_lists, out_idx, out_score):
        st = _lib.load().hba_b200_decode_shard_select(
            ctypes.byref(sh.c), sh.B, sh.n_loc, sh.tok_lo, level, ptr(sh.glens), ptr(sh.scales), ptr(sh.q),
            ptr(sh.local.q_gain), ptr(sh.local.summaries), ptr(sh.local.supers), ptr(in_idx), ptr(in_score),
            n_in_lists, ptr(out_idx), ptr(out_score), stream_of(sh.device))
        _lib.check(st, "hba_b200_decode_shard_select")

    def attend(self, sh, in_idx, in_score, n_in, part_o, part_l, part_m2, sel_idx, sel_score):
        st = _lib.load().hba_b200_decode_shard_attend(
            ctypes.byref(sh.c), sh.B, sh.n_loc, sh.tok_lo, ptr(sh.glens), ptr(sh.scales), ptr(sh.q),
            ptr(sh.local.q_gain), ptr(sh.local.k_gain), ptr(sh.local.k), ptr(sh.local.kr), ptr(sh.local.v),
            ptr(sh.cos), ptr(sh.sin), ptr(in_idx), ptr(in_score), n_in, ptr(part_o), ptr(part_l), ptr(part_m2),
            ptr(sel_idx), ptr(sel_score), ptr(sh.status), stream_of(sh.device))
        _lib.check(st, "hba_b200_decode_shard_attend")

    def finish(self, sh, parts, out, lse):
        st = _lib.load().hba_b200_decode_shard_finish(
            ctypes.byref(sh.c), sh.B, int(parts.shape[0]), ptr(parts), ptr(out), ptr(lse), stream_of(sh.device))
        _lib.check(st, "hba_b200_decode_shard_finish")


class HBAShardedDecode:
    """Decode over a context sharded by token range across the ranks of
    `comm` (default: the torch.distributed world).  `local` is this rank's
    cache of tokens [tok_lo, tok_lo + n_loc) (default: an `HBADecodeCache`
    with pos_offset = tok_lo on `device`); `ops` runs the per-rank pieces
    (default: the CUDA library)."""

    def __init__(self, cfg, batch, max_len, summ, qkn, cos, sin, device="cuda", hier=False, comm=None,
                 ops=None, local=None, fused=None):
        # fused: the one-launch NVLink path (default when the collectives and
        # kernels are the real ones on GPUs); else the split path
        if fused is None:
            fused = comm is None and ops is None and torch.device(device).type == "cuda"
        self.fused = bool(fused)
        self.comm = comm if comm is not None else TorchComm()
        self.ops = ops if ops is not None else CudaShardOps()
        self.cfg = cfg
        self.hier = bool(hier)
        self.B = int(batch)
        self.rank, self.world = self.comm.rank, self.comm.world
        self.tok_lo, self.n_loc, self.n_total = shard_range(cfg, max_len, self.rank, self.world, self.hier)
        if cos.shape[0] < self.n_total:
            raise ValueError(f"RoPE tables cover {cos.shape[0]} positions < sharded capacity {self.n_total}")
        self.device = torch.device(device)
        self.local = local if local is not None else HBADecodeCache(
            cfg, batch, self.n_loc, summ, qkn, cos, sin, device=device, hier=hier, pos_offset=self.tok_lo)
        self.c = c_config(cfg, self.hier)
        dev = self.device
        self.cos = as_f32(cos[: self.n_total], dev)     # the query is rotated at its global position
        self.sin = as_f32(sin[: self.n_total], dev)
        self.glens_host = np.zeros(self.B, dtype=np.int64)
        self.glens = torch.zeros(self.B, dtype=torch.int32, device=dev)
        self.scales = torch.zeros(self.B, dtype=torch.float32, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        BH, K, Hq, dh = self.B * cfg.n_kv, cfg.k_blocks, cfg.n_heads, cfg.head_dim
        self.l_idx = torch.empty(BH, K, dtype=torch.int32, device=dev)
        self.l_sc = torch.empty(BH, K, dtype=torch.float32, device=dev)
        if self.hier:
            self.s_idx = torch.empty(BH, cfg.beam, dtype=torch.int32, device=dev)
            self.s_sc = torch.empty(BH, cfg.beam, dtype=torch.float32, device=dev)
        # this rank's partial [m2 | l | O] in one buffer: one all-gather per step
        BHq = self.B * Hq
        self.part = torch.empty(BHq * (dh + 2), dtype=torch.float32, device=dev)
        self.part_m2 = self.part[:BHq].view(self.B, Hq)
        self.part_l = self.part[BHq: 2 * BHq].view(self.B, Hq)
        self.part_o = self.part[2 * BHq:].view(self.B, Hq, dh)
        self.q = None
        self.x = PeerExchange(cfg, self.B, self.hier, dev, self.comm.group) if self.fused else None

    # ---------------------------------------------------------------- state --
    def _set_lengths(self, n):
        self.glens_host[:] = n
        self.glens.fill_(int(n))
        s = union_scale(self.cfg, self.cfg.head_dim, max(1, int(n)))
        self.scales.fill_(float(s))

    def fill(self, k_full, v_full):
        """Load a whole context (every sequence n tokens): k_full, v_full
        [B, n, Hkv, dh] raw projections; this rank keeps its token range."""
        n = int(k_full.shape[1])
        if n > self.n_total:
            raise ValueError(f"context {n} exceeds the sharded capacity {self.n_total}")
        lo, hi = self.tok_lo, min(self.tok_lo + self.n_loc, n)
        if hi > lo:
            self.local.append(k_full[:, lo:hi], v_full[:, lo:hi])
        self._set_lengths(n)

    def fill_local(self, k_loc, v_loc, n):
        """Load this rank's part of a context of n tokens (every sequence):
        k_loc, v_loc [B, t, Hkv, dh] raw projections of tokens [tok_lo,
        tok_lo + t) -- the rows a prefill split by token range computed on
        this rank (t = 0 when the context ends before the range)."""
        if n > self.n_total:
            raise ValueError(f"context {n} exceeds the sharded capacity {self.n_total}")
        t = int(k_loc.shape[1])
        if t != max(0, min(self.tok_lo + self.n_loc, n) - self.tok_lo):
            raise ValueError(f"rank {self.rank} holds tokens [{self.tok_lo}, {self.tok_lo + self.n_loc}) of {n}: "
                             f"got {t}")
        if t > 0:
            self.local.append(k_loc, v_loc)
        self._set_lengths(n)

    def append(self, k_new, v_new):
        """Append t tokens to every sequence (all sequences hold the same
        length): each rank keeps the part that falls in its range."""
        if (self.glens_host != self.glens_host[0]).any():
            raise ValueError("sharded append needs equal sequence lengths")
        L, t = int(self.glens_host[0]), int(k_new.shape[1])
        if L + t > self.n_total:
            raise ValueError(f"sharded capacity {self.n_total} exceeded")
        lo, hi = max(L, self.tok_lo), min(L + t, self.tok_lo + self.n_loc)
        if hi > lo:
            self.local.append(k_new[:, lo - L: hi - L], v_new[:, lo - L: hi - L])
        self._set_lengths(L + t)

    # --------------------------------------------------------------- decode --
    def _gather_lists(self, idx, sc):
        """[BH, k] local lists of every rank -> [BH, P*k] (rank-major per row)."""
        BH, k = idx.shape
        packed = torch.cat([idx.reshape(-1), sc.reshape(-1).view(torch.int32)])
        g = self.comm.all_gather(packed)                                  # [P, 2*BH*k]
        gi = g[:, : BH * k].reshape(self.world, BH, k).permute(1, 0, 2).reshape(BH, self.world * k)
        gs = g[:, BH * k:].reshape(self.world, BH, k).permute(1, 0, 2).reshape(BH, self.world * k)
        return gi.contiguous(), gs.contiguous().view(torch.float32)

    def decode_into(self, q, out, lse=None, sel_idx=None, sel_score=None):
        """q [B, Hq, dh] bf16 (the same on every rank) -> out [B, Hq, dh] bf16,
        lse [B, Hq] natural log, picks [B, Hkv, K] (global block ids)."""
        if (self.glens_host < 1).any():
            raise ValueError("every sequence needs at least one cached token")
        self.q = q
        if self.fused:
            loc = self.local
            st = _lib.load().hba_b200_decode_shard_fused(
                ctypes.byref(self.c), self.B, self.n_loc, self.tok_lo, self.world, self.rank, self.x.ptrs,
                ptr(self.x.epoch), ptr(self.glens), ptr(self.scales), ptr(q), ptr(loc.q_gain), ptr(loc.k_gain),
                ptr(loc.summaries), ptr(loc.supers), ptr(loc.k), ptr(loc.kr), ptr(loc.v), ptr(self.cos),
                ptr(self.sin), ptr(out), ptr(lse), ptr(sel_idx), ptr(sel_score), ptr(self.status),
                stream_of(self.device))
            _lib.check(st, "hba_b200_decode_shard_fused")
            return
        if not self.hier:
            self.ops.select(self, 0, None, None, 0, self.l_idx, self.l_sc)
        else:
            self.ops.select(self, 1, None, None, 0, self.s_idx, self.s_sc)
            si, ss = self._gather_lists(self.s_idx, self.s_sc)           # [BH, P*beam]
            self.ops.select(self, 2, si, ss, self.world, self.l_idx, self.l_sc)
        gi, gs = self._gather_lists(self.l_idx, self.l_sc)               # [BH, P*K]
        self.ops.attend(self, gi, gs, gi.shape[1], self.part_o, self.part_l, self.part_m2, sel_idx, sel_score)
        parts = self.comm.all_gather(self.part)                          # [P, B*Hq*(dh+2)]
        self.ops.finish(self, parts, out, lse)

    def capture(self, q, out, lse=None, sel_idx=None, sel_score=None):
        """Capture one step -- kernels, list reshuffles and collectives -- as a
        CUDA graph on these fixed buffers; `replay()` runs it.  Every rank must
        capture (the collectives are part of the graph).  Call `release()`
        before the process group is destroyed."""
        self.decode_into(q, out, lse, sel_idx, sel_score)  # warm-up outside the capture
        torch.cuda.synchronize(self.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.decode_into(q, out, lse, sel_idx, sel_score)
        torch.cuda.synchronize(self.device)

    def replay(self):
        self.graph.replay()

    def release(self):
        """Drop the captured graph (before the process group is destroyed)."""
        self.graph = None

    def close(self):
        """Release the graph and, on the fused path, the exchange buffers
        (collective: every rank calls it)."""
        self.release()
        if self.x is not None:
            self.x.close()
            self.x = None

    def attend(self, q, return_lse=False):
        """Allocating convenience wrapper of `decode_into`."""
        if q.dim() == 4:
            q = q[:, 0]
        qb = as_bf16(q.to(self.device))
        out = torch.empty_like(qb)
        lse = torch.empty(self.B, self.cfg.n_heads, dtype=torch.float32, device=self.device) if return_lse else None
        self.decode_into(qb, out, lse)
        if self.device.type == "cuda":
            self.check_status()
        return (out, lse) if return_lse else out

    def check_status(self, clear=False):
        """Raise HBAError (ERR_DEVICE_TIMEOUT) if a step since the last clear
        met an expired bounded device wait (e.g. a rank that never arrived at
        an exchange); waits for the current stream."""
        _lib.check_device(ptr(self.status), stream_of(self.device), "sharded decode (device status)", clear)
