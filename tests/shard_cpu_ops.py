"""CPU stand-ins for the KV-range shard kernels, built from the oracle
(float64 numpy), so the sharded decode's host orchestration -- the
collectives, the list merges, the partial sums -- can run as gloo ranks on
CPU.  Test infrastructure only: the product path is the CUDA library.

`CpuShard` is one rank's local state (QKNorm'd keys, values and the stored
summaries / supers of its token range); `CpuShardOps` implements
select / attend / finish with the semantics of hba_b200_decode_shard_*."""

import math

import numpy as np
import torch

from oracle import hba_oracle as orc

NEG_INF = -np.inf


class CpuShard:
    """Rank-local slices of a global context: kc, v [B, n_loc, Hkv, dh],
    S0 [B, Hkv, n_loc/Bk, m, dh], S1 [B, Hkv, n_loc/(Bk*F), m, dh]."""

    def __init__(self, kc, v, S0, S1, q_gain, k_gain, tok_lo, n_loc, Bk, F):
        self.tok_lo, self.n_loc = tok_lo, n_loc
        lo, hi = tok_lo, tok_lo + n_loc
        self.kc, self.v = kc[:, lo:hi], v[:, lo:hi]
        self.S0 = S0[:, :, lo // Bk: hi // Bk]
        self.S1 = None if S1 is None else S1[:, :, lo // (Bk * F): hi // (Bk * F)]
        self.q_gain = torch.as_tensor(q_gain)
        self.k_gain = torch.as_tensor(k_gain)
        # placeholders the orchestration never dereferences on CPU
        self.k = self.kr = self.summaries = self.supers = None

    def append(self, k, v):
        raise NotImplementedError("the CPU shard is built from a whole context")


def _top(scores, ids, k):
    """Best k (score desc, id asc) of finite scores -> (ids, scores) padded with (-1, -inf)."""
    order = np.lexsort((ids, -scores))
    order = [o for o in order if np.isfinite(scores[o])][:k]
    out_i = np.full(k, -1, np.int64)
    out_s = np.full(k, NEG_INF)
    out_i[: len(order)] = ids[order]
    out_s[: len(order)] = scores[order]
    return out_i, out_s


class CpuShardOps:
    def __init__(self, cfg, cos, sin):
        self.cfg = cfg
        self.cos = np.asarray(cos, np.float64)
        self.sin = np.asarray(sin, np.float64)

    # --------------------------------------------------------------- pieces --
    def _geometry(self, sh):
        c = self.cfg
        n = int(sh.glens_host[0])
        pos, nb = n - 1, n // c.block
        cand = orc.route_candidates([pos], c.window, nb, c.block)[0]      # [nb]
        return n, pos, nb, cand

    def _qg(self, sh):
        q = sh.q.float().numpy()
        qc = orc.head_rmsnorm(q, sh.local.q_gain.numpy(), bf16=True)
        return qc, orc.grouped_query(qc[:, None], self.cfg.n_kv, bf16=True)[:, :, 0]

    def _merge(self, in_idx, in_score, k):
        ids = in_idx.numpy().astype(np.int64)
        sc = np.where(ids >= 0, in_score.numpy().astype(np.float64), NEG_INF)
        return _top(sc, np.where(ids >= 0, ids, np.iinfo(np.int64).max), k)

    # ---------------------------------------------------------------- ops ----
    def select(self, sh, level, in_idx, in_score, n_in_lists, out_idx, out_score):
        c, loc = self.cfg, sh.local
        n, pos, nb, cand = self._geometry(sh)
        scale = float(sh.scales[0])
        _, qg = self._qg(sh)
        blo, bhi = sh.tok_lo // c.block, (sh.tok_lo + sh.n_loc) // c.block
        F = c.fanout
        B, Hkv = sh.B, c.n_kv
        for b in range(B):
            for g in range(Hkv):
                r = b * Hkv + g
                if level == 0:
                    ids = np.arange(blo, min(bhi, nb))
                    ids = ids[cand[ids]]
                    sc = orc.slot_scores(qg[b, g], loc.S0[b, g][ids - blo], scale) if len(ids) else np.zeros(0)
                    oi, os_ = _top(sc, ids, out_idx.shape[1])
                elif level == 1:
                    ns = -(-nb // F)
                    pad = ns * F - nb
                    cm = np.concatenate([cand, np.zeros(pad, bool)]) if pad else cand
                    cand_sup = cm.reshape(ns, F).any(-1)
                    ids = np.arange(blo // F, min(bhi // F, ns))
                    ids = ids[cand_sup[ids]]
                    sc = (orc.slot_scores(qg[b, g], loc.S1[b, g][ids - blo // F], scale)
                          if len(ids) else np.zeros(0))
                    oi, os_ = _top(sc, ids, out_idx.shape[1])
                else:
                    ns = -(-nb // F)
                    sup, _ = self._merge(in_idx[r], in_score[r], min(c.beam, ns))
                    kids = np.array([s * F + f for s in sup if s >= 0 for f in range(F)], np.int64)
                    kids = kids[(kids < nb) & (kids >= blo) & (kids < bhi)]
                    kids = kids[cand[kids]] if len(kids) else kids
                    sc = orc.slot_scores(qg[b, g], loc.S0[b, g][kids - blo], scale) if len(kids) else np.zeros(0)
                    oi, os_ = _top(sc, kids, out_idx.shape[1])
                out_idx[r] = torch.as_tensor(oi, dtype=torch.int32)
                out_score[r] = torch.as_tensor(os_, dtype=torch.float32)

    def attend(self, sh, in_idx, in_score, n_in, part_o, part_l, part_m2, sel_idx, sel_score):
        c, loc = self.cfg, sh.local
        n, pos, nb, cand = self._geometry(sh)
        scale = float(sh.scales[0])
        qc, _ = self._qg(sh)
        G, dh, Bk = c.n_heads // c.n_kv, c.head_dim, c.block
        kk = min(c.k_blocks, nb)
        if sh.hier:
            kk = min(kk, min(c.beam, -(-nb // c.fanout)) * c.fanout)
        lo, hi = sh.tok_lo, sh.tok_lo + sh.n_loc
        for b in range(sh.B):
            for g in range(c.n_kv):
                r = b * c.n_kv + g
                picks, _ = self._merge(in_idx[r], in_score[r], kk)
                picks = [int(p) for p in picks if p >= 0]
                q = qc[b, g * G:(g + 1) * G].astype(np.float64)                    # [G, dh]
                qr = orc.apply_rope_bf16(q, self.cos[pos][None], self.sin[pos][None])
                kcg, vg = loc.kc[b, :, g].astype(np.float64), loc.v[b, :, g].astype(np.float64)
                lg, vals = [], []
                for j in range(0, min(c.sinks, pos + 1)):                      # sinks (NoPE)
                    if lo <= j < hi:
                        lg.append(q @ kcg[j - lo])
                        vals.append(vg[j - lo])
                for j in range(max(c.sinks, pos - c.window + 1), pos + 1):      # window (RoPE)
                    if lo <= j < hi:
                        kr = orc.apply_rope_bf16(kcg[j - lo][None], self.cos[j][None], self.sin[j][None])[0]
                        lg.append(qr @ kr)
                        vals.append(vg[j - lo])
                for p in picks:                                                 # routed (NoPE)
                    for j in range(p * Bk, (p + 1) * Bk):
                        if lo <= j < hi:
                            lg.append(q @ kcg[j - lo])
                            vals.append(vg[j - lo])
                # this rank's own reference maximum per head (a running max of
                # the owned logits: it differs between ranks, so the finish
                # merge has to rescale)
                if lg:
                    L = np.stack(lg, 1) * scale                                  # [G, keys]
                    M = L.max(1)
                    e = np.exp(L - M[:, None])
                    O, l = e @ np.stack(vals), e.sum(1)
                else:
                    M = np.full(G, NEG_INF)
                    O, l = np.zeros((G, dh)), np.zeros(G)
                part_o[b, g * G:(g + 1) * G] = torch.as_tensor(O, dtype=torch.float32)
                part_l[b, g * G:(g + 1) * G] = torch.as_tensor(l, dtype=torch.float32)
                part_m2[b, g * G:(g + 1) * G] = torch.as_tensor(M / math.log(2), dtype=torch.float32)
                if sel_idx is not None:
                    ids = np.full(sel_idx.shape[-1], -1)
                    ids[: len(picks)] = picks[: sel_idx.shape[-1]]
                    sel_idx[b, g] = torch.as_tensor(ids, dtype=torch.int32)

    def finish(self, sh, parts, out, lse):
        """Max-rescaled merge of the gathered [world, B*Hq*(dh+2)] partials
        (per rank [m2 | l | O], m2 in log2 units)."""
        P = parts.shape[0]
        B, Hq, dh = out.shape
        BHq = B * Hq
        p = parts.double()
        m = p[:, :BHq].view(P, B, Hq)
        l = p[:, BHq: 2 * BHq].view(P, B, Hq)
        O = p[:, 2 * BHq:].view(P, B, Hq, dh)
        M = m.max(0).values
        w = torch.where(torch.isinf(m) & (m < 0), torch.zeros_like(m), torch.exp2(m - M))
        Ls = (w * l).sum(0)
        out.copy_(((w[..., None] * O).sum(0) / Ls[..., None].clamp_min(1e-300)).to(out.dtype))
        if lse is not None:
            lse.copy_(((M + torch.log2(Ls)) * math.log(2)).to(lse.dtype))
