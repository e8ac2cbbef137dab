"""Seeded synthetic workloads with the shapes and value distributions of the
BASELINE configurations (there is no dataset for this path: inputs are
random, with planted target blocks so that routing has a well-separated
answer).

* q/k/v ~ N(0, 1) (raw projections; the cache / forward applies QKNorm).
* Summarizer probes ~ N(0, 1/dh), proj = I + 0.02 N(0, 1) (the reference
  init, src/hba/summarizer.py:25,31-32); QKNorm gains 1 unless `gains` is set:
  True draws them from U[0.6, 1.6]; "trained" from U[7, 17], so that
  gain_q * gain_k spans ~50-290 -- the magnitude the reference's
  data-dependent init gives a trained donor (gain_q * gain_k =
  sqrt(dh) * rms_q * rms_k, src/hba/model.py:197-253), where the logits
  reach the hundreds.
* Decode planting: per (sequence, kv head), 8 distinct candidate blocks of
  the query at n-1 (hierarchical: in 8 distinct super-nodes) get keys
  sqrt(dh) * (0.8 q^ + 0.6 w_t), w_t a random unit vector orthogonal to the
  normalised grouped query q^ -- cosine 0.8 with q^.
* Prefill planting: 64-query tiles share a topic direction d (queries get
  + alpha*sqrt(dh)*d per head); each topic owns 8 planted blocks in the first
  half of the sequence whose keys have cosine 0.8 with d.
"""

import math

import torch

BF16 = torch.bfloat16


def rope_tables(n, dh, theta, device="cuda"):
    """NeoX tables cat(fr, fr), fr = pos * theta^(-2i/dh), fp32 [n, dh] (the
    reference's rope_tables layout, src/hba/attention.py:27-32)."""
    inv = 1.0 / (theta ** (torch.arange(0, dh, 2, device=device).float() / dh))
    pos = torch.arange(n, device=device).float()
    fr = torch.outer(pos, inv)
    emb = torch.cat((fr, fr), dim=-1)
    return emb.cos(), emb.sin()


class _Gain:
    def __init__(self, g):
        self.gain = g


class QKNormGains:
    """Holds q.gain [Hq] and k.gain [Hkv] (the attribute layout of the
    reference QKNorm module)."""

    def __init__(self, q_gain, k_gain):
        self.q = _Gain(q_gain)
        self.k = _Gain(k_gain)


class SummarizerWeights:
    """Holds probes [Hkv, m, dh] and proj [Hkv, dh, dh] (the attribute layout
    of the reference SlotSummarizer)."""

    def __init__(self, probes, proj):
        self.probes = probes
        self.proj = proj


def make_weights(cfg, device="cuda", seed=0, gains=False):
    g = torch.Generator(device="cpu").manual_seed(seed)
    Hkv, m, dh = cfg.n_kv, cfg.slots, cfg.head_dim
    probes = torch.randn(Hkv, m, dh, generator=g) * dh ** -0.5
    proj = torch.eye(dh).unsqueeze(0).repeat(Hkv, 1, 1) + torch.randn(Hkv, dh, dh, generator=g) * 0.02
    if gains == "trained":
        qg = torch.rand(cfg.n_heads, generator=g) * 10.0 + 7.0
        kg = torch.rand(Hkv, generator=g) * 10.0 + 7.0
    elif gains:
        qg = torch.rand(cfg.n_heads, generator=g) * 1.0 + 0.6
        kg = torch.rand(Hkv, generator=g) * 1.0 + 0.6
    else:
        qg = torch.ones(cfg.n_heads)
        kg = torch.ones(Hkv)
    return (SummarizerWeights(probes.to(device), proj.to(device)),
            QKNormGains(qg.to(device), kg.to(device)))


def _unit(x):
    return x / x.norm(dim=-1, keepdim=True).clamp_min(1e-12)


def _qknorm(x, gain):
    xf = x.float()
    return xf / xf.pow(2).mean(-1, keepdim=True).clamp_min(1e-6).sqrt() * gain.float().view(-1, 1)


def _planted_rows(direction, count, dh, gen):
    """count keys with cosine 0.8 to `direction` [..., dh] -> [..., count, dh], RMS 1."""
    shape = direction.shape[:-1] + (count, dh)
    w = torch.randn(shape, generator=gen, device=direction.device)
    d = direction.unsqueeze(-2)
    w = _unit(w - (w * d).sum(-1, keepdim=True) * d)
    return (0.8 * d + 0.6 * w) * math.sqrt(dh)


def decode_workload(cfg, batch, n, hier=False, seed=0, device="cuda", qkn=None, planted=8):
    """One decode query per sequence at position n-1 over n cached tokens.
    Returns dict(q [B, Hq, dh], k, v [B, n, Hkv, dh] raw bf16, planted [B, Hkv, p])."""
    gen = torch.Generator(device=device).manual_seed(seed)
    B, Hq, Hkv, dh, G, Bk = batch, cfg.n_heads, cfg.n_kv, cfg.head_dim, cfg.n_heads // cfg.n_kv, cfg.block
    q = torch.randn(B, Hq, dh, generator=gen, device=device, dtype=BF16)
    k = torch.randn(B, n, Hkv, dh, generator=gen, device=device, dtype=BF16)
    v = torch.randn(B, n, Hkv, dh, generator=gen, device=device, dtype=BF16)
    qg = torch.ones(Hq, device=device) if qkn is None else qkn.q.gain.float()
    qc = _qknorm(q, qg).to(BF16).float()
    qhat = _unit(qc.view(B, Hkv, G, dh).sum(2))                               # [B, Hkv, dh]
    lim = n - 1 - cfg.window + 1
    bmax = lim // Bk - 1 if lim >= 2 * Bk else 0
    planted_idx = torch.full((B, Hkv, planted), -1, dtype=torch.long, device=device)
    if bmax >= 1 and planted > 0:
        cpu = torch.Generator().manual_seed(seed + 1)
        if hier:
            F = cfg.fanout
            nsup = bmax // F + 1
            p = min(planted, nsup)
            sup = torch.stack([torch.randperm(nsup, generator=cpu)[:p] for _ in range(B * Hkv)]).view(B, Hkv, p)
            lo = torch.clamp(sup * F, min=1)
            hi = torch.clamp(sup * F + F - 1, max=bmax)
            r = torch.rand(B, Hkv, p, generator=cpu)
            blk = lo + (r * (hi - lo + 1).float()).long().clamp(max=(hi - lo))
        else:
            p = min(planted, bmax)
            blk = torch.stack([torch.randperm(bmax, generator=cpu)[:p] + 1 for _ in range(B * Hkv)]).view(B, Hkv, p)
        blk = blk.to(device)
        planted_idx[..., :p] = blk
        rows = _planted_rows(qhat[:, :, None, :].expand(B, Hkv, p, dh), Bk, dh, gen)   # [B,Hkv,p,Bk,dh]
        tok = (blk[..., None] * Bk + torch.arange(Bk, device=device))                    # [B,Hkv,p,Bk]
        bi = torch.arange(B, device=device).view(B, 1, 1, 1).expand_as(tok)
        gi = torch.arange(Hkv, device=device).view(1, Hkv, 1, 1).expand_as(tok)
        k[bi, tok, gi] = rows.to(BF16)
    return dict(q=q, k=k, v=v, planted=planted_idx)


def prefill_workload(cfg, batch, n, seed=0, device="cuda", alpha=1.0, planted=8, tile=64):
    """A full-sequence forward workload.  Returns dict(q [B, n, Hq, dh],
    k, v [B, n, Hkv, dh] raw bf16, topic [B, Hkv, T, dh], planted [B, Hkv, T, p])."""
    gen = torch.Generator(device=device).manual_seed(seed)
    B, Hq, Hkv, dh, G, Bk = batch, cfg.n_heads, cfg.n_kv, cfg.head_dim, cfg.n_heads // cfg.n_kv, cfg.block
    nb = n // Bk
    q = torch.randn(B, n, Hq, dh, generator=gen, device=device, dtype=torch.float32)
    k = torch.randn(B, n, Hkv, dh, generator=gen, device=device, dtype=BF16)
    v = torch.randn(B, n, Hkv, dh, generator=gen, device=device, dtype=BF16)
    T = max(0, min(16, (nb // 2 - 1) // max(1, planted)))
    info = dict(topic=None, planted=None)
    if T >= 1:
        topic = _unit(torch.randn(B, Hkv, T, dh, generator=gen, device=device))
        cpu = torch.Generator().manual_seed(seed + 1)
        blk = torch.stack([torch.randperm(nb // 2 - 1, generator=cpu)[:T * planted] + 1
                           for _ in range(B * Hkv)]).view(B, Hkv, T, planted).to(device)
        rows = _planted_rows(topic[:, :, :, None, :].expand(B, Hkv, T, planted, dh), Bk, dh, gen)
        tok = blk[..., None] * Bk + torch.arange(Bk, device=device)                         # [B,Hkv,T,p,Bk]
        bi = torch.arange(B, device=device).view(B, 1, 1, 1, 1).expand_as(tok)
        gi = torch.arange(Hkv, device=device).view(1, Hkv, 1, 1, 1).expand_as(tok)
        k[bi, tok, gi] = rows.to(BF16)
        tile_topic = (torch.arange(n, device=device) // tile) % T                            # [n]
        d = topic[:, :, tile_topic]                                                          # [B,Hkv,n,dh]
        q += alpha * math.sqrt(dh) * d.permute(0, 2, 1, 3).repeat_interleave(G, dim=2)
        info = dict(topic=topic, planted=blk)
    return dict(q=q.to(BF16), k=k, v=v, **info)
