"""A converted HBA model over contexts split by token range across GPUs
(one process per GPU, torch.distributed over NCCL): the sequence-sharded
long-context prefill + decode of the BASELINE's 8-GPU configuration.

Rank r of P owns tokens [r * n_loc, (r + 1) * n_loc) of every sequence: their
hidden states through the prefill, and afterwards their keys / values /
summaries in every layer's ``HBAShardedDecode`` cache.

* ``prefill(ids)``: each rank embeds its own tokens and runs the layer loop
  of ``HBAModel.forward`` (``block_fn``, src/hba/model.py:119-144) on them.
  Per layer the ranks all-gather the new keys and values (NCCL), so every
  rank holds those of tokens [0, its last token] -- the routed blocks and the
  window of its queries may sit on earlier ranks -- and runs the B200 prefill
  for its query rows only (``hba_attention_b200_range``, one temperature
  tau(N) for all rows as the reference's forward uses); its own keys and
  values go into its shard of the layer's cache.  The logits of the last
  position come from the rank that holds it and are broadcast.
* ``step(tokens)``: the new token's projections and MLP are computed on every
  rank (replicated, a few MB of weights); each layer's attention is one
  ``HBAShardedDecode`` step -- each rank selects among and attends over the
  tokens it owns, the per-rank top-k lists and (O, l, m) partials are
  exchanged inside the fused decode kernel over NVLink -- and every rank gets
  the whole output.

The reference runs one device and has no equivalent; the result is its
forward (prefill) and its decode at cs = n-1 over the whole context.
"""

import torch
import torch.distributed as dist

from .attention import hba_attention_b200_range
from .sharded import HBAShardedDecode
from .synth import rope_tables


class HBAShardedModelDecoder:
    def __init__(self, model, batch, max_len, device):
        self.m = model
        self.cfg = model.cfg
        self.group = None  # the default torch.distributed group (the shards' exchange buffers live there)
        self.B = int(batch)
        self.device = torch.device(device)
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        cfg = self.cfg
        n_layers = len(model.core.layers)
        # one layer's shard fixes the token ranges (the same for every layer)
        unit = cfg.block * self.world
        self.n_total = -(-int(max_len) // unit) * unit
        self.cos, self.sin = rope_tables(self.n_total, cfg.head_dim, cfg.rope_theta, device=self.device)
        self.shards = [HBAShardedDecode(cfg, self.B, self.n_total, model.summarizers[i], model.qknorms[i], self.cos,
                                        self.sin, device=self.device, comm=None)
                       for i in range(n_layers)]
        self.tok_lo, self.n_loc = self.shards[0].tok_lo, self.shards[0].n_loc
        self.n = 0

    def _gather_tokens(self, t_loc, hi):
        """[B, n_loc_used, ...] per rank (zero-padded to n_loc) -> tokens [0, hi) of the whole context."""
        pad = torch.zeros((self.B, self.n_loc) + tuple(t_loc.shape[2:]), dtype=t_loc.dtype, device=self.device)
        pad[:, : t_loc.shape[1]] = t_loc
        parts = [torch.empty_like(pad) for _ in range(self.world)]
        dist.all_gather(parts, pad, group=self.group)
        return torch.cat(parts, dim=1)[:, :hi]

    @torch.no_grad()
    def prefill(self, ids):
        """ids [B, N] (the whole prompt on every rank, N a multiple of the
        block): fill every layer's sharded cache; returns the logits of the
        last position [B, V] on every rank."""
        cfg, core = self.cfg, self.m.core
        B, N = ids.shape
        if N > self.n_total or N % cfg.block != 0:
            raise ValueError(f"prompt of {N} tokens: needs a multiple of {cfg.block} <= {self.n_total}")
        lo = self.tok_lo
        hi = max(lo, min(lo + self.n_loc, N))  # this rank's queries [lo, hi) use the keys of tokens [0, hi)
        n_own = hi - lo
        x = core.embed_tokens(ids[:, lo:lo + n_own].to(self.device))
        for i, lyr in enumerate(core.layers):
            a = lyr.input_layernorm(x)
            q = lyr.self_attn.q_proj(a).view(B, n_own, cfg.n_heads, cfg.head_dim)
            k = lyr.self_attn.k_proj(a).view(B, n_own, cfg.n_kv, cfg.head_dim)
            v = lyr.self_attn.v_proj(a).view(B, n_own, cfg.n_kv, cfg.head_dim)
            k_all = self._gather_tokens(k, hi)  # every rank takes part in the collectives
            v_all = self._gather_tokens(v, hi)
            self.shards[i].fill_local(k, v, N)
            if n_own > 0:
                o = hba_attention_b200_range(q, k_all, v_all, self.cos, self.sin, cfg, self.m.summarizers[i],
                                             self.m.qknorms[i], q_lo=lo, n_total=N)
                x = x + lyr.self_attn.o_proj(o.reshape(B, n_own, cfg.n_heads * cfg.head_dim))
                x = x + lyr.mlp(lyr.post_attention_layernorm(x))
        self.n = N
        owner = (N - 1) // self.n_loc
        logits = torch.empty(B, self.m.lm_head.out_features, dtype=x.dtype, device=self.device)
        if self.rank == owner:
            logits.copy_(self.m.lm_head(core.norm(x[:, -1:]))[:, 0])
        dist.broadcast(logits, src=owner, group=self.group)
        return logits

    @torch.no_grad()
    def step(self, tokens):
        """tokens [B] (the same on every rank): the next token of every
        sequence; returns its logits [B, V] on every rank."""
        cfg, core = self.cfg, self.m.core
        x = core.embed_tokens(tokens.to(self.device).view(self.B, 1))
        for i, lyr in enumerate(core.layers):
            a = lyr.input_layernorm(x)
            q = lyr.self_attn.q_proj(a).view(self.B, cfg.n_heads, cfg.head_dim)
            k = lyr.self_attn.k_proj(a).view(self.B, 1, cfg.n_kv, cfg.head_dim)
            v = lyr.self_attn.v_proj(a).view(self.B, 1, cfg.n_kv, cfg.head_dim)
            sh = self.shards[i]
            sh.append(k, v)
            o = sh.attend(q)
            x = x + lyr.self_attn.o_proj(o.reshape(self.B, 1, cfg.n_heads * cfg.head_dim).to(x.dtype))
            x = x + lyr.mlp(lyr.post_attention_layernorm(x))
        self.n += 1
        return self.m.lm_head(core.norm(x))[:, 0]

    def close(self):
        """Release every layer's exchange buffers (collective: every rank calls it)."""
        for sh in self.shards:
            sh.close()
