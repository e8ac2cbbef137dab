"""Incremental decoding of a converted HBA model on the B200 path.

The reference's ``HBAModel`` (src/hba/model.py:20-180) has no decode path:
every ``forward`` re-runs the whole sequence, recomputing QKNorm and every
block summary of every layer (src/hba/attention.py:631, :659).
``HBAModelDecoder`` keeps one ``HBADecodeCache`` per layer and serves the
same model token by token:

* ``prefill(ids)`` runs ``HBAModel.forward``'s layer loop (``block_fn``,
  src/hba/model.py:119-144, eval or eval_hier) with the attention on the
  B200 prefill kernels and appends every layer's keys and values to its
  cache (QKNorm, the RoPE'd key copy and the summaries of completed blocks
  are built by the append);
* ``step(tokens)`` runs one new token per sequence through every layer:
  the projections, ``cache.step`` (append + one decode attention over the
  cache), the output projection and the MLP, and returns the logits.

The decode of the token at position n equals row n of a prefill over the
sequence (the last row of ``hba_attention_eval`` at length n + 1, with that
length's temperature tau(n + 1)).

``model`` is any object with the ``HBAModel`` attribute layout: ``cfg`` (an
``HBAConfig``), ``core`` (a Hugging Face decoder stack: ``embed_tokens``,
``layers[i].{input_layernorm, self_attn.{q,k,v,o}_proj,
post_attention_layernorm, mlp}``, ``norm``), ``lm_head``, ``summarizers[i]``
(``probes``, ``proj``) and ``qknorms[i]`` (``q.gain``, ``k.gain``) -- the
reference's own ``HBAModel`` included.
"""

import torch

from .attention import hba_attention_b200
from .cache import HBADecodeCache
from .synth import rope_tables


class HBAModelDecoder:
    def __init__(self, model, batch, max_len, device="cuda", hier=False):
        self.m = model
        self.cfg = model.cfg
        self.hier = bool(hier)
        self.B = int(batch)
        self.device = torch.device(device)
        cfg = self.cfg
        Bk = cfg.block
        self.max_len = -(-int(max_len) // Bk) * Bk
        self.cos, self.sin = rope_tables(self.max_len, cfg.head_dim, cfg.rope_theta, device=self.device)
        self.caches = [HBADecodeCache(cfg, self.B, self.max_len, model.summarizers[i], model.qknorms[i], self.cos,
                                      self.sin, device=self.device, hier=self.hier)
                       for i in range(len(model.core.layers))]
        self.n = 0  # tokens held per sequence

    def _heads(self, t, n, heads):
        return t.view(self.B, n, heads, self.cfg.head_dim)

    @torch.no_grad()
    def prefill(self, ids, all_logits=False):
        """ids [B, n] (n a multiple of the block size, as the reference
        asserts): fill every layer's cache and return the logits of the last
        position [B, V] (every position [B, n, V] with ``all_logits``)."""
        cfg, core = self.cfg, self.m.core
        B, n = ids.shape
        if B != self.B:
            raise ValueError("batch mismatch")
        if self.n != 0:
            raise ValueError("prefill runs on an empty decoder")
        if n > self.max_len:
            raise ValueError(f"prompt of {n} tokens exceeds the cache capacity {self.max_len}")
        x = core.embed_tokens(ids.to(self.device))
        cos, sin = self.cos[:n], self.sin[:n]
        for i, lyr in enumerate(core.layers):
            a = lyr.input_layernorm(x)
            q = self._heads(lyr.self_attn.q_proj(a), n, cfg.n_heads)
            k = self._heads(lyr.self_attn.k_proj(a), n, cfg.n_kv)
            v = self._heads(lyr.self_attn.v_proj(a), n, cfg.n_kv)
            self.caches[i].append(k, v)
            o = hba_attention_b200(q, k, v, cos, sin, cfg, self.m.summarizers[i], self.m.qknorms[i], hier=self.hier)
            x = x + lyr.self_attn.o_proj(o.reshape(B, n, cfg.n_heads * cfg.head_dim))
            x = x + lyr.mlp(lyr.post_attention_layernorm(x))
        self.n = n
        x = core.norm(x)
        return self.m.lm_head(x if all_logits else x[:, -1])

    @torch.no_grad()
    def step(self, tokens):
        """tokens [B]: the next token of every sequence; returns its logits [B, V]."""
        cfg, core = self.cfg, self.m.core
        if self.n + 1 > self.max_len:
            raise ValueError(f"cache capacity {self.max_len} exceeded")
        x = core.embed_tokens(tokens.to(self.device).view(self.B, 1))
        for i, lyr in enumerate(core.layers):
            a = lyr.input_layernorm(x)
            q = lyr.self_attn.q_proj(a).view(self.B, cfg.n_heads, cfg.head_dim)
            k = self._heads(lyr.self_attn.k_proj(a), 1, cfg.n_kv)
            v = self._heads(lyr.self_attn.v_proj(a), 1, cfg.n_kv)
            o = self.caches[i].step(q, k, v)
            x = x + lyr.self_attn.o_proj(o.reshape(self.B, 1, cfg.n_heads * cfg.head_dim).to(x.dtype))
            x = x + lyr.mlp(lyr.post_attention_layernorm(x))
        self.n += 1
        return self.m.lm_head(core.norm(x))[:, 0]
