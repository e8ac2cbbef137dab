"""A config object with the reference ``HBAConfig`` field names and defaults
(src/hba/config.py:105-184), for callers that do not import the reference.
Any object with these attributes (the reference's own ``HBAConfig`` included)
is accepted by every function of this package."""

from dataclasses import dataclass
from typing import Optional


@dataclass
class HBAConfig:
    n_layers: int = 24
    n_heads: int = 14
    n_kv: int = 2
    head_dim: int = 64
    hidden: int = 896
    rope_theta: float = 1_000_000.0
    native_ctx: int = 32768
    vocab_size: int = 151936
    block: int = 64
    window: int = 1024
    sinks: int = 4
    k_blocks: int = 16
    slots: int = 4
    aux_w: float = 1.0
    fanout: int = 16
    beam: int = 4
    hier_from: int = 32768
    heal_ctx: int = 4096
    mem_elem_cap: float = 1.0e8
    qknorm: bool = True
    content_scale_mode: str = "inv_d"
    temp_c: float = 0.1
    n_cal: Optional[int] = None
    attn_backend: str = "fused"

    @property
    def G(self):
        return self.n_heads // self.n_kv


# The BASELINE workloads (shapes of the reference's headline configurations).
BASELINE = {
    "cfg0": dict(batch=1, n=4096, n_heads=14, n_kv=2, head_dim=64, window=1024, sinks=4, block=64, slots=4,
                 k_blocks=16, hier=False, native_ctx=32768),
    "cfg1": dict(batch=64, n=32768, n_heads=14, n_kv=2, head_dim=64, window=1024, sinks=4, block=64, slots=4,
                 k_blocks=16, hier=False, native_ctx=32768),
    "cfg2": dict(batch=4, n=32768, n_heads=32, n_kv=8, head_dim=128, window=1024, sinks=4, block=64, slots=4,
                 k_blocks=16, hier=False, native_ctx=32768),
    "cfg3": dict(batch=32, n=131072, n_heads=32, n_kv=8, head_dim=128, window=1024, sinks=4, block=64, slots=4,
                 k_blocks=16, hier=True, fanout=16, beam=8, native_ctx=32768),
}


def baseline_config(name, **overrides):
    """(HBAConfig, batch, n, hier) for a BASELINE workload name."""
    d = dict(BASELINE[name])
    d.update(overrides)
    batch, n, hier = d.pop("batch"), d.pop("n"), d.pop("hier")
    cfg = HBAConfig(**{k: v for k, v in d.items() if k in HBAConfig.__dataclass_fields__})
    return cfg, batch, n, hier
