"""hba_b200 -- B200-native (sm_100a) Hierarchical Block Attention hot path.

Public API:
  hba_attention_b200        drop-in for hba_attention_eval  (full forward)
  hba_attention_b200_fused  drop-in for the (out, aux) train-forward contract
  HBADecodeCache            KV/summary cache + incremental decode
  HBAModelDecoder           token-by-token decoding of a converted HBAModel (per-layer caches)
  install                   rebinds a reference hba.model module to this library
  HBAConfig, BASELINE       reference-compatible config and the BASELINE shapes
All compute runs in libhba_b200.so (CUDA); nothing falls back to the CPU.
"""

from ._lib import HBAError, load as load_library
from .attention import (content_scale, hba_attention_b200, hba_attention_b200_fused, hba_attention_b200_range,
                        log_len_tau, union_scale)
from .cache import HBADecodeCache
from .config import BASELINE, HBAConfig, baseline_config
from .decoder import HBAModelDecoder
from .ops import build_super_b200, qknorm_b200, summarize_b200
from .patch import install

__all__ = ["HBAError", "load_library", "content_scale", "log_len_tau", "union_scale", "hba_attention_b200",
           "hba_attention_b200_fused", "hba_attention_b200_range", "HBADecodeCache", "HBAModelDecoder", "HBAConfig", "BASELINE", "baseline_config", "install",
           "qknorm_b200", "summarize_b200", "build_super_b200"]
