"""Component ops of the hot path, one C-ABI call each, mirroring the
reference functions they replace:

* ``qknorm_b200``        -- ``_HeadRMSNorm.forward`` (src/hba/attention.py:88-94)
* ``summarize_b200``     -- ``SlotSummarizer.summarize`` (src/hba/summarizer.py:34-42)
* ``build_super_b200``   -- ``build_super`` (src/hba/attention.py:202-214)
"""

import ctypes

import torch

from . import _lib
from .attention import as_bf16, as_f32, c_config, ptr, stream_of


def qknorm_b200(x, gain, eps=1e-6):
    """x: [..., H, dh] -> bf16 x / sqrt(max(mean(x^2), eps)) * gain[h]."""
    xb = as_bf16(x)
    H, dh = xb.shape[-2], xb.shape[-1]
    rows = xb.numel() // (H * dh)
    y = torch.empty_like(xb)
    with torch.cuda.device(xb.device):
        g = as_f32(gain, xb.device)
        st = _lib.load().hba_b200_qknorm(ptr(xb), ptr(y), ptr(g), rows, H, dh, ctypes.c_float(eps),
                                         stream_of(xb.device))
    _lib.check(st, "hba_b200_qknorm")
    return y


def summarize_b200(kc, probes, proj, cfg):
    """kc: [B, n, Hkv, dh] QKNorm'd keys -> S [B, Hkv, n/block, m, dh] bf16."""
    kb = as_bf16(kc)
    B, n, Hkv, dh = kb.shape
    nb = n // cfg.block
    c = c_config(cfg, False)
    S = torch.empty(B, Hkv, nb, cfg.slots, dh, dtype=torch.bfloat16, device=kb.device)
    with torch.cuda.device(kb.device):
        pr, pj = as_f32(probes, kb.device), as_f32(proj, kb.device)
        st = _lib.load().hba_b200_summarize(ctypes.byref(c), B, n - n % cfg.block, ptr(kb), ptr(pr), ptr(pj),
                                            ptr(S), 0, nb, stream_of(kb.device))
    _lib.check(st, "hba_b200_summarize")
    return S


def build_super_b200(S0, cfg, nb=None):
    """S0: [B, Hkv, nb_cap, m, dh] -> (S1 [B, Hkv, ceil(nb/F), m, dh] bf16, ns),
    the mean over the first `nb` blocks (default all)."""
    Sb = as_bf16(S0)
    B, Hkv, nb_cap, m, dh = Sb.shape
    nb = nb_cap if nb is None else nb
    F = cfg.fanout
    ns = -(-nb // F)
    ns_cap = -(-nb_cap // F)
    c = c_config(cfg, True)
    S1 = torch.zeros(B, Hkv, ns_cap, m, dh, dtype=torch.bfloat16, device=Sb.device)
    with torch.cuda.device(Sb.device):
        st = _lib.load().hba_b200_build_supers(ctypes.byref(c), B, nb_cap, nb, ptr(Sb), ptr(S1), 0, ns,
                                               stream_of(Sb.device))
    _lib.check(st, "hba_b200_build_supers")
    return S1[:, :, :ns], ns
