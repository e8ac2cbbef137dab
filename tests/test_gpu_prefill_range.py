"""The query-range prefill (hba_b200_prefill_range): rows [q_lo, q_lo + n_q)
over the keys of tokens [0, n) must equal those rows of the full prefill --
the piece one rank computes in a prefill split by token range."""

import pytest
import torch

import gpu_helpers as H
from hba_b200 import hba_attention_b200, hba_attention_b200_range, synth

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("q_lo,n_q", [(1024, 512), (576, 448), (0, 320), (1600, 448)])
@pytest.mark.parametrize("gains", [True, "trained"])
def test_range_rows_equal_full_prefill_rows(q_lo, n_q, gains):
    cfg = H.cfg_of(n_heads=8, n_kv=2, head_dim=128, native_ctx=1024)   # tau(2048) != 1: the scale of the whole length
    N = 2048
    summ, qkn = synth.make_weights(cfg, "cuda", seed=81, gains=gains)
    cos, sin = synth.rope_tables(N, cfg.head_dim, 1e6)
    wl = synth.prefill_workload(cfg, 2, N, seed=81)
    q, k, v = wl["q"], wl["k"], wl["v"]
    with torch.no_grad():
        out, lse, (si, ss) = hba_attention_b200(q, k, v, cos, sin, cfg, summ, qkn, return_lse=True,
                                                return_selection=True)
        hi = q_lo + n_q
        o2, l2, (si2, ss2) = hba_attention_b200_range(q[:, q_lo:hi], k[:, :hi], v[:, :hi], cos, sin, cfg, summ, qkn,
                                                      q_lo=q_lo, n_total=N, return_lse=True, return_selection=True)
    torch.cuda.synchronize()
    assert torch.equal(si2, si[:, :, q_lo:hi])
    assert torch.equal(ss2, ss[:, :, q_lo:hi])
    assert (o2.float() - out[:, q_lo:hi].float()).abs().max().item() <= 1e-2
    assert (l2 - lse[:, :, q_lo:hi]).abs().max().item() <= 1e-4


def test_range_rejects_paths_without_the_tensor_cores():
    cfg = H.cfg_of(n_heads=4, n_kv=2)   # G = 2: no tensor-core union
    summ, qkn = synth.make_weights(cfg, "cuda")
    q = torch.zeros(1, 64, 4, 64, device="cuda", dtype=torch.bfloat16)
    k = torch.zeros(1, 128, 2, 64, device="cuda", dtype=torch.bfloat16)
    cos, sin = synth.rope_tables(128, 64, 1e6)
    with pytest.raises(NotImplementedError):
        hba_attention_b200_range(q, k, k, cos, sin, cfg, summ, qkn, q_lo=64)
