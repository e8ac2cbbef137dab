"""Loader of ``tests/golden/model_layer.npz``: layer 0 of the reference's own
``HBAModel`` (tiny random Qwen2 donor, q/k projections scaled to a trained
donor's magnitude, QKNorm gains from the reference's ``init_qknorm_gains``,
gain_q * gain_k ~ 81), written by ``make_model_golden.py`` from the
reference itself.  Holds the q/k/v that ``HBAModel.forward``'s ``block_fn``
hands to ``hba_attention_eval`` (rounded to bf16), the layer's summarizer
weights and gains, and the reference's ``hba_attention_eval`` outputs on
those exact values (fp32) at sampled rows, flat and hierarchical."""

import json
import os

import numpy as np

PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "model_layer.npz")


def unbits(b):
    return (np.asarray(b).astype(np.uint32) << 16).view(np.float32)


def load():
    z = np.load(PATH)
    cfg = json.loads(str(z["cfg"]))
    return dict(cfg=cfg, q=unbits(z["q_bits"]), k=unbits(z["k_bits"]), v=unbits(z["v_bits"]),
                probes=z["probes"], proj=z["proj"], q_gain=z["q_gain"], k_gain=z["k_gain"], rows=z["rows"],
                out_eval=z["out_eval"], out_eval_hier=z["out_eval_hier"])


def oracle_cfg(cfg):
    return dict(block=cfg["block"], window=cfg["window"], sinks=cfg["sinks"], k_blocks=cfg["k_blocks"],
                fanout=cfg["fanout"], beam=cfg["beam"], qknorm=cfg["qknorm"],
                content_scale_mode=cfg["content_scale_mode"], temp_c=cfg["temp_c"], n_cal=cfg["n_cal"],
                native_ctx=cfg["native_ctx"])
