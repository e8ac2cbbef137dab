"""Route a reference ``HBAModel`` through the B200 library.

``HBAModel.forward`` (reference src/hba/model.py:119-141) calls the
module-level names ``hba_attention_eval``, ``hba_attention_fused`` and
``hba_attention_dense`` of ``hba.model``.  ``install(hba.model)`` rebinds
those three names to the B200 forwards and returns a function that restores
them, so a converted model runs its eval / eval_hier / train-forward modes on
the CUDA kernels without any other change.  Mode ``equiv`` (dense
uniform-RoPE attention, not the HBA path) keeps the module's own function.
"""

from .attention import hba_attention_b200, hba_attention_b200_fused

NAMES = ("hba_attention_eval", "hba_attention_fused", "hba_attention_dense")


def install(model_module):
    saved = {name: getattr(model_module, name) for name in NAMES if hasattr(model_module, name)}
    orig_eval = saved.get("hba_attention_eval")

    def eval_b200(q, k, v, cos, sin, cfg, summ, qkn, cap, hier=False, equiv=False):
        if equiv:
            if orig_eval is None:
                raise NotImplementedError("equiv mode is not part of the HBA path")
            return orig_eval(q, k, v, cos, sin, cfg, summ, qkn, cap, equiv=True)
        return hba_attention_b200(q, k, v, cos, sin, cfg, summ, qkn, cap, hier=hier)

    def dense_b200(q, k, v, cos, sin, cfg, summ, qkn, equiv=False):
        if equiv:
            raise NotImplementedError("equiv mode is not part of the HBA path")
        return hba_attention_b200_fused(q, k, v, cos, sin, cfg, summ, qkn)

    model_module.hba_attention_eval = eval_b200
    model_module.hba_attention_fused = hba_attention_b200_fused
    model_module.hba_attention_dense = dense_b200

    def restore():
        for name, fn in saved.items():
            setattr(model_module, name, fn)

    return restore
