"""B200-native megakernel for REKI's action-expert Euler loop (steps 2..N).

Public API mirrors the reference's ``src/mk_expert.py``: ``ExpertMegakernel`` and ``install``.
Importing ``reki_megakernel_b200.mk_expert`` loads the CUDA library ``libmkx.so``; there is no
CPU fallback.
"""
from .synthetic import ExpertDims, ExpertWeights, StepInputs, make_inputs, make_model, make_past, make_weights

__all__ = ["ExpertDims", "ExpertWeights", "StepInputs", "make_inputs", "make_model", "make_past", "make_weights",
           "ExpertMegakernel", "install", "RegisterPrepare", "register_prepare"]


def __getattr__(name):
    if name in ("ExpertMegakernel", "install"):
        from . import mk_expert
        return getattr(mk_expert, name)
    if name in ("RegisterPrepare", "register_prepare"):
        from . import prepare
        return getattr(prepare, name)
    raise AttributeError(name)
