"""nightrun_b200 — B200 (sm_100a) implementation of NIGHTRUN's quantized
transformer forward path behind a C ABI (include/nrcuda.h).

    from nightrun_b200 import Model, configs
    m = Model.synth(configs.CONFIGS["llama1b_q8"], configs.MODEL_SEED)
    ctx = m.ctx(256)
    logits = ctx.prefill(ids)
"""
from . import configs
from ._lib import NrcError, lib
from .infer import BatchCtx, InferCtx, Model, gguf_to_nrm, tp_unique_id

__all__ = ["configs", "lib", "Model", "InferCtx", "BatchCtx", "NrcError", "gguf_to_nrm", "tp_unique_id"]
