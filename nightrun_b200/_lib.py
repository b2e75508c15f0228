"""ctypes binding of libnrcuda.so (include/nrcuda.h).

The library is built in-tree (nightrun_b200/libnrcuda.so, see build.py). There
is no CPU fallback: importing a compute entry point without the library raises.
"""
import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libnrcuda.so")

ERRORS = {
    0: "OK", -1: "INVALID", -2: "CUDA", -3: "ALLOC", -4: "DEVICE", -10: "TOO_SHORT", -11: "BAD_MAGIC",
    -12: "BAD_VERSION", -13: "META_CRC", -14: "BAD_TABLE", -15: "MISSING", -16: "DATA_CRC", -17: "UNSUPPORTED",
    -20: "CTX_FULL", -21: "BAD_BATCH", -22: "BAD_TOKEN",
}
for _code, _name in ERRORS.items():
    if _code:
        globals()["NRC_ERR_" + _name] = _code
MAX_BATCH = 64
NOALLOC_MAX_COLS = 16384


class NrcError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"nrcuda error {ERRORS.get(code, code)} ({code}): {msg}")
        self.code = code
        self.name = ERRORS.get(code, str(code))


class Meta(C.Structure):
    _fields_ = [("arch", C.c_int32)] + \
               [(n, C.c_uint32) for n in ("dim", "n_layers", "n_heads", "n_kv_heads", "head_dim", "ffn_dim",
                                          "vocab", "ctx_train")] + \
               [(n, C.c_float) for n in ("rope_theta", "norm_eps", "rope_factor", "rope_low", "rope_high",
                                         "rope_orig_ctx")] + \
               [("flags", C.c_uint32)] + \
               [(n, C.c_float) for n in ("embed_scale", "attn_scale", "residual_scale", "logit_scale")] + \
               [("name", C.c_char * 48)]


class SynthCfg(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in ("arch", "dim", "n_layers", "n_heads", "n_kv_heads", "head_dim",
                                          "ffn_dim", "vocab", "ctx_train")] + \
               [(n, C.c_float) for n in ("rope_theta", "norm_eps", "rope_factor", "rope_low", "rope_high",
                                         "rope_orig_ctx", "embed_scale", "attn_scale", "residual_scale",
                                         "logit_scale")] + \
               [("quant", C.c_uint32), ("tied", C.c_uint32), ("rope_freqs_tensor", C.c_uint32),
                ("name", C.c_char * 48)]


def synth_cfg(cfg):
    s = SynthCfg()
    for k, _ in SynthCfg._fields_:
        if k == "name":
            s.name = cfg.get("name", "synthetic").encode()[:47]
        else:
            setattr(s, k, cfg[k])
    return s


_LIB = None

# (name, restype, argtypes) of every exported entry point.
P, S, F, I, U32, U64 = C.c_void_p, C.c_size_t, C.c_float, C.c_int, C.c_uint32, C.c_uint64
SIGNATURES = [
    ("nrc_last_error", C.c_char_p, []),
    ("nrc_version", I, []),
    ("nrc_sync_check", I, [P]),
    ("nrc_wait_selftest", I, [I, U64, P]),
    ("nrc_quantize_q8_0", I, [P, P, S, P]),
    ("nrc_dequantize_q8_0", I, [P, P, S, P]),
    ("nrc_quantize_q8k", I, [P, P, S, P]),
    ("nrc_dequant_q4k", I, [P, P, S, P]),
    ("nrc_dequant_q6k", I, [P, P, S, P]),
    ("nrc_matvec_q8_0", I, [P, P, P, S, S, P]),
    ("nrc_matmul_q8_0", I, [P, P, P, S, S, S, P]),
    ("nrc_matmul_q8_0_noalloc", I, [P, P, P, S, S, S, P]),
    ("nrc_matvec_q4k", I, [P, P, P, S, S, P]),
    ("nrc_matvec_q6k", I, [P, P, P, S, S, P]),
    ("nrc_matmul_q4k", I, [P, P, P, S, S, S, P]),
    ("nrc_matmul_q6k", I, [P, P, P, S, S, S, P]),
    ("nrc_f32_to_f16", I, [P, P, S, P]),
    ("nrc_f16_to_f32", I, [P, P, S, P]),
    ("nrc_rmsnorm", I, [P, P, P, S, S, F, P]),
    ("nrc_softmax", I, [P, S, S, P]),
    ("nrc_swiglu", I, [P, P, S, P]),
    ("nrc_argmax", I, [P, S, P, P]),
    ("nrc_expf", I, [P, P, S, P]),
    ("nrc_expf_hash", I, [P, I, I, P]),
    ("nrc_sample", I, [P, S, F, F, P, P, P]),
    ("nrc_rope_freqs", I, [P, S, F, F, F, F, F]),
    ("nrc_rope_apply", I, [P, S, S, P, S, I, P]),
    ("nrc_model_load", I, [P, S, I, I, C.POINTER(P)]),
    ("nrc_gguf_to_nrm", I, [P, S, P, S, C.POINTER(S)]),
    ("nrc_model_load_gguf", I, [P, S, I, C.POINTER(P)]),
    ("nrc_model_synth", I, [C.POINTER(SynthCfg), U64, I, C.POINTER(P)]),
    ("nrc_model_meta", I, [P, C.POINTER(Meta)]),
    ("nrc_model_nrm_size", S, [P]),
    ("nrc_model_export", I, [P, P, S]),
    ("nrc_model_data_crc", I, [P, C.POINTER(U32)]),
    ("nrc_model_free", I, [P]),
    ("nrc_ctx_required_bytes", I, [P, S, C.POINTER(S)]),
    ("nrc_ctx_new", I, [P, S, C.POINTER(P)]),
    ("nrc_ctx_free", I, [P]),
    ("nrc_ctx_forward", I, [P, U32, P, P]),
    ("nrc_ctx_prefill_chunk", I, [P, P, S, P, P]),
    ("nrc_ctx_prefill", I, [P, P, S, P, P]),
    ("nrc_ctx_generate", I, [P, U32, S, P]),
    ("nrc_ctx_decode_async", I, [P, S]),
    ("nrc_ctx_sync", I, [P, P]),
    ("nrc_ctx_set_sampler", I, [P, F, F, U64]),
    ("nrc_ctx_set_mode", I, [P, I]),
    ("nrc_ctx_reset", I, [P]),
    ("nrc_ctx_pos", S, [P]),
    ("nrc_ctx_remaining", S, [P]),
    ("nrc_ctx_logits_device", I, [P, C.POINTER(P)]),
    ("nrc_ctx_stream", P, [P]),
    ("nrc_ctx_kv", I, [P, S, S, P, P]),
    ("nrc_tp_unique_id", I, [P]),
    ("nrc_tp_ctx_new", I, [P, S, I, I, P, C.POINTER(P)]),
    ("nrc_tp_shard", I, [P, P]),
    ("nrc_batch_new", I, [P, S, S, C.POINTER(P)]),
    ("nrc_batch_prefill", I, [P, P, P, P]),
    ("nrc_batch_step", I, [P, P, P]),
    ("nrc_batch_generate", I, [P, S, P]),
    ("nrc_batch_decode_async", I, [P, S]),
    ("nrc_batch_sync", I, [P, P]),
    ("nrc_batch_size", S, [P]),
    ("nrc_batch_pos", S, [P, S]),
    ("nrc_batch_kv", I, [P, S, S, S, P, P]),
]


def lib(path=LIB_PATH):
    """Load libnrcuda.so (once). Raises if it is missing: there is no fallback."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(path):
            raise RuntimeError(f"libnrcuda.so not built at {path}: run `python -m nightrun_b200.build`")
        L = C.CDLL(path)
        for name, res, args in SIGNATURES:
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


def check(rc):
    if rc != 0:
        raise NrcError(rc, lib().nrc_last_error().decode(errors="replace"))
    return rc
