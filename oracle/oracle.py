"""TEST INFRASTRUCTURE ONLY — ctypes wrapper of the CPU oracle (oracle/liboracle.so).

The oracle restates the reference's Rust kernels and forward pass in C++
(see oracle/oracle.h). Only tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline legs import this module; the product package never does.
"""
import ctypes as C
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")

# Block layouts (crates/nr-tensor/src/q8.rs:11-14, kquant.rs:26-52).
Q8_0 = np.dtype([("d", "<u2"), ("qs", "i1", 32)])
Q4K = np.dtype([("d", "<u2"), ("dmin", "<u2"), ("scales", "u1", 12), ("qs", "u1", 128)])
Q6K = np.dtype([("ql", "u1", 128), ("qh", "u1", 64), ("scales", "i1", 16), ("d", "<u2")])
Q8K = np.dtype([("d", "<f4"), ("qs", "i1", 256), ("bsums", "<i2", 16)])
assert Q8_0.itemsize == 34 and Q4K.itemsize == 144 and Q6K.itemsize == 210 and Q8K.itemsize == 292

PE = {0: "ok", -1: "TooShort", -2: "BadMagic", -3: "BadVersion", -4: "MetaCrc", -5: "BadTable",
      -6: "MissingTensor", -20: "ContextFull", -21: "BadBatch", -22: "BadToken"}


class SynthCfg(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in ("arch", "dim", "n_layers", "n_heads", "n_kv_heads",
                                          "head_dim", "ffn_dim", "vocab", "ctx_train")] + \
               [(n, C.c_float) for n in ("rope_theta", "norm_eps", "rope_factor", "rope_low",
                                         "rope_high", "rope_orig_ctx", "embed_scale", "attn_scale",
                                         "residual_scale", "logit_scale")] + \
               [("quant", C.c_uint32), ("tied", C.c_uint32), ("rope_freqs_tensor", C.c_uint32),
                ("name", C.c_char * 48)]


class Meta(C.Structure):
    _fields_ = [("arch", C.c_int)] + \
               [(n, C.c_uint32) for n in ("dim", "n_layers", "n_heads", "n_kv_heads", "head_dim",
                                          "ffn_dim", "vocab", "ctx_train")] + \
               [(n, C.c_float) for n in ("rope_theta", "norm_eps", "rope_factor", "rope_low",
                                         "rope_high", "rope_orig_ctx")] + \
               [("flags", C.c_uint32)] + \
               [(n, C.c_float) for n in ("embed_scale", "attn_scale", "residual_scale", "logit_scale")] + \
               [("name", C.c_char * 48)]


class TensorEntry(C.Structure):
    _fields_ = [("kind", C.c_uint16), ("layer", C.c_uint16), ("dtype", C.c_uint16),
                ("offset", C.c_uint64), ("size", C.c_uint64), ("rows", C.c_uint32), ("cols", C.c_uint32)]


def cfg_struct(cfg):
    """Build a SynthCfg from a model-config dict (nightrun_b200.configs layout)."""
    s = SynthCfg()
    for k, _ in SynthCfg._fields_:
        if k == "name":
            s.name = cfg.get("name", "synthetic").encode()[:47]
        else:
            setattr(s, k, cfg[k])
    return s


class Oracle:
    def __init__(self, path=_LIB_PATH):
        if not os.path.exists(path):
            raise RuntimeError(f"oracle library missing: {path} (run oracle/build.sh)")
        L = self.L = C.CDLL(path)
        P, S, F, I, U32, U64 = C.c_void_p, C.c_size_t, C.c_float, C.c_int, C.c_uint32, C.c_uint64
        sig = {
            "or_set_mode": (None, [I, I]), "or_pool_start": (None, [I]), "or_pool_threads": (I, []),
            "or_expf": (None, [P, P, S]), "or_expf_hash": (None, [P, I, I]),
            "or_f16_to_f32": (None, [P, P, S]), "or_f32_to_f16": (None, [P, P, S]),
            "or_q8_quantize": (None, [P, S, P]), "or_q8_dequantize": (None, [P, S, P]),
            "or_quantize_q8k": (None, [P, S, P]), "or_dequant_q4k": (None, [P, S, P]),
            "or_dequant_q6k": (None, [P, S, P]), "or_quantize_q4k_ref": (None, [P, S, P]),
            "or_quantize_q6k_ref": (None, [P, S, P]),
            "or_dot_q8": (F, [P, P, S, I]), "or_dot_q4k": (F, [P, P, S, I]), "or_dot_q6k": (F, [P, P, S, I]),
            "or_matvec_q8": (None, [P, P, P, S, S]), "or_matmul_q8": (None, [P, P, P, S, S, S]),
            "or_matvec_q4k": (None, [P, P, P, S, S]), "or_matvec_q6k": (None, [P, P, P, S, S]),
            "or_matmul_q4k": (None, [P, P, P, S, S, S]), "or_matmul_q6k": (None, [P, P, P, S, S, S]),
            "or_dot_f16": (F, [P, P, S]), "or_axpy_f16": (None, [P, F, P, S]),
            "or_rmsnorm": (None, [P, P, P, S, F]), "or_rmsnorm_inplace": (None, [P, P, S, F]),
            "or_softmax": (None, [P, S]), "or_swiglu": (None, [P, P, S]), "or_argmax": (S, [P, S]),
            "or_saxpy": (None, [P, F, P, S]), "or_scale_inplace": (None, [P, S, F]),
            "or_rope_freqs": (None, [P, S, F, F, F, F, F]), "or_rope_apply": (None, [P, S, S, P, S, I]),
            "or_crc32": (U32, [P, S]),
            "or_model_parse": (I, [P, S, C.POINTER(P)]), "or_model_free": (None, [P]),
            "or_model_meta": (None, [P, C.POINTER(Meta)]), "or_model_verify": (I, [P]),
            "or_model_tensor_count": (S, [P]), "or_model_tensor": (I, [P, S, C.POINTER(TensorEntry)]),
            "or_ctx_new": (I, [P, S, C.POINTER(P)]), "or_ctx_free": (None, [P]),
            "or_ctx_forward": (I, [P, U32, P]), "or_ctx_prefill_chunk": (I, [P, P, S, P]),
            "or_ctx_prefill": (I, [P, P, S, P]), "or_ctx_reset": (None, [P]), "or_ctx_pos": (S, [P]),
            "or_ctx_kv": (I, [P, S, S, P, P]),
            "or_sampler_sample": (U32, [F, F, C.POINTER(U64), P, S]),
            "or_synth_size": (U64, [C.POINTER(SynthCfg)]),
            "or_synth_write": (I, [C.POINTER(SynthCfg), U64, P, U64, I]),
            "or_synth_gauss": (F, [U64, U64]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args

    # ---- helpers ----
    @staticmethod
    def _p(a):
        return a.ctypes.data_as(C.c_void_p)

    def set_mode(self, fast_path, fast_f16=None):
        """fast_path=True selects the AVX2 kernels (the x86 path), False the scalar ones."""
        self.L.or_set_mode(int(fast_path), int(fast_path if fast_f16 is None else fast_f16))

    def pool_start(self, threads):
        self.L.or_pool_start(int(threads))

    def f16_to_f32(self, bits):
        bits = np.ascontiguousarray(bits, dtype=np.uint16)
        out = np.empty(bits.shape, np.float32)
        self.L.or_f16_to_f32(self._p(bits), self._p(out), bits.size)
        return out

    def f32_to_f16(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty(x.shape, np.uint16)
        self.L.or_f32_to_f16(self._p(x), self._p(out), x.size)
        return out

    def q8_quantize(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32).ravel()
        out = np.zeros(x.size // 32, Q8_0)
        self.L.or_q8_quantize(self._p(x), x.size, self._p(out))
        return out

    def q8_dequantize(self, b):
        out = np.empty(b.size * 32, np.float32)
        self.L.or_q8_dequantize(self._p(b), out.size, self._p(out))
        return out

    def quantize_q8k(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32).ravel()
        out = np.zeros(x.size // 256, Q8K)
        self.L.or_quantize_q8k(self._p(x), x.size, self._p(out))
        return out

    def dequant_q4k(self, b):
        out = np.empty(b.size * 256, np.float32)
        self.L.or_dequant_q4k(self._p(b), b.size, self._p(out))
        return out

    def dequant_q6k(self, b):
        out = np.empty(b.size * 256, np.float32)
        self.L.or_dequant_q6k(self._p(b), b.size, self._p(out))
        return out

    def quantize_q4k_ref(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32).ravel()
        out = np.zeros(x.size // 256, Q4K)
        self.L.or_quantize_q4k_ref(self._p(x), out.size, self._p(out))
        return out

    def quantize_q6k_ref(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32).ravel()
        out = np.zeros(x.size // 256, Q6K)
        self.L.or_quantize_q6k_ref(self._p(x), out.size, self._p(out))
        return out

    def dot(self, fmt, w, x, mode=0):
        fn = {"q8_0": self.L.or_dot_q8, "q4k": self.L.or_dot_q4k, "q6k": self.L.or_dot_q6k}[fmt]
        return fn(self._p(w), self._p(x), w.size, mode)

    def matvec(self, fmt, w, x, rows, cols):
        y = np.empty(rows, np.float32)
        fn = {"q8_0": self.L.or_matvec_q8, "q4k": self.L.or_matvec_q4k, "q6k": self.L.or_matvec_q6k}[fmt]
        fn(self._p(y), self._p(w), self._p(x), rows, cols)
        return y

    def matmul(self, fmt, w, xs, rows, cols, batch):
        y = np.empty(batch * rows, np.float32)
        fn = {"q8_0": self.L.or_matmul_q8, "q4k": self.L.or_matmul_q4k, "q6k": self.L.or_matmul_q6k}[fmt]
        fn(self._p(y), self._p(w), self._p(xs), rows, cols, batch)
        return y.reshape(batch, rows)

    def dot_f16(self, k, q):
        return self.L.or_dot_f16(self._p(k), self._p(q), k.size)

    def rmsnorm(self, x, w, eps):
        x = np.ascontiguousarray(x, np.float32)
        w = np.ascontiguousarray(w, np.float32)
        out = np.empty_like(x)
        self.L.or_rmsnorm(self._p(out), self._p(x), self._p(w), x.size, eps)
        return out

    def rmsnorm_inplace(self, x, w, eps):
        x = np.array(x, np.float32)
        w = np.ascontiguousarray(w, np.float32)
        self.L.or_rmsnorm_inplace(self._p(x), self._p(w), x.size, eps)
        return x

    def expf(self, x):
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty_like(x)
        self.L.or_expf(self._p(x), self._p(y), x.size)
        return y

    def expf_hash(self, chunk0, nchunks):
        out = np.empty(nchunks, np.uint64)
        self.L.or_expf_hash(self._p(out), chunk0, nchunks)
        return out

    def softmax(self, x):
        x = np.array(x, np.float32)
        self.L.or_softmax(self._p(x), x.size)
        return x

    def swiglu(self, g, u):
        g = np.array(g, np.float32)
        u = np.ascontiguousarray(u, np.float32)
        self.L.or_swiglu(self._p(g), self._p(u), g.size)
        return g

    def argmax(self, x):
        x = np.ascontiguousarray(x, np.float32)
        return self.L.or_argmax(self._p(x), x.size)

    def sample(self, logits, temperature, top_p, state):
        """Sampler::sample (sample.rs:32-96) with xorshift state `state` (already
        seed | 1); returns (token, new state)."""
        x = np.ascontiguousarray(logits, np.float32)
        st = C.c_uint64(state)
        tok = self.L.or_sampler_sample(temperature, top_p, C.byref(st), self._p(x), x.size)
        return int(tok), int(st.value)

    def rope_freqs(self, head_dim, theta, scaling=None):
        out = np.empty(head_dim // 2, np.float32)
        f, lo, hi, orig = scaling if scaling else (0.0, 0.0, 0.0, 0.0)
        self.L.or_rope_freqs(self._p(out), head_dim, theta, f, lo, hi, orig)
        return out

    def rope_apply(self, x, head_dim, freqs, pos, style):
        x = np.array(x, np.float32)
        freqs = np.ascontiguousarray(freqs, np.float32)
        self.L.or_rope_apply(self._p(x), x.size, head_dim, self._p(freqs), pos, style)
        return x

    def crc32(self, data):
        data = np.frombuffer(bytes(data), np.uint8) if not isinstance(data, np.ndarray) else data
        return self.L.or_crc32(self._p(data), data.size)

    # ---- model ----
    def synth_nrm(self, cfg, seed, threads=8):
        s = cfg_struct(cfg)
        n = self.L.or_synth_size(C.byref(s))
        buf = np.empty(n, np.uint8)
        rc = self.L.or_synth_write(C.byref(s), seed, self._p(buf), n, threads)
        if rc:
            raise RuntimeError(f"synth failed {rc}")
        return buf

    def model(self, blob):
        return OracleModel(self, blob)


class OracleModel:
    def __init__(self, orc, blob):
        self.orc, self.blob = orc, np.ascontiguousarray(blob, np.uint8)
        h = C.c_void_p()
        rc = orc.L.or_model_parse(Oracle._p(self.blob), self.blob.size, C.byref(h))
        if rc:
            raise ValueError(f"parse error {PE.get(rc, rc)}")
        self.h = h
        self.meta = Meta()
        orc.L.or_model_meta(h, C.byref(self.meta))

    def tensors(self):
        out = []
        for i in range(self.orc.L.or_model_tensor_count(self.h)):
            e = TensorEntry()
            self.orc.L.or_model_tensor(self.h, i, C.byref(e))
            out.append((e.kind, e.layer, e.dtype, e.offset, e.size, e.rows, e.cols))
        return out

    def verify(self):
        return bool(self.orc.L.or_model_verify(self.h))

    def ctx(self, ctx_len):
        return OracleCtx(self, ctx_len)

    def __del__(self):
        if getattr(self, "h", None):
            self.orc.L.or_model_free(self.h)
            self.h = None


class OracleCtx:
    """Mirror of nr_model::InferCtx (crates/nr-model/src/infer.rs:264-760)."""

    def __init__(self, model, ctx_len):
        self.model, self.orc = model, model.orc
        h = C.c_void_p()
        rc = self.orc.L.or_ctx_new(model.h, ctx_len, C.byref(h))
        if rc:
            raise ValueError(f"ctx error {PE.get(rc, rc)}")
        self.h = h
        self.vocab = model.meta.vocab
        self.logits = np.zeros(self.vocab, np.float32)

    def forward(self, token):
        rc = self.orc.L.or_ctx_forward(self.h, int(token), Oracle._p(self.logits))
        if rc:
            raise ValueError(PE.get(rc, rc))
        return self.logits.copy()

    def prefill_chunk(self, tokens):
        t = np.ascontiguousarray(tokens, np.uint32)
        rc = self.orc.L.or_ctx_prefill_chunk(self.h, Oracle._p(t), t.size, Oracle._p(self.logits))
        if rc:
            raise ValueError(PE.get(rc, rc))
        return self.logits.copy()

    def prefill(self, tokens):
        t = np.ascontiguousarray(tokens, np.uint32)
        rc = self.orc.L.or_ctx_prefill(self.h, Oracle._p(t), t.size, Oracle._p(self.logits))
        if rc:
            raise ValueError(PE.get(rc, rc))
        return self.logits.copy()

    def reset(self):
        self.orc.L.or_ctx_reset(self.h)

    @property
    def pos(self):
        return self.orc.L.or_ctx_pos(self.h)

    def kv(self, layer, pos, kv_dim):
        k = np.empty(kv_dim, np.uint16)
        v = np.empty(kv_dim, np.uint16)
        if self.orc.L.or_ctx_kv(self.h, layer, pos, Oracle._p(k), Oracle._p(v)):
            raise IndexError("kv out of range")
        return k, v

    def __del__(self):
        if getattr(self, "h", None):
            self.orc.L.or_ctx_free(self.h)
            self.h = None


_ORACLE = None


def get():
    global _ORACLE
    if _ORACLE is None:
        _ORACLE = Oracle()
    return _ORACLE
