"""Model and inference context (crates/nr-model): `.nrm` models on the GPU and
the InferCtx surface (new / forward / prefill_chunk / prefill / reset /
logits / remaining / pos) over the nrcuda C ABI.
"""
import ctypes as C

import numpy as np

from . import _lib
from ._lib import check, lib


def gguf_to_nrm(gguf):
    """GGUF bytes -> .nrm v3 blob (numpy uint8), the conversion of
    tools/nrconvert (tensor order, alignment, header and CRCs; empty tokenizer
    section). Raises NrcError for what the converter rejects."""
    buf = np.ascontiguousarray(np.frombuffer(bytes(gguf), np.uint8) if not isinstance(gguf, np.ndarray) else gguf,
                               dtype=np.uint8)
    n = C.c_size_t()
    check(lib().nrc_gguf_to_nrm(buf.ctypes.data_as(C.c_void_p), buf.size, None, 0, C.byref(n)))
    out = np.empty(n.value, np.uint8)
    check(lib().nrc_gguf_to_nrm(buf.ctypes.data_as(C.c_void_p), buf.size, out.ctypes.data_as(C.c_void_p), out.size,
                                C.byref(n)))
    return out


class Model:
    """A `.nrm` model resident in device memory (Model::parse + upload, format.rs:260-406)."""

    def __init__(self, handle, device):
        self.h = handle
        self.device = device
        self.meta = _lib.Meta()
        check(lib().nrc_model_meta(self.h, C.byref(self.meta)))

    @classmethod
    def load(cls, blob, device=0, verify_crc=True):
        buf = np.ascontiguousarray(np.frombuffer(bytes(blob), np.uint8) if not isinstance(blob, np.ndarray) else blob,
                                   dtype=np.uint8)
        h = C.c_void_p()
        check(lib().nrc_model_load(buf.ctypes.data_as(C.c_void_p), buf.size, device, int(verify_crc), C.byref(h)))
        return cls(h, device)

    @classmethod
    def load_gguf(cls, gguf, device=0):
        """A GGUF file's bytes (dense llama / qwen3 / granite; F32, Q8_0, Q4_K,
        Q6_K tensors) converted as tools/nrconvert does and uploaded."""
        buf = np.ascontiguousarray(np.frombuffer(bytes(gguf), np.uint8) if not isinstance(gguf, np.ndarray) else gguf,
                                   dtype=np.uint8)
        h = C.c_void_p()
        check(lib().nrc_model_load_gguf(buf.ctypes.data_as(C.c_void_p), buf.size, device, C.byref(h)))
        return cls(h, device)

    @classmethod
    def synth(cls, cfg, seed, device=0):
        """Seeded synthetic model of a nightrun_b200.configs preset, built on the device."""
        s = _lib.synth_cfg(cfg)
        h = C.c_void_p()
        check(lib().nrc_model_synth(C.byref(s), seed, device, C.byref(h)))
        return cls(h, device)

    def export(self):
        """The model as a complete `.nrm` blob (numpy uint8)."""
        n = lib().nrc_model_nrm_size(self.h)
        out = np.empty(n, np.uint8)
        check(lib().nrc_model_export(self.h, out.ctypes.data_as(C.c_void_p), n))
        return out

    def data_crc(self):
        v = C.c_uint32()
        check(lib().nrc_model_data_crc(self.h, C.byref(v)))
        return v.value

    def required_bytes(self, ctx):
        v = C.c_size_t()
        check(lib().nrc_ctx_required_bytes(self.h, ctx, C.byref(v)))
        return v.value

    def ctx(self, ctx_len, tp=None):
        return InferCtx(self, ctx_len, tp)

    def batch(self, ctx_len, n_seqs):
        return BatchCtx(self, ctx_len, n_seqs)

    def close(self):
        if getattr(self, "h", None):
            lib().nrc_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def tp_unique_id():
    """A fresh NCCL id (bytes) for nrc_tp_ctx_new; create it on one rank and share it."""
    buf = (C.c_uint8 * 128)()
    check(lib().nrc_tp_unique_id(buf))
    return bytes(buf)


class InferCtx:
    """Mirror of nr_model::InferCtx (crates/nr-model/src/infer.rs:264-760).
    With tp=(nranks, rank, id) the context is this rank's part of a
    tensor-parallel group (every rank calls the same methods in order)."""

    MAX_BATCH = _lib.MAX_BATCH

    def __init__(self, model, ctx_len, tp=None):
        self.model = model
        h = C.c_void_p()
        if tp is None:
            check(lib().nrc_ctx_new(model.h, ctx_len, C.byref(h)))
        else:
            nranks, rank, uid = tp
            ub = (C.c_uint8 * 128).from_buffer_copy(uid)
            check(lib().nrc_tp_ctx_new(model.h, ctx_len, nranks, rank, ub, C.byref(h)))
        self.h = h
        self.vocab = model.meta.vocab
        self.ctx_len = ctx_len
        self._logits = np.zeros(self.vocab, np.float32)
        self._next = C.c_uint32()

    def _lp(self):
        return self._logits.ctypes.data_as(C.c_void_p)

    def forward(self, token):
        """One token at the current position (infer.rs:510-595); returns the logits."""
        check(lib().nrc_ctx_forward(self.h, int(token), self._lp(), C.byref(self._next)))
        return self._logits.copy()

    def forward_greedy(self, token):
        """forward + vec::argmax without copying the logits; returns the next token id."""
        check(lib().nrc_ctx_forward(self.h, int(token), None, C.byref(self._next)))
        return self._next.value

    def prefill_chunk(self, tokens):
        """Batched prefill of 1..=64 tokens (infer.rs:601-750); last token's logits."""
        t = np.ascontiguousarray(tokens, np.uint32)
        check(lib().nrc_ctx_prefill_chunk(self.h, t.ctypes.data_as(C.c_void_p), t.size, self._lp(),
                                          C.byref(self._next)))
        return self._logits.copy()

    def prefill(self, tokens):
        """Prefill of any length in chunks of 64 (infer.rs:753-759)."""
        t = np.ascontiguousarray(tokens, np.uint32)
        check(lib().nrc_ctx_prefill(self.h, t.ctypes.data_as(C.c_void_p), t.size, self._lp(), C.byref(self._next)))
        return self._logits.copy()

    def generate(self, first, n):
        """Greedy generation of n tokens after `first`, entirely on the device."""
        out = np.zeros(n, np.uint32)
        check(lib().nrc_ctx_generate(self.h, int(first), n, out.ctypes.data_as(C.c_void_p)))
        return out

    def decode_async(self, n):
        """Enqueue n device-side greedy decode steps (no host round trip)."""
        check(lib().nrc_ctx_decode_async(self.h, n))

    def sync(self):
        """Wait for enqueued steps; returns the last greedy token."""
        check(lib().nrc_ctx_sync(self.h, C.byref(self._next)))
        return self._next.value

    def forward_into(self, token, logits_out_ptr, next_out_ptr):
        """forward() writing the logits/next token into caller-provided (pinned) host buffers."""
        check(lib().nrc_ctx_forward(self.h, int(token), logits_out_ptr, next_out_ptr))

    @property
    def next_token(self):
        """Greedy choice (argmax) of the most recent logits."""
        return self._next.value

    def logits(self):
        return self._logits.copy()

    EXACT, FAST = 0, 1

    def set_mode(self, mode):
        """EXACT (default): bit-identical to the reference's scalar path. FAST:
        decode steps with tree reductions, within the north star's tolerance."""
        check(lib().nrc_ctx_set_mode(self.h, int(mode)))

    def set_sampler(self, temperature, top_p, seed):
        """Attach Sampler::new(temperature, top_p, seed) (sample.rs:15-21): every
        step that returns a next token draws once on the device."""
        check(lib().nrc_ctx_set_sampler(self.h, float(temperature), float(top_p), int(seed) & 0xFFFFFFFFFFFFFFFF))

    def reset(self):
        check(lib().nrc_ctx_reset(self.h))

    @property
    def pos(self):
        return lib().nrc_ctx_pos(self.h)

    def remaining(self):
        return lib().nrc_ctx_remaining(self.h)

    def shard(self):
        """(nranks, rank, q head0, q heads, kv head0, kv heads, dim row0, dim rows,
        ffn row0, ffn rows, vocab row0, vocab rows) of this context."""
        out = (C.c_int32 * 12)()
        check(lib().nrc_tp_shard(self.h, out))
        return tuple(out)

    def kv(self, layer, pos):
        sh = self.shard()
        kvd = sh[5] * self.model.meta.head_dim
        k = np.empty(kvd, np.uint16)
        v = np.empty(kvd, np.uint16)
        check(lib().nrc_ctx_kv(self.h, layer, pos, k.ctypes.data_as(C.c_void_p), v.ctypes.data_as(C.c_void_p)))
        return k, v

    def stream_handle(self):
        return lib().nrc_ctx_stream(self.h)

    def close(self):
        if getattr(self, "h", None):
            lib().nrc_ctx_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class BatchCtx:
    """n_seqs independent sequences decoded together (one InferCtx per stream in
    the reference, crates/nr-model/src/infer.rs:319-778): per-sequence KV caches
    and positions, every linear layer once per pass over all sequences."""

    def __init__(self, model, ctx_len, n_seqs):
        self.model = model
        h = C.c_void_p()
        check(lib().nrc_batch_new(model.h, ctx_len, n_seqs, C.byref(h)))
        self.h = h
        self.n = n_seqs
        self.vocab = model.meta.vocab

    def prefill(self, prompts):
        """Prefill every sequence with its prompt (a list of n_seqs token lists);
        returns each sequence's greedy choice."""
        assert len(prompts) == self.n
        toks = np.ascontiguousarray(np.concatenate([np.asarray(p, np.uint32) for p in prompts]), np.uint32)
        lens = np.array([len(p) for p in prompts], np.uint32)
        nxt = np.zeros(self.n, np.uint32)
        check(lib().nrc_batch_prefill(self.h, toks.ctypes.data_as(C.c_void_p), lens.ctypes.data_as(C.c_void_p),
                                      nxt.ctypes.data_as(C.c_void_p)))
        return nxt

    def step(self, logits=True):
        """One decode step of every sequence; returns (logits [n][vocab] or None, next ids)."""
        nxt = np.zeros(self.n, np.uint32)
        lg = np.zeros((self.n, self.vocab), np.float32) if logits else None
        check(lib().nrc_batch_step(self.h, lg.ctypes.data_as(C.c_void_p) if logits else None,
                                   nxt.ctypes.data_as(C.c_void_p)))
        return lg, nxt

    def generate(self, n):
        """n device-side greedy steps; returns [n_seqs][n] ids."""
        out = np.zeros((self.n, n), np.uint32)
        check(lib().nrc_batch_generate(self.h, n, out.ctypes.data_as(C.c_void_p)))
        return out

    def decode_async(self, n):
        check(lib().nrc_batch_decode_async(self.h, n))

    def sync(self):
        nxt = np.zeros(self.n, np.uint32)
        check(lib().nrc_batch_sync(self.h, nxt.ctypes.data_as(C.c_void_p)))
        return nxt

    def pos(self, seq):
        return lib().nrc_batch_pos(self.h, seq)

    def kv(self, seq, layer, pos):
        kvd = self.model.meta.n_kv_heads * self.model.meta.head_dim
        k = np.empty(kvd, np.uint16)
        v = np.empty(kvd, np.uint16)
        check(lib().nrc_batch_kv(self.h, seq, layer, pos, k.ctypes.data_as(C.c_void_p),
                                 v.ctypes.data_as(C.c_void_p)))
        return k, v

    def reset(self):
        check(lib().nrc_ctx_reset(self.h))

    def stream_handle(self):
        return lib().nrc_ctx_stream(self.h)

    def close(self):
        if getattr(self, "h", None):
            lib().nrc_ctx_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
