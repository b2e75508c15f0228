"""Test data for GGUF ingestion: a GGUF v3 writer (the file layout
tools/nrconvert/src/gguf.rs reads: magic, version, counts, metadata KVs,
tensor infos, data section aligned to general.alignment) and the GGUF form of
a `.nrm` model (tensor names and metadata keys of tools/nrconvert/src/main.rs:
201-315), so a conversion can be checked against the model it came from."""
import struct

import numpy as np

HEADER = 192
NAME_LEN = 48
ENTRY = 32
ARCH_NAMES = {1: "llama", 2: "qwen3", 3: "granite"}
GGML_OF_DTYPE = {0: 0, 1: 8, 2: 12, 3: 14}  # .nrm dtype -> ggml type (F32, Q8_0, Q4_K, Q6_K)
LAYER_NAMES = {10: "attn_norm", 11: "attn_q", 12: "attn_k", 13: "attn_v", 14: "attn_output", 15: "ffn_norm",
               16: "ffn_gate", 17: "ffn_up", 18: "ffn_down", 19: "attn_q_norm", 20: "attn_k_norm"}
GLOBAL_NAMES = {1: "token_embd", 2: "output_norm", 3: "output", 4: "rope_freqs"}

# GGUF value types
U8, I8, U16, I16, U32, I32, F32, BOOL, STR, ARR, U64, I64, F64 = range(13)


def nrm_fields(blob):
    """Header fields and tensor table of a .nrm v3 blob (format.rs:97-215)."""
    b = bytes(blob)
    h = {
        "arch": struct.unpack_from("<I", b, 8)[0],
        "dims": struct.unpack_from("<8I", b, 12),
        "floats": struct.unpack_from("<6f", b, 44),
        "flags": struct.unpack_from("<I", b, 68)[0],
        "mup": struct.unpack_from("<4f", b, 72),
        "name": b[88:88 + NAME_LEN].rstrip(b"\0").decode("utf-8", "replace"),
        "tok_off": struct.unpack_from("<Q", b, 136)[0],
        "tok_len": struct.unpack_from("<Q", b, 144)[0],
        "table_off": struct.unpack_from("<Q", b, 152)[0],
        "count": struct.unpack_from("<I", b, 160)[0],
        "data_off": struct.unpack_from("<Q", b, 168)[0],
        "data_size": struct.unpack_from("<Q", b, 176)[0],
        "data_crc": struct.unpack_from("<I", b, 184)[0],
        "meta_crc": struct.unpack_from("<I", b, 188)[0],
    }
    table = []
    for i in range(h["count"]):
        kind, layer, dtype, _, off, size, rows, cols = struct.unpack_from("<4HQQII", b, h["table_off"] + i * ENTRY)
        table.append((kind, layer, dtype, off, size, rows, cols))
    return h, table


def tensor_name(kind, layer):
    if kind in LAYER_NAMES:
        return f"blk.{layer}.{LAYER_NAMES[kind]}.weight"
    return f"{GLOBAL_NAMES[kind]}.weight"


class GgufWriter:
    def __init__(self, alignment=32, version=3):
        self.kv = []
        self.tensors = []  # (name, dims, ggml type, bytes)
        self.alignment = alignment
        self.version = version

    def add(self, key, vtype, value):
        self.kv.append((key, vtype, value))

    def tensor(self, name, dims, gtype, data):
        self.tensors.append((name, list(dims), gtype, bytes(data)))

    @staticmethod
    def _str(s):
        b = s.encode() if isinstance(s, str) else s
        return struct.pack("<Q", len(b)) + b

    def _value(self, vtype, v):
        if vtype == STR:
            return self._str(v)
        if vtype == ARR:
            etype, items = v
            return struct.pack("<IQ", etype, len(items)) + b"".join(self._value(etype, x) for x in items)
        fmt = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<B", U64: "<Q",
               I64: "<q", F64: "<d"}[vtype]
        return struct.pack(fmt, v)

    def bytes(self):
        out = bytearray(b"GGUF" + struct.pack("<IQQ", self.version, len(self.tensors), len(self.kv)))
        for key, vtype, value in self.kv:
            out += self._str(key) + struct.pack("<I", vtype) + self._value(vtype, value)
        offs, cur = [], 0
        for _, _, _, data in self.tensors:
            cur = (cur + self.alignment - 1) // self.alignment * self.alignment
            offs.append(cur)
            cur += len(data)
        for (name, dims, gtype, _), off in zip(self.tensors, offs):
            out += self._str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
            out += struct.pack("<IQ", gtype, off)
        start = (len(out) + self.alignment - 1) // self.alignment * self.alignment
        out += b"\0" * (start - len(out))
        for (_, _, _, data), off in zip(self.tensors, offs):
            out += b"\0" * (start + off - len(out))
            out += data
        return bytes(out)


def gguf_from_nrm(blob, file_type=None, alignment=32, drop=(), extra_kv=(), extra_tensors=(), retype=None,
                  name="Test Model"):
    """The GGUF a model's `.nrm` came from: metadata keys and tensor names the
    converter reads. `drop` removes metadata keys or tensor names, `retype`
    maps a tensor name to (ggml type, bytes)."""
    h, table = nrm_fields(blob)
    b = bytes(blob)
    arch = ARCH_NAMES[h["arch"]]
    dim, n_layers, n_heads, n_kv, head_dim, ffn, vocab, ctx = h["dims"]
    theta, eps, factor = h["floats"][:3]
    w = GgufWriter(alignment=alignment)
    kv = [("general.architecture", STR, arch), ("general.name", STR, name),
          (f"{arch}.embedding_length", U32, dim), (f"{arch}.block_count", U32, n_layers),
          (f"{arch}.attention.head_count", U32, n_heads), (f"{arch}.attention.head_count_kv", U32, n_kv),
          (f"{arch}.feed_forward_length", U32, ffn), (f"{arch}.context_length", U32, ctx),
          (f"{arch}.rope.freq_base", F32, theta), (f"{arch}.attention.layer_norm_rms_epsilon", F32, eps),
          ("tokenizer.ggml.tokens", ARR, (STR, [f"t{i}" for i in range(vocab)]))]
    if alignment != 32:
        kv.append(("general.alignment", U32, alignment))
    if file_type is not None:
        kv.append(("general.file_type", U32, file_type))
    if head_dim != dim // n_heads:
        kv.append((f"{arch}.attention.key_length", U32, head_dim))
    if factor != 0.0:
        kv.append(("llama.rope.scaling.factor", F32, factor))
    if arch == "granite":
        es, at, rs, ls = h["mup"]
        kv += [(f"{arch}.embedding_scale", F32, es), (f"{arch}.attention.scale", F32, at),
               (f"{arch}.residual_scale", F32, rs), (f"{arch}.logit_scale", F32, ls)]
    for key, vtype, value in kv:
        if key not in drop:
            w.add(key, vtype, value)
    for key, vtype, value in extra_kv:
        w.add(key, vtype, value)
    for kind, layer, dtype, off, size, rows, cols in table:
        tname = tensor_name(kind, layer)
        if tname in drop:
            continue
        data = b[h["data_off"] + off:h["data_off"] + off + size]
        gtype = GGML_OF_DTYPE[dtype]
        if retype and tname in retype:
            gtype, data = retype[tname]
        w.tensor(tname, [cols] if rows == 1 else [cols, rows], gtype, data)
    for t in extra_tensors:
        w.tensor(*t)
    return w.bytes()


def as_array(data):
    return np.frombuffer(bytes(data), np.uint8).copy()
