"""Test-data generators restated from the reference's tests.

`Rng` is the xorshift generator of crates/nr-tensor/tests/kernels.rs:9-29 and
crates/nr-tensor/tests/kquant.rs:7-39 (f32 arithmetic reproduced with numpy
float32 so the values are bit-identical). `tiny_nrm` restates
crates/nr-model/tests/format_malformed.rs:9-70 and `reseal` :74-95.
"""
import struct

import numpy as np

M64 = 0xFFFFFFFFFFFFFFFF
F = np.float32


class Rng:
    def __init__(self, seed):
        self.s = seed & M64

    def next(self):
        x = self.s
        x ^= (x << 13) & M64
        x ^= x >> 7
        x ^= (x << 17) & M64
        self.s = x
        return x

    def f32(self):
        # (next >> 40) as f32 / (1 << 23) as f32 * 2.0 - 1.0, in f32
        return F(F(F(self.next() >> 40) / F(1 << 23)) * F(2.0)) - F(1.0)

    def vec(self, n):
        return np.array([self.f32() for _ in range(n)], np.float32)

    def adversarial(self, n):
        out = []
        for i in range(n):
            m = self.next() % 7
            if m == 0:
                out.append(F(0.0))
            elif m == 1:
                out.append(F(100.0) * self.f32())
            elif m == 2:
                out.append(F(1e-4) * self.f32())
            elif m == 3:
                out.append(F(-50.0) + self.f32())
            else:
                out.append(self.f32() * F(1 + i % 13))
        return np.array(out, np.float32)


HEADER_SIZE, ENTRY_SIZE, DATA_ALIGN = 192, 32, 64


def crc32(data):
    import zlib
    return zlib.crc32(bytes(data)) & 0xFFFFFFFF


def tiny_nrm():
    """Smallest valid v3 .nrm: 16-byte tokenizer blob, one 8x8 F32 tensor."""
    tok_blob = bytes([0xEE] * 16)
    tok_off = HEADER_SIZE
    tok_size = len(tok_blob)
    table_off = tok_off + tok_size
    table_len = ENTRY_SIZE
    data_off = (table_off + table_len + DATA_ALIGN - 1) // DATA_ALIGN * DATA_ALIGN
    rows = cols = 8
    tsize = rows * cols * 4
    b = bytearray(data_off + tsize)
    b[0:4] = b"NRUN"
    b[4:8] = struct.pack("<I", 3)
    b[8:12] = struct.pack("<I", 1)
    for i, v in enumerate([8, 1, 1, 1, 8, 8, 16, 128]):
        b[12 + 4 * i:16 + 4 * i] = struct.pack("<I", v)
    b[72:76] = struct.pack("<f", 1.0)
    b[76:80] = struct.pack("<f", 0.0)
    b[80:84] = struct.pack("<f", 1.0)
    b[84:88] = struct.pack("<f", 1.0)
    b[88:92] = b"test"
    b[136:144] = struct.pack("<Q", tok_off)
    b[144:152] = struct.pack("<Q", tok_size)
    b[152:160] = struct.pack("<Q", table_off)
    b[160:164] = struct.pack("<I", 1)
    b[168:176] = struct.pack("<Q", data_off)
    b[176:184] = struct.pack("<Q", tsize)
    b[tok_off:tok_off + tok_size] = tok_blob
    t = table_off
    b[t:t + 2] = struct.pack("<H", 1)
    b[t + 4:t + 6] = struct.pack("<H", 0)
    b[t + 8:t + 16] = struct.pack("<Q", 0)
    b[t + 16:t + 24] = struct.pack("<Q", tsize)
    b[t + 24:t + 28] = struct.pack("<I", rows)
    b[t + 28:t + 32] = struct.pack("<I", cols)
    b[184:188] = struct.pack("<I", crc32(b[data_off:data_off + tsize]))
    meta = crc32(bytes(b[:HEADER_SIZE - 8]) + bytes(8) + bytes(b[tok_off:tok_off + tok_size]) +
                 bytes(b[table_off:table_off + table_len]))
    b[188:192] = struct.pack("<I", meta)
    return b


def reseal(b):
    tok_off = struct.unpack("<Q", b[136:144])[0]
    tok_size = struct.unpack("<Q", b[144:152])[0]
    table_off = struct.unpack("<Q", b[152:160])[0]
    count = struct.unpack("<I", b[160:164])[0]
    n = len(b)
    t0 = min(tok_off, n)
    t1 = min(min(tok_off + tok_size, M64), n)
    e0 = min(table_off, n)
    e1 = min(min(table_off + count * ENTRY_SIZE, M64), n)
    meta = crc32(bytes(b[:HEADER_SIZE - 8]) + bytes(8) + bytes(b[t0:max(t1, t0)]) + bytes(b[e0:max(e1, e0)]))
    b[188:192] = struct.pack("<I", meta)


def malformed_cases():
    """(name, blob, expect_meta_crc) for every case of format_malformed.rs:110-206."""
    out = []
    base = tiny_nrm()
    for cut in [0, 3, 4, 100, HEADER_SIZE - 1, HEADER_SIZE, len(base) - 1]:
        out.append((f"truncated to {cut}", bytes(base[:cut]), False))
    b = tiny_nrm(); b[0] = ord("X"); out.append(("magic", bytes(b), False))
    b = tiny_nrm(); b[4:8] = struct.pack("<I", 99); out.append(("version", bytes(b), False))
    b = tiny_nrm(); b[136:144] = struct.pack("<Q", M64 - 4); reseal(b); out.append(("wrapping tok_off", bytes(b), False))
    b = tiny_nrm(); b[168:176] = struct.pack("<Q", M64 - 4); reseal(b); out.append(("wrapping data_off", bytes(b), False))
    b = tiny_nrm(); b[152:160] = struct.pack("<Q", M64 - 31); b[160:164] = struct.pack("<I", 0xFFFFFFFF); reseal(b)
    out.append(("wrapping table", bytes(b), False))
    tab = struct.unpack("<Q", base[152:160])[0]
    b = tiny_nrm(); b[tab + 8:tab + 16] = struct.pack("<Q", M64 - 63); reseal(b); out.append(("entry wrap", bytes(b), False))
    b = tiny_nrm(); b[tab + 8:tab + 16] = struct.pack("<Q", 4); reseal(b); out.append(("misaligned offset", bytes(b), False))
    b = tiny_nrm(); b[tab + 24:tab + 28] = struct.pack("<I", 0xFFFFFFFF); b[tab + 28:tab + 32] = struct.pack("<I", 0xFFFFFFFF)
    reseal(b); out.append(("rows*cols overflow", bytes(b), False))
    b = tiny_nrm(); b[tab + 16:tab + 24] = struct.pack("<Q", 8); reseal(b); out.append(("size/dtype mismatch", bytes(b), False))
    b = tiny_nrm(); b[100] ^= 0x40; out.append(("meta crc flip", bytes(b), True))
    b = tiny_nrm(); b[80:84] = struct.pack("<f", float("nan")); reseal(b); out.append(("NaN residual scale", bytes(b), False))
    return out
