"""GGUF ingestion (nrc_gguf_to_nrm, tools/nrconvert/src/{gguf,main}.rs) on the
CPU: a seeded synthetic model written as the GGUF it would come from converts
back to the same tensor table and data bytes, with the header fields the
converter sets, and every condition the converter panics or exits on is a
status code. The GPU test loads a converted model and checks its logits
against the original's."""
import os
import struct

import numpy as np
import pytest

from nightrun_b200.configs import CONFIGS, MODEL_SEED
from tests.ggufdata import F64, I32, STR, U32, U64, as_array, gguf_from_nrm, nrm_fields

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

FAMILIES = ["tiny_llama_q8", "tiny_llama_q4km", "tiny_qwen3", "tiny_granite"]


@pytest.fixture(scope="module")
def NB():
    from nightrun_b200 import _lib
    if not os.path.exists(_lib.LIB_PATH):
        from nightrun_b200 import build
        build.build()
    import nightrun_b200
    return nightrun_b200


@pytest.fixture(scope="module")
def blobs(orc):
    return {name: orc.synth_nrm(CONFIGS[name], MODEL_SEED) for name in FAMILIES}


def convert(NB, data):
    return NB.gguf_to_nrm(as_array(data))


def status(NB, data):
    with pytest.raises(NB.NrcError) as e:
        convert(NB, data)
    return e.value.code


@pytest.mark.parametrize("name", FAMILIES)
@pytest.mark.parametrize("alignment", [32, 64])
def test_gguf_converts_back_to_the_model(NB, orc, blobs, name, alignment):
    src = blobs[name]
    file_type = 7 if CONFIGS[name]["quant"] == 0 else 15
    out = convert(NB, gguf_from_nrm(src, file_type=file_type, alignment=alignment, name="Tiny"))
    h0, t0 = nrm_fields(src)
    h1, t1 = nrm_fields(out)
    # main.rs:231-277 order, 64-byte offsets: the same table and data section.
    assert t1 == t0
    assert h1["count"] == h0["count"] and h1["data_size"] == h0["data_size"]
    d0 = src[h0["data_off"]:h0["data_off"] + h0["data_size"]]
    d1 = out[h1["data_off"]:h1["data_off"] + h1["data_size"]]
    assert d1.tobytes() == d0.tobytes()
    assert h1["data_crc"] == h0["data_crc"] == orc.crc32(d0)
    # Header fields (main.rs:374-399): dims, rope theta / eps / factor, tied flag, muP scalars;
    # the Llama-3 low/high/original-context fields are written as zero by the converter.
    assert h1["arch"] == h0["arch"] and h1["dims"] == h0["dims"]
    assert h1["floats"][:3] == h0["floats"][:3] and h1["floats"][3:] == (0.0, 0.0, 0.0)
    assert h1["flags"] == h0["flags"]
    if h0["arch"] == 3:
        assert h1["mup"] == h0["mup"]
    else:
        assert h1["mup"] == (1.0, 0.0, 1.0, 1.0)
    assert h1["name"] == ("Tiny Q8_0" if file_type == 7 else "Tiny Q4_K_M")
    assert h1["tok_off"] == 192 and h1["tok_len"] == 0 and h1["table_off"] == 192
    assert h1["data_off"] == (192 + 32 * h1["count"] + 63) // 64 * 64
    # Metadata CRC: header with both CRC fields zeroed + tokenizer + table (main.rs:401-408).
    meta = bytearray(out[:192].tobytes())
    meta[184:192] = b"\0" * 8
    assert h1["meta_crc"] == orc.crc32(np.frombuffer(bytes(meta) + out[192:192 + 32 * h1["count"]].tobytes(),
                                                     np.uint8))


def test_gguf_labels_and_defaults(NB, blobs):
    src = blobs["tiny_granite"]
    for ft, label in ((14, "Q4_K_S"), (17, "Q5_K_M"), (18, "Q6_K"), (2, "quantized"), (None, "quantized")):
        h, _ = nrm_fields(convert(NB, gguf_from_nrm(src, file_type=ft, name="G")))
        assert h["name"] == f"G {label}"
    # No general.name: "Unknown Model"; names past 48 bytes are cut.
    h, _ = nrm_fields(convert(NB, gguf_from_nrm(src, file_type=15, drop=("general.name",))))
    assert h["name"] == "Unknown Model Q4_K_M"
    h, _ = nrm_fields(convert(NB, gguf_from_nrm(src, file_type=15, name="x" * 60)))
    assert h["name"] == "x" * 48


def test_gguf_rejections(NB, blobs):
    from nightrun_b200 import _lib
    E = {k: getattr(_lib, k) for k in dir(_lib) if k.startswith("NRC_ERR_")}
    src = blobs["tiny_qwen3"]
    good = gguf_from_nrm(src, file_type=15)
    assert status(NB, b"GGUX" + good[4:]) == E["NRC_ERR_BAD_MAGIC"]
    for v in (1, 4):
        assert status(NB, good[:4] + struct.pack("<I", v) + good[8:]) == E["NRC_ERR_BAD_VERSION"]
    for cut in (0, 3, 10, 30, len(good) // 3, len(good) - 1):
        assert status(NB, good[:cut]) == E["NRC_ERR_TOO_SHORT"]
    # arch_verdict (main.rs:63-110)
    for arch in ("mamba", "granitehybrid", "granitemoehybrid"):
        bad = gguf_from_nrm(src, drop=("general.architecture",), extra_kv=[("general.architecture", STR, arch)])
        assert status(NB, bad) == E["NRC_ERR_UNSUPPORTED"], arch
    for key in ("ssm_conv_kernel", "ssm_state_size", "expert_count", "expert_used_count"):
        assert status(NB, gguf_from_nrm(src, extra_kv=[(f"qwen3.{key}", U32, 4)])) == E["NRC_ERR_UNSUPPORTED"], key
    # A zero-valued feature key is accepted.
    convert(NB, gguf_from_nrm(src, extra_kv=[("qwen3.expert_count", U32, 0)]))
    moe = ("blk.0.ffn_gate_exps.weight", [32], 0, b"\0" * 128)
    assert status(NB, gguf_from_nrm(src, extra_tensors=[moe])) == E["NRC_ERR_UNSUPPORTED"]
    ssm = ("blk.1.ssm_a.weight", [32], 0, b"\0" * 128)
    assert status(NB, gguf_from_nrm(src, extra_tensors=[ssm])) == E["NRC_ERR_UNSUPPORTED"]
    # Missing keys and tensors (the converter panics "missing ..." / "gguf missing tensor").
    for key in ("qwen3.block_count", "qwen3.rope.freq_base", "tokenizer.ggml.tokens"):
        assert status(NB, gguf_from_nrm(src, drop=(key,))) == E["NRC_ERR_MISSING"], key
    for t in ("token_embd.weight", "blk.1.ffn_up.weight", "blk.0.attn_q_norm.weight", "output_norm.weight"):
        assert status(NB, gguf_from_nrm(src, drop=(t,))) == E["NRC_ERR_MISSING"], t
    gsrc = blobs["tiny_granite"]
    assert status(NB, gguf_from_nrm(gsrc, drop=("granite.logit_scale",))) == E["NRC_ERR_MISSING"]
    # Tensor types: F16 / Q5_K are sized but not converted; an unknown type is rejected while parsing.
    n = CONFIGS["tiny_qwen3"]["dim"]
    f16 = {"blk.0.attn_norm.weight": (1, b"\0" * (2 * n))}
    assert status(NB, gguf_from_nrm(src, retype=f16)) == E["NRC_ERR_UNSUPPORTED"]
    unk = {"blk.0.attn_norm.weight": (99, b"\0" * (4 * n))}
    assert status(NB, gguf_from_nrm(src, retype=unk)) == E["NRC_ERR_UNSUPPORTED"]
    # A tensor whose data would lie past the end of the file.
    assert status(NB, good[:-64]) == E["NRC_ERR_TOO_SHORT"]


def test_gguf_optional_tensors_and_ints(NB, blobs):
    # Tied output (no output.weight) sets the tied flag; u64 / i32 metadata read as u32 (gguf.rs:24-33).
    src = blobs["tiny_qwen3"]
    h0, _ = nrm_fields(src)
    h, _ = nrm_fields(convert(NB, gguf_from_nrm(src)))
    assert h["flags"] == h0["flags"] == 1
    alt = gguf_from_nrm(src, drop=("qwen3.block_count", "qwen3.feed_forward_length"),
                        extra_kv=[("qwen3.block_count", U64, h0["dims"][1]), ("qwen3.feed_forward_length", I32,
                                                                               h0["dims"][5])])
    assert nrm_fields(convert(NB, alt))[0]["dims"] == h0["dims"]
    neg = gguf_from_nrm(src, drop=("qwen3.block_count",), extra_kv=[("qwen3.block_count", I32, -2)])
    from nightrun_b200 import _lib
    assert status(NB, neg) == _lib.NRC_ERR_MISSING
    # An f64 epsilon is read through as_f32.
    f64 = gguf_from_nrm(src, drop=("qwen3.attention.layer_norm_rms_epsilon",),
                        extra_kv=[("qwen3.attention.layer_norm_rms_epsilon", F64, float(h0["floats"][1]))])
    assert nrm_fields(convert(NB, f64))[0]["floats"][1] == h0["floats"][1]


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["tiny_llama_q4km", "tiny_qwen3", "tiny_granite"])
def test_gguf_model_runs_like_the_original(NB, blobs, name):
    """A converted model's logits equal the original model's bit for bit
    (models whose RoPE needs no Llama-3 header fields the converter zeroes)."""
    from nightrun_b200.configs import prompt_ids
    src = blobs[name]
    a = NB.Model.load(src)
    b = NB.Model.load_gguf(as_array(gguf_from_nrm(src, file_type=15)))
    assert a.data_crc() == b.data_crc()
    ids = prompt_ids(12, CONFIGS[name]["vocab"])
    ca, cb = a.ctx(32), b.ctx(32)
    assert ca.prefill(ids).tobytes() == cb.prefill(ids).tobytes()
    for t in (3, 5):
        assert ca.forward(t).tobytes() == cb.forward(t).tobytes()
