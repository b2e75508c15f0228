"""nr-tensor entry points over CUDA tensors (crates/nr-tensor/src).

Same names, argument order and meaning as the reference's Rust functions;
block arrays are uint8 CUDA tensors holding the reference's in-place block
bytes, f32 vectors are float32 CUDA tensors. Shape violations that the
reference asserts raise NrcError (code INVALID). Calls are asynchronous on
the current torch stream (or `stream=`).
"""
import ctypes as C

import torch

from ._lib import check, lib

Q8_0_BYTES, Q4K_BYTES, Q6K_BYTES, Q8K_BYTES = 34, 144, 210, 292
QK8_0, QK_K = 32, 256


def _ptr(t):
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("nrcuda kernels take CUDA tensors")
    return C.c_void_p(t.data_ptr())


def _stream(stream):
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


def quantize(x, out, stream=None):
    """q8::quantize (q8.rs:27-44): f32[n] -> Q8_0 blocks [n/32]."""
    check(lib().nrc_quantize_q8_0(_ptr(x), _ptr(out), x.numel(), _stream(stream)))


def dequantize(blocks, out, stream=None):
    """q8::dequantize (q8.rs:47-55)."""
    check(lib().nrc_dequantize_q8_0(_ptr(blocks), _ptr(out), out.numel(), _stream(stream)))


def quantize_q8k(x, out, stream=None):
    """kquant::quantize_q8k (kquant.rs:157-187)."""
    check(lib().nrc_quantize_q8k(_ptr(x), _ptr(out), x.numel(), _stream(stream)))


def dequant_q4k(blocks, out, stream=None):
    """kquant::dequant_q4k over every block (kquant.rs:95-118)."""
    check(lib().nrc_dequant_q4k(_ptr(blocks), _ptr(out), out.numel() // QK_K, _stream(stream)))


def dequant_q6k(blocks, out, stream=None):
    """kquant::dequant_q6k over every block (kquant.rs:121-142)."""
    check(lib().nrc_dequant_q6k(_ptr(blocks), _ptr(out), out.numel() // QK_K, _stream(stream)))


def matvec_q8(y, w, x, rows, cols, stream=None):
    """kernels::matvec_q8 (kernels.rs:36-47)."""
    check(lib().nrc_matvec_q8_0(_ptr(y), _ptr(w), _ptr(x), rows, cols, _stream(stream)))


def matmul_q8(y, w, xs, rows, cols, batch, stream=None):
    """kernels::matmul_q8 (kernels.rs:91-143); y is [batch][rows]."""
    check(lib().nrc_matmul_q8_0(_ptr(y), _ptr(w), _ptr(xs), rows, cols, batch, _stream(stream)))


def matmul_q8_noalloc(y, w, xs, rows, cols, batch, stream=None):
    """matmul_q8 through the entry point that allocates nothing (static device
    scratch, cols <= 16384, synchronous); same results as matmul_q8."""
    check(lib().nrc_matmul_q8_0_noalloc(_ptr(y), _ptr(w), _ptr(xs), rows, cols, batch, _stream(stream)))


def matvec_q4k(y, w, x, rows, cols, stream=None):
    """kquant::matvec_q4k (kquant.rs:563)."""
    check(lib().nrc_matvec_q4k(_ptr(y), _ptr(w), _ptr(x), rows, cols, _stream(stream)))


def matvec_q6k(y, w, x, rows, cols, stream=None):
    """kquant::matvec_q6k (kquant.rs:564)."""
    check(lib().nrc_matvec_q6k(_ptr(y), _ptr(w), _ptr(x), rows, cols, _stream(stream)))


def matmul_q4k(y, w, xs, rows, cols, batch, stream=None):
    """kquant::matmul_q4k (kquant.rs:626-632)."""
    check(lib().nrc_matmul_q4k(_ptr(y), _ptr(w), _ptr(xs), rows, cols, batch, _stream(stream)))


def matmul_q6k(y, w, xs, rows, cols, batch, stream=None):
    """kquant::matmul_q6k (kquant.rs:633-639)."""
    check(lib().nrc_matmul_q6k(_ptr(y), _ptr(w), _ptr(xs), rows, cols, batch, _stream(stream)))


def f32_to_f16(x, out, stream=None):
    """f16::f32_to_f16 elementwise (f16.rs:25-56); out is int16/uint16 storage."""
    check(lib().nrc_f32_to_f16(_ptr(x), _ptr(out), x.numel(), _stream(stream)))


def f16_to_f32(x, out, stream=None):
    """f16::f16_to_f32 elementwise (f16.rs:3-23)."""
    check(lib().nrc_f16_to_f32(_ptr(x), _ptr(out), x.numel(), _stream(stream)))


def rmsnorm(out, x, weight, eps, rows=1, stream=None):
    """vec::rmsnorm (vec.rs:4-14) over `rows` rows."""
    check(lib().nrc_rmsnorm(_ptr(out), _ptr(x), _ptr(weight), weight.numel(), rows, eps, _stream(stream)))


def softmax(x, rows=1, stream=None):
    """vec::softmax (vec.rs:30-41), in place over `rows` rows."""
    check(lib().nrc_softmax(_ptr(x), x.numel() // rows, rows, _stream(stream)))


def swiglu(gate, up, stream=None):
    """vec::swiglu (vec.rs:44-50), in place on gate."""
    check(lib().nrc_swiglu(_ptr(gate), _ptr(up), gate.numel(), _stream(stream)))


def expf(x, out, stream=None):
    """The expf of vec.rs:34,47 / sample.rs:70, correctly rounded, elementwise."""
    check(lib().nrc_expf(_ptr(x), _ptr(out), x.numel(), _stream(stream)))


def expf_hash(out, chunk0, nchunks, stream=None):
    """Per-chunk hashes of expf over every binary32 input (2^20 inputs per chunk)."""
    check(lib().nrc_expf_hash(_ptr(out), chunk0, nchunks, _stream(stream)))


class Sampler:
    """nr_model::Sampler (crates/nr-model/src/sample.rs:5-96) drawing on the
    device: `sample(logits)` takes a float32 CUDA tensor and returns the token id.
    The xorshift64 state lives in device memory (seed | 1 at construction)."""

    def __init__(self, temperature, top_p, seed, device="cuda"):
        self.temperature = float(temperature)
        self.top_p = float(top_p)
        self.rng = torch.tensor([(seed | 1) & 0xFFFFFFFFFFFFFFFF], dtype=torch.uint64, device=device)
        self._out = torch.zeros(1, dtype=torch.int32, device=device)

    def sample(self, logits, stream=None):
        check(lib().nrc_sample(_ptr(logits), logits.numel(), self.temperature, self.top_p, _ptr(self.rng),
                               _ptr(self._out), _stream(stream)))
        return int(self._out.item())

    def state(self):
        return int(self.rng.cpu().item())


def argmax(x, stream=None):
    """vec::argmax (vec.rs:80-90): index of the first maximum (host int)."""
    out = torch.zeros(1, dtype=torch.int32, device=x.device)
    check(lib().nrc_argmax(_ptr(x), x.numel(), _ptr(out), _stream(stream)))
    return int(out.item())


def rope_freqs(head_dim, theta, scaling=None):
    """rope::rope_freqs (rope.rs:14-34); scaling = (factor, low, high, original_context)."""
    out = (C.c_float * (head_dim // 2))()
    f, lo, hi, orig = scaling if scaling else (0.0, 0.0, 0.0, 0.0)
    check(lib().nrc_rope_freqs(out, head_dim, theta, f, lo, hi, orig))
    return list(out)


def rope_apply(x, head_dim, freqs, pos, style, stream=None):
    """rope::apply (rope.rs:49-65); style 0 = Adjacent, 1 = Neox."""
    arr = (C.c_float * len(freqs))(*freqs)
    check(lib().nrc_rope_apply(_ptr(x), x.numel(), head_dim, arr, pos, style, _stream(stream)))


def sync_check(stream=None):
    """Synchronize and raise if a kernel recorded a device-side error."""
    check(lib().nrc_sync_check(_stream(stream)))
