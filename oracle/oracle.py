"""ctypes/numpy front end of the CPU oracle (oracle/oracle.c).

TEST INFRASTRUCTURE ONLY.  tests/, __graft_entry__.smoke() and bench.py's CPU-baseline and
reference arms import this module as the checker; the product package (decisive_b200) never
imports it.  Each wrapper names the reference function (decisive, src/models/pplx_flash/...)
that the C code restates.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
GROUP = 64


def build(force: bool = False) -> str:
    src = os.path.join(HERE, "oracle.c")
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-C", HERE, "-s"], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = C.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


_f = C.POINTER(C.c_float)
_u8 = C.POINTER(C.c_uint8)
_i8 = C.POINTER(C.c_int8)
_u16 = C.POINTER(C.c_uint16)
_i32 = C.POINTER(C.c_int32)
_sz = C.c_size_t


def _declare(l):
    l.oracle_f32_to_bf16.restype = C.c_uint16
    l.oracle_f32_to_bf16.argtypes = [C.c_float]
    l.oracle_f32_to_bf16_array.argtypes = [_f, _sz, _u16]
    l.oracle_group_scale.restype = C.c_float
    l.oracle_group_scale.argtypes = [_f, _sz, C.c_int]
    l.oracle_pack_codes.argtypes = [_f, _sz, C.c_float, C.c_int, _i8]
    l.oracle_packed_size.restype = _sz
    l.oracle_packed_size.argtypes = [_sz, _sz, C.c_int]
    l.oracle_packed_pack.restype = C.c_int
    l.oracle_packed_pack.argtypes = [_u16, _sz, _sz, C.c_int, _u8]
    l.oracle_packed_unpack.restype = C.c_int
    l.oracle_packed_unpack.argtypes = [_u8, _sz, C.c_int, _f]
    l.oracle_packed_project.restype = C.c_int
    l.oracle_packed_project.argtypes = [_u8, _sz, C.c_int, _sz, _f, _sz, _f]
    l.oracle_matrix_data_bytes.restype = _sz
    l.oracle_matrix_data_bytes.argtypes = [_sz, _sz, C.c_int]
    l.oracle_matrix_scale_count.restype = _sz
    l.oracle_matrix_scale_count.argtypes = [_sz, _sz]
    l.oracle_matrix_from_bf16.restype = C.c_int
    l.oracle_matrix_from_bf16.argtypes = [_u16, _sz, _sz, C.c_int, C.c_int, C.c_int, _i8, _f, _f]
    l.oracle_matrix_prepare.argtypes = [_f, _sz, _sz, C.c_int, _i8, _f, _i32]
    l.oracle_matrix_apply_prepared.argtypes = [_i8, _f, _f, _sz, _sz, C.c_int, _i8, _f, _i32, _sz, C.c_int, _f]
    l.oracle_matrix_apply.argtypes = [_i8, _f, _f, _sz, _sz, C.c_int, C.c_int, _f, _sz, C.c_int, _f]
    l.oracle_fit_mse.restype = C.c_float
    l.oracle_fit_mse.argtypes = [_f, _sz, C.c_int, _i8]
    l.oracle_fit_affine.argtypes = [_f, _sz, C.c_int, _i8, _f, _f]
    l.oracle_fit_nf4.restype = C.c_float
    l.oracle_fit_nf4.argtypes = [_f, _sz, _i8]
    l.oracle_embedding_from_bf16.restype = C.c_int
    l.oracle_embedding_from_bf16.argtypes = [_u16, _sz, _sz, C.c_int, C.c_int, C.c_int, _u8, _f, _f]
    l.oracle_embedding_append.argtypes = [_u8, _f, _f, _sz, C.c_int, C.c_int, _sz, _f]
    l.oracle_rms.argtypes = [_f, _f, _sz, _sz, _f, C.c_float, C.c_int]
    l.oracle_silu_mul.argtypes = [_f, _f, _sz]
    l.oracle_softmax.argtypes = [_f, _sz]
    l.oracle_rope.argtypes = [_f, _sz, _sz, _sz, _sz, _sz, C.c_float]
    l.oracle_attention.argtypes = [_f, _f, _f, _sz, _sz, _sz, _sz, C.c_float, _f]
    l.oracle_attention_masked.argtypes = [_f, _f, _f, _sz, _sz, _sz, _sz, C.c_float, C.c_int, _f]
    l.oracle_encoder_create.restype = C.c_void_p
    l.oracle_encoder_create.argtypes = [C.c_void_p, C.c_void_p]
    l.oracle_encoder_destroy.argtypes = [C.c_void_p]
    l.oracle_encoder_forward.restype = C.c_int
    l.oracle_encoder_forward.argtypes = [C.c_void_p, _i32, _sz, C.c_int, C.c_int, _f, _f]
    l.oracle_decima_scale.restype = C.c_float
    l.oracle_decima_scale.argtypes = [_f, _sz]
    l.oracle_decima_quantize.restype = C.c_int8
    l.oracle_decima_quantize.argtypes = [C.c_float, C.c_float]
    l.oracle_decima_quantize_rows.argtypes = [_f, _sz, _sz, _sz, _i8, _f]
    l.oracle_decima_apply_w8a8.argtypes = [_i8, _f, _sz, _sz, _sz, _f, _sz, _f, C.c_int, _f]
    l.oracle_decima_apply_w8a32.argtypes = [_i8, _f, _sz, _sz, _sz, _f, _sz, _f, C.c_int, _f]
    l.oracle_layer_norm.argtypes = [_f, _sz, _sz, _f, _f, C.c_float]
    l.oracle_gelu.argtypes = [_f, _sz]
    l.oracle_num_threads.restype = C.c_int
    l.oracle_set_threads.argtypes = [C.c_int]
    l.oracle_has_avx2.restype = C.c_int


def _p(a, t):
    return a.ctypes.data_as(t) if a is not None else None


# ------------------------------------------------------------------ bf16
def f32_to_bf16(x) -> np.ndarray:
    """half 2.7.1 bf16::from_f32 (RNE), as used by every reference test to make weights."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().oracle_f32_to_bf16_array(_p(x, _f), x.size, _p(out, _u16))
    return out


def bf16_to_f32(b) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def bf16_truncate(x) -> np.ndarray:
    """The bytes of `(v.to_bits() >> 16) as u16` used by packed.rs tests (truncation)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    return (x.view(np.uint32) >> 16).astype(np.uint16)


# ------------------------------------------------------------------ primitives
def group_scale(x, bits: int) -> np.float32:
    x = np.ascontiguousarray(x, dtype=np.float32)
    return np.float32(lib().oracle_group_scale(_p(x, _f), x.size, bits))


def pack_codes(x, scale, bits: int) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros(x.size, dtype=np.int8)
    lib().oracle_pack_codes(_p(x, _f), x.size, float(np.float32(scale)), bits, _p(out, _i8))
    return out


# ------------------------------------------------------------------ packed rows
def packed_size(rows, columns, bits) -> int:
    return int(lib().oracle_packed_size(rows, columns, bits))


def packed_pack(bf16: np.ndarray, rows: int, columns: int, bits: int) -> np.ndarray:
    bf16 = np.ascontiguousarray(bf16, dtype=np.uint16)
    n = packed_size(rows, columns, bits)
    if not n:
        raise ValueError("invalid group-64 matrix shape")
    out = np.zeros(n, dtype=np.uint8)
    rc = lib().oracle_packed_pack(_p(bf16, _u16), rows, columns, bits, _p(out, _u8))
    if rc:
        raise ValueError("nonfinite packed weight" if rc == -2 else "invalid shape")
    return out


def packed_unpack(packed: np.ndarray, bits: int) -> np.ndarray:
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    stride = packed_size(1, GROUP, bits)
    if not stride or packed.size == 0 or packed.size % stride:
        raise ValueError("invalid packed rows")
    out = np.zeros(packed.size // stride * GROUP, dtype=np.float32)
    if lib().oracle_packed_unpack(_p(packed, _u8), packed.size, bits, _p(out, _f)):
        raise ValueError("invalid packed scale")
    return out


def packed_project(packed, bits, columns, x, outputs) -> np.ndarray:
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros(outputs, dtype=np.float32)
    rc = lib().oracle_packed_project(_p(packed, _u8), packed.size, bits, columns, _p(x, _f), outputs, _p(y, _f))
    if rc:
        raise ValueError("nonfinite readout activation" if rc == -2 else "invalid packed readout shape")
    return y


# ------------------------------------------------------------------ int8::Matrix
class Matrix:
    """int8::Matrix (int8.rs:13-289): panel-layout codes + f32 scales (+ affine offsets)."""

    def __init__(self, bf16, input_, output, weight_bits=8, activation_bits=8, fit=0, simd=1):
        bf16 = np.ascontiguousarray(bf16, dtype=np.uint16)
        if input_ <= 0 or output <= 0 or bf16.size != input_ * output:
            raise ValueError("invalid INT8 matrix shape")
        self.input, self.output = input_, output
        self.weight_bits, self.activation_bits = weight_bits, activation_bits
        l = lib()
        self.data = np.zeros(l.oracle_matrix_data_bytes(input_, output, weight_bits), dtype=np.int8)
        self.scales = np.zeros(l.oracle_matrix_scale_count(input_, output), dtype=np.float32)
        self.offsets = np.zeros_like(self.scales) if fit == 2 else None
        rc = l.oracle_matrix_from_bf16(_p(bf16, _u16), input_, output, weight_bits, fit, simd,
                                       _p(self.data, _i8), _p(self.scales, _f), _p(self.offsets, _f))
        if rc:
            raise ValueError("non-finite INT8 weight" if rc == -2 else "unsupported quantization")

    @property
    def groups(self):
        return (self.input + GROUP - 1) // GROUP

    def bytes(self) -> int:
        """int8.rs:162-164"""
        return self.data.size + (self.scales.size + (0 if self.offsets is None else self.offsets.size)) * 4

    def code(self, index: int) -> int:
        """int8.rs:154-160"""
        if self.weight_bits == 4:
            return int((int(self.data[index // 2]) & 0xFF) >> (index % 2 * 4) & 15) - 8
        return int(self.data[index])

    def weight_codes(self) -> np.ndarray:
        """Dense [output, groups*64] int8 codes decoded from the panel layout (int8.rs:121-132)."""
        G = self.groups
        c = np.arange(self.output)[:, None, None]
        g = np.arange(G)[None, :, None]
        k = np.arange(GROUP)[None, None, :]
        index = (c // 8 * G + g) * GROUP * 8 + k // 4 * 32 + c % 8 * 4 + k % 4
        if self.weight_bits == 4:
            raw = self.data.view(np.uint8)[index // 2]
            codes = ((raw >> (index % 2 * 4)) & 15).astype(np.int16) - 8
        else:
            codes = self.data[index].astype(np.int16)
        return codes.reshape(self.output, G * GROUP).astype(np.int8)

    def weight_scales(self) -> np.ndarray:
        """[output, groups] scales from the panel layout."""
        G = self.groups
        c = np.arange(self.output)[:, None]
        g = np.arange(G)[None, :]
        return self.scales[(c // 8 * G + g) * 8 + c % 8]

    def weight_offsets(self):
        if self.offsets is None:
            return None
        G = self.groups
        c = np.arange(self.output)[:, None]
        g = np.arange(G)[None, :]
        return self.offsets[(c // 8 * G + g) * 8 + c % 8]

    def prepare(self, x):
        """int8.rs:178-202 -> (values [T, G*64] i8, scales [T, G] f32, sums [T, G] i32)"""
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
        tokens = x.size // self.input
        values = np.zeros(tokens * self.groups * GROUP, dtype=np.int8)
        scales = np.zeros(tokens * self.groups, dtype=np.float32)
        sums = np.zeros(tokens * self.groups, dtype=np.int32)
        lib().oracle_matrix_prepare(_p(x, _f), tokens, self.input, self.activation_bits,
                                    _p(values, _i8), _p(scales, _f), _p(sums, _i32))
        return values, scales, sums

    def apply(self, x, mode: int = 0) -> np.ndarray:
        """int8.rs:166-176; mode 0 AVX2 numerics (fma), 1 portable (mul+add), 2 AVX2 instructions."""
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
        assert x.size % self.input == 0
        tokens = x.size // self.input
        y = np.zeros(tokens * self.output, dtype=np.float32)
        lib().oracle_matrix_apply(_p(self.data, _i8), _p(self.scales, _f), _p(self.offsets, _f),
                                  self.input, self.output, self.weight_bits, self.activation_bits,
                                  _p(x, _f), tokens, mode, _p(y, _f))
        return y.reshape(tokens, self.output)


# ------------------------------------------------------------------ fitters
def fit_mse(x, simd=1):
    x = np.ascontiguousarray(x, dtype=np.float32)
    codes = np.zeros(x.size, dtype=np.int8)
    s = lib().oracle_fit_mse(_p(x, _f), x.size, simd, _p(codes, _i8))
    return np.float32(s), codes


def fit_affine(x, simd=1):
    x = np.ascontiguousarray(x, dtype=np.float32)
    codes = np.zeros(x.size, dtype=np.int8)
    s = np.zeros(1, np.float32)
    b = np.zeros(1, np.float32)
    lib().oracle_fit_affine(_p(x, _f), x.size, simd, _p(codes, _i8), _p(s, _f), _p(b, _f))
    return s[0], b[0], codes


def fit_nf4(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    codes = np.zeros(x.size, dtype=np.int8)
    s = lib().oracle_fit_nf4(_p(x, _f), x.size, _p(codes, _i8))
    return np.float32(s), codes


NF4 = np.array([-1., -0.6961928, -0.52507305, -0.3949175, -0.28444138, -0.18477343, -0.091050036, 0.,
                0.0795803, 0.1609302, 0.2461123, 0.33791524, 0.44070983, 0.562617, 0.72295684, 1.],
               dtype=np.float32)


# ------------------------------------------------------------------ embeddings
class Embedding:
    """quantized_rows.rs:4-115"""

    def __init__(self, bf16, columns, bits, fit=0, simd=1):
        bf16 = np.ascontiguousarray(bf16, dtype=np.uint16)
        if bits not in (4, 8) or columns <= 0 or columns % GROUP or bf16.size % columns:
            raise ValueError("invalid embedding precision or width")
        self.columns, self.bits, self.nf4 = columns, bits, fit == 3
        groups = bf16.size // GROUP
        self.rows = bf16.size // columns
        self.data = np.zeros(bf16.size * bits // 8, dtype=np.uint8)
        self.scales = np.zeros(groups, dtype=np.float32)
        self.offsets = np.zeros(groups, dtype=np.float32) if fit == 2 else None
        rc = lib().oracle_embedding_from_bf16(_p(bf16, _u16), self.rows, columns, bits, fit, simd,
                                              _p(self.data, _u8), _p(self.scales, _f), _p(self.offsets, _f))
        if rc:
            raise ValueError("non-finite embedding" if rc == -2 else "invalid embedding")

    def bytes(self):
        return self.data.size + (self.scales.size + (0 if self.offsets is None else self.offsets.size)) * 4

    def append(self, id_: int) -> np.ndarray:
        out = np.zeros(self.columns, dtype=np.float32)
        lib().oracle_embedding_append(_p(self.data, _u8), _p(self.scales, _f), _p(self.offsets, _f),
                                      self.columns, self.bits, int(self.nf4), id_, _p(out, _f))
        return out


# ------------------------------------------------------------------ layer math
def rms(x, weight, eps=1e-6, zero_centered=False):
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(weight, dtype=np.float32)
    y = np.empty_like(x)
    lib().oracle_rms(_p(x, _f), _p(y, _f), x.size // w.size, w.size, _p(w, _f), eps, int(zero_centered))
    return y


def silu_mul(g, u):
    g = np.array(g, dtype=np.float32, copy=True)
    u = np.ascontiguousarray(u, dtype=np.float32)
    lib().oracle_silu_mul(_p(g, _f), _p(u, _f), g.size)
    return g


def rope(x, heads, head_dim, rotary, offset=0, theta=1e6):
    x = np.array(x, dtype=np.float32, copy=True)
    tokens = x.size // (heads * head_dim)
    lib().oracle_rope(_p(x, _f), tokens, heads, head_dim, rotary, offset, theta)
    return x


def attention(q, k, v, q_heads, kv_heads, head_dim, scale=None):
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    tokens = q.size // (q_heads * head_dim)
    out = np.zeros_like(q)
    s = 1.0 / np.sqrt(head_dim) if scale is None else scale
    lib().oracle_attention(_p(q, _f), _p(k, _f), _p(v, _f), tokens, q_heads, kv_heads, head_dim,
                           float(np.float32(s)), _p(out, _f))
    return out


# ------------------------------------------------------------------ composed encoder
class _Cfg(C.Structure):
    _fields_ = [("layers", C.c_int), ("hidden", C.c_int), ("q_heads", C.c_int), ("kv_heads", C.c_int),
                ("head_dim", C.c_int), ("ffn", C.c_int), ("vocab", C.c_int), ("weight_bits", C.c_int),
                ("activation_bits", C.c_int), ("rope_theta", C.c_float), ("eps", C.c_float), ("causal", C.c_int)]


class _W(C.Structure):
    _fields_ = [("embedding", _u16)] + [(n, C.POINTER(_u16)) for n in ("q", "k", "v", "o", "gate", "up", "down")] + \
               [(n, C.POINTER(_f)) for n in ("input_norm", "post_norm", "q_norm", "k_norm")] + [("final_norm", _f)]


PROJECTIONS = ("q", "k", "v", "o", "gate", "up", "down")
NORMS = ("input_norm", "post_norm", "q_norm", "k_norm")


class Encoder:
    """Composed Qwen3-shaped encoder forward from the primitives above.

    weights: dict with 'embedding' bf16 [vocab, hidden], per-layer lists of bf16 [out, in] for
    PROJECTIONS, per-layer f32 lists for NORMS, and 'final_norm' f32 [hidden]."""

    def __init__(self, cfg: dict, weights: dict):
        self.cfg = cfg
        c = _Cfg(cfg["layers"], cfg["hidden"], cfg["q_heads"], cfg["kv_heads"], cfg["head_dim"], cfg["ffn"],
                 cfg["vocab"], cfg.get("weight_bits", 4), cfg.get("activation_bits", 8),
                 cfg.get("rope_theta", 1e6), cfg.get("eps", 1e-6), int(cfg.get("causal", 0)))
        keep = []

        def arr(a, dt):
            a = np.ascontiguousarray(a, dtype=dt)
            keep.append(a)
            return a

        L = cfg["layers"]
        w = _W()
        w.embedding = _p(arr(weights["embedding"], np.uint16), _u16)
        for n in PROJECTIONS:
            ptrs = (_u16 * L)(*[_p(arr(t, np.uint16), _u16) for t in weights[n]])
            keep.append(ptrs)
            setattr(w, n, C.cast(ptrs, C.POINTER(_u16)))
        for n in NORMS:
            ptrs = (_f * L)(*[_p(arr(t, np.float32), _f) for t in weights[n]])
            keep.append(ptrs)
            setattr(w, n, C.cast(ptrs, C.POINTER(_f)))
        w.final_norm = _p(arr(weights["final_norm"], np.float32), _f)
        self._h = lib().oracle_encoder_create(C.byref(c), C.byref(w))
        if not self._h:
            raise ValueError("oracle encoder creation failed")

    def forward(self, ids, layers=-1, mode=2, hidden=False):
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        D = self.cfg["hidden"]
        pooled = np.zeros(D, dtype=np.float32)
        h = np.zeros((ids.size, D), dtype=np.float32) if hidden else None
        rc = lib().oracle_encoder_forward(self._h, _p(ids, _i32), ids.size, layers, mode, _p(pooled, _f),
                                          _p(h, _f))
        if rc:
            raise ValueError("oracle encoder forward failed")
        return (pooled, h) if hidden else pooled

    def __del__(self):
        if getattr(self, "_h", None):
            lib().oracle_encoder_destroy(self._h)
            self._h = None


def num_threads() -> int:
    return int(lib().oracle_num_threads())


def set_threads(n: int) -> None:
    lib().oracle_set_threads(n)


def lm_logprobs(embedding_bf16, hidden_rows, continuations, weight_bits=4, mode=0):
    """Log-probabilities of continuation tokens from an LM head tied to the embedding matrix.  The
    reference has no LM head for this path (its Kev/Jev score through small heads on the hidden
    state); this is the scoring the C5 configuration names: logits = int8::Matrix(embedding)
    applied to the final-normed rows (int8.rs:166-288 numerics, activation codes of 8 bits), then a
    float64 log-softmax.  hidden_rows [1 + B*T, D]: the prefix's last state, then continuation b's
    token j at row 1 + b*T + j; continuations [B, T] -> [B, T]."""
    hidden_rows = np.ascontiguousarray(hidden_rows, dtype=np.float32)
    D = hidden_rows.shape[1]
    emb = np.ascontiguousarray(embedding_bf16, dtype=np.uint16).reshape(-1, D)
    V = emb.shape[0]
    conts = np.asarray(continuations)
    B, T = conts.shape
    logits = Matrix(emb.reshape(-1), D, V, weight_bits, 8).apply(hidden_rows, mode=mode).astype(np.float64)
    mx = logits.max(axis=1, keepdims=True)
    lse = (mx + np.log(np.exp(logits - mx).sum(axis=1, keepdims=True)))[:, 0]
    out = np.empty((B, T), np.float64)
    for b in range(B):
        for t in range(T):
            row = 0 if t == 0 else 1 + b * T + t - 1
            out[b, t] = logits[row, conts[b, t]] - lse[row]
    return out


# ------------------------------------------------------------------ Decima int8 (decima/int8.rs)
def decima_quantize_rows(x, block: int):
    """[rows, cols] f32 -> (codes int8 [rows, groups*block], scales f32 [rows, groups])."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, cols = x.shape
    groups = -(-cols // block)
    codes = np.zeros((rows, groups * block), np.int8)
    scales = np.zeros((rows, groups), np.float32)
    lib().oracle_decima_quantize_rows(_p(x, _f), rows, cols, block, _p(codes, _i8), _p(scales, _f))
    return codes, scales


class DecimaMatrix:
    """decima::int8::Matrix, weights f32 [rows, cols]: WeightsActivations mode (W8A8) by default,
    Weights mode (W8A32: f32 activations) with weights_only=True."""

    def __init__(self, weights, block: int, weights_only: bool = False):
        self.weights_only = weights_only
        w = np.ascontiguousarray(weights, dtype=np.float32)
        if block not in (16, 32, 64, 128) or not np.all(np.isfinite(w)):
            raise ValueError("INT8 block must be 16, 32, 64 or 128 and weights finite")
        self.rows, self.cols = w.shape
        self.block = block
        self.codes, self.scales = decima_quantize_rows(w, block)

    def apply(self, x, bias=None, mode: int = 0):
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, self.cols)
        y = np.zeros((x.shape[0], self.rows), np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        fn = lib().oracle_decima_apply_w8a32 if self.weights_only else lib().oracle_decima_apply_w8a8
        fn(_p(self.codes, _i8), _p(self.scales, _f), self.rows, self.cols, self.block, _p(x, _f), x.shape[0],
           _p(b, _f), mode, _p(y, _f))
        return y


def layer_norm(x, w, b, eps):
    x = np.array(x, dtype=np.float32, copy=True)
    rows, d = x.reshape(-1, x.shape[-1]).shape
    lib().oracle_layer_norm(_p(x, _f), rows, d, _p(np.ascontiguousarray(w, np.float32), _f),
                            _p(np.ascontiguousarray(b, np.float32), _f), eps)
    return x


def gelu(x):
    x = np.array(x, dtype=np.float32, copy=True)
    lib().oracle_gelu(_p(x, _f), x.size)
    return x


def bert_score_head(pooled, w, b):
    """The scorer head of the cross-encoder: an f32 linear over each pooled state, summed in index
    order from 0 with a separate multiply and add per term, then the bias (decima/mod.rs:482, 701:
    the `score` linear, Precision::F32, Kernel::Portable).  pooled [S, D], w [O, D], b [O] ->
    [S, O]."""
    pooled = np.asarray(pooled, np.float32)
    w, b = np.asarray(w, np.float32), np.asarray(b, np.float32)
    out = np.empty((pooled.shape[0], w.shape[0]), np.float32)
    for s in range(pooled.shape[0]):
        for o in range(w.shape[0]):
            acc = np.float32(0)
            for k in range(w.shape[1]):
                acc = np.float32(acc + np.float32(pooled[s, k] * w[o, k]))
            out[s, o] = np.float32(acc + b[o])
    return out


def bert_forward(cfg: dict, w: dict, ids, mode: int = 0):
    """Composed Decima (BERT-shaped, decima/mod.rs:492-556) encoder forward with W8A8 block
    projections: x = LN(word[id] + type[0] + pos[p]); per layer x = LN(x + o(attn(q, k, v)));
    x = LN(x + ff2(gelu(ff1(x)))).  cfg["mode"] = 1 runs the projections in Weights mode (W8A32).
    Returns (mean-pooled, hidden [T, D])."""
    D, H, block, eps = cfg["hidden"], cfg["heads"], cfg["block"], cfg["eps"]
    wo = bool(cfg.get("mode", 0))  # 1: Weights mode (W8A32)
    hd = D // H
    ids = np.asarray(ids)
    T = ids.size
    x = ((w["word"][ids] + w["type"][0][None, :]).astype(np.float32) + w["pos"][:T]).astype(np.float32)
    x = layer_norm(x, w["emb_ln_w"], w["emb_ln_b"], eps)
    for l in range(cfg["layers"]):
        L = w["layers"][l]
        q = DecimaMatrix(L["q"], block, wo).apply(x, bias=L["bq"], mode=mode)
        k = DecimaMatrix(L["k"], block, wo).apply(x, bias=L["bk"], mode=mode)
        v = DecimaMatrix(L["v"], block, wo).apply(x, bias=L["bv"], mode=mode)
        ctx = attention(q, k, v, H, H, hd, scale=1.0 / np.sqrt(hd))
        o = DecimaMatrix(L["o"], block, wo).apply(ctx, bias=L["bo"], mode=mode)
        x = layer_norm((x + o).astype(np.float32), L["ln1_w"], L["ln1_b"], eps)
        h = gelu(DecimaMatrix(L["ff1"], block, wo).apply(x, bias=L["b1"], mode=mode))
        o2 = DecimaMatrix(L["ff2"], block, wo).apply(h, bias=L["b2"], mode=mode)
        x = layer_norm((x + o2).astype(np.float32), L["ln2_w"], L["ln2_b"], eps)
    return x.mean(axis=0, dtype=np.float32), x
