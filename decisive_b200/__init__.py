"""decisive_b200: B200 (sm_100a) backend for decisive's quantised projection path.

Two layers, both thin over the C ABI of libdecisive_b200.so (include/decisive_b200.h):

* kernel level -- torch-tensor wrappers of the group-64 quantiser, weight packer, grouped GEMM
  (tensor-core and GEMV paths), fused MLP, attention and dequantisation.  torch supplies device
  memory and streams only; every computation runs in this library's CUDA kernels.
* model level -- ``Model`` / ``Cache`` / ``Cancellation`` / ``Error`` mirroring the reference's
  ``inference`` module (src/inference/mod.rs:17-273): ``predict`` and ``predict_batch`` with the
  same error codes, cache ownership and cancellation rules.
"""
from __future__ import annotations

import ctypes as C
import json
from dataclasses import dataclass, field

from . import _lib
from ._lib import CudaError, check, load

GROUP = 64
CODES_NATURAL, CODES_GEMV, CODES_TC, CODES_DQ = 0, 1, 2, 3
DTYPES = {"float32": 0, "float16": 1, "bfloat16": 2}


def _ptr(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


def _stream(stream=None):
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


def padded(k: int) -> int:
    return (k + GROUP - 1) // GROUP * GROUP


def scale_stride(n: int) -> int:
    """Row stride of scale arrays: roundup(n, 128) (db_scale_row_stride)."""
    return (n + 127) // 128 * 128


# ------------------------------------------------------------------ kernel level
def quantize_activations(x, bits: int = 8, layout: int = CODES_TC, sums: bool = False, nonfinite=None):
    """int8::Matrix::prepare (int8.rs:178-202) on the GPU -> (codes, scales [G, M], sums [G, M] | None)."""
    import torch
    assert x.is_cuda and x.dim() == 2
    M, K = x.shape
    Kp = padded(K)
    G = Kp // GROUP
    dt = torch.float16 if layout in (CODES_TC, CODES_DQ) else torch.int8
    codes = torch.zeros((M, Kp), dtype=dt, device=x.device)
    lds = scale_stride(max(M, 1))
    scales = torch.zeros((G, lds), dtype=torch.float32, device=x.device)
    s = torch.zeros((G, lds), dtype=torch.int32, device=x.device) if sums else None
    check(load().db_quantize_activations_g64(_ptr(x), DTYPES[str(x.dtype).split(".")[1]], x.stride(0), M, K, bits,
                                             _ptr(codes), layout, Kp, _ptr(scales), _ptr(s), lds,
                                             _ptr(nonfinite), _stream()))
    return codes, scales, s


def pack_weights(bf16, bits: int = 4):
    """Absmax group-64 weight quantiser (int8.rs:51-152, packed.rs:31-56): bf16 [N, K] (as int16/uint16
    bits or torch.bfloat16) -> (codes, scales [G, N])."""
    import torch
    N, K = bf16.shape
    Kp = padded(K)
    codes = torch.empty((N, Kp * bits // 8), dtype=torch.uint8, device=bf16.device)
    scales = torch.empty((Kp // GROUP, scale_stride(N)), dtype=torch.float32, device=bf16.device)
    check(load().db_pack_weights_g64(_ptr(bf16), N, K, bits, _ptr(codes), _ptr(scales), _stream()))
    return codes, scales


def import_packed(packed, N: int, K: int, bits: int):
    import torch
    codes = torch.empty((N, K * bits // 8), dtype=torch.uint8, device=packed.device)
    scales = torch.empty((K // GROUP, scale_stride(N)), dtype=torch.float32, device=packed.device)
    check(load().db_import_packed(_ptr(packed), N, K, bits, _ptr(codes), _ptr(scales), _stream()))
    return codes, scales


def export_packed(codes, scales, N: int, K: int, bits: int):
    import torch
    out = torch.empty(N * (K // GROUP) * (GROUP * bits // 8 + 4), dtype=torch.uint8, device=codes.device)
    check(load().db_export_packed(_ptr(codes), _ptr(scales), N, K, bits, _ptr(out), _stream()))
    return out


def dequant_rows(codes, scales, N: int, K: int, bits: int, ids=None):
    import torch
    T = N if ids is None else ids.numel()
    out = torch.empty((T, K), dtype=torch.float32, device=codes.device)
    check(load().db_dequant_rows_g64(_ptr(codes), _ptr(scales), N, K, bits, _ptr(ids), T, _ptr(out), K, _stream()))
    return out


class GemmConfig(C.Structure):
    """db_gemm_config: tile width (0 = default, 64, 128, 256), persistent grid cap (0 = all SMs) and
    CTA pairing (1 = clusters of two CTAs with M = 256 MMAs).  The tuner's candidate space."""
    _fields_ = [("block_n", C.c_int), ("max_ctas", C.c_int), ("pair_ctas", C.c_int)]


def gemm(a_codes, layout, sa, w_codes, sw, M, N, K, bits, fused=True, a_sums=None, residual=None, nonfinite=None,
         config=None):
    """Matrix::apply_prepared (int8.rs:229-288) on prepared activations -> y f32 [M, N].
    config: optional GemmConfig (tile configuration of the tensor-core path).  CODES_DQ: a_codes are
    the dequantised f16 activations (sa may be None); the kind::f16 full-K GEMM (tolerance numerics)."""
    import torch
    y = residual if residual is not None else torch.empty((M, N), dtype=torch.float32, device=w_codes.device)
    cfg = C.byref(config) if config is not None else None
    check(load().db_gemm_g64_config(_ptr(a_codes), layout, a_codes.stride(0), _ptr(sa), _ptr(a_sums),
                                    sa.stride(0) if sa is not None else 0,
                                    _ptr(w_codes), _ptr(sw), M, N, K, bits, int(fused), int(residual is not None),
                                    _ptr(y), N, _ptr(nonfinite), cfg, _stream()))
    return y


def decima_quantize_weights(w, block: int = 32):
    """decima::int8::Matrix::new (W8, decima/int8.rs:106-151): f32 [N, K] device tensor ->
    (codes uint8 [N, Kp], scales f32 [ceil(K/block), scale_stride(N)])."""
    import torch
    N, K = w.shape
    Kp = -(-K // GROUP) * GROUP
    codes = torch.zeros((N, Kp), dtype=torch.uint8, device=w.device)
    scales = torch.empty((-(-K // block), scale_stride(N)), dtype=torch.float32, device=w.device)
    check(load().db_decima_quantize_weights(_ptr(w), N, K, block, _ptr(codes), _ptr(scales), _stream()))
    return codes, scales


def decima_quantize_activations(x, block: int = 32, layout: int = CODES_TC):
    """The activation fill of decima Matrix::apply_with_rows: f32 [M, K] -> (codes, scales, nonfinite flag)."""
    import torch
    M, K = x.shape
    Kp = -(-K // GROUP) * GROUP
    dt = torch.float16 if layout == CODES_TC else torch.int8
    codes = torch.zeros((M, Kp), dtype=dt, device=x.device)
    scales = torch.empty((-(-K // block), scale_stride(M)), dtype=torch.float32, device=x.device)
    flag = torch.zeros(1, dtype=torch.int32, device=x.device)
    check(load().db_decima_quantize_activations(_ptr(x), M, K, block, _ptr(codes), layout, Kp, _ptr(scales),
                                                scales.stride(0), _ptr(flag), _stream()))
    return codes, scales, flag


def decima_linear(x, w_codes, w_scales, N: int, block: int = 32, fused: bool = True, bias=None):
    """decima Matrix::apply_with_rows, WeightsActivations mode: y [M, N] = W8A8 grouped GEMM + bias."""
    import torch
    M, K = x.shape
    ws = torch.empty(load().db_decima_workspace_bytes(M, K, block), dtype=torch.uint8, device=x.device)
    y = torch.empty((M, N), dtype=torch.float32, device=x.device)
    check(load().db_decima_linear(_ptr(x), M, K, _ptr(w_codes), _ptr(w_scales), N, block, int(fused), _ptr(bias),
                                  _ptr(y), _ptr(ws), _stream()))
    return y


def decima_linear_w8a32(x, w_codes, w_scales, N: int, block: int = 32, fused: bool = True, bias=None):
    """decima Matrix::apply_with_rows, Weights mode: y [M, N] = f32 x times the int8 weight codes
    (decoded with their block scales) + bias."""
    import torch
    M, K = x.shape
    flag = torch.zeros(1, dtype=torch.int32, device=x.device)
    y = torch.empty((M, N), dtype=torch.float32, device=x.device)
    check(load().db_decima_linear_w8a32(_ptr(x), M, K, _ptr(w_codes), _ptr(w_scales), N, block, int(fused),
                                        _ptr(bias), _ptr(y), _ptr(flag), _stream()))
    return y


EPILOGUE_STORE, EPILOGUE_RESIDUAL, EPILOGUE_SWIGLU = 0, 1, 2


def tune_gemm(M: int, N: int, K: int, bits: int, epilogue: int = EPILOGUE_STORE, cache_path: str | None = None):
    """Kernel-selection tuner for one GEMM shape (the reference's rule, webgpu/checkpoint.rs:420-565):
    the fastest tile configuration bitwise equal to the default and >= 1 % faster.  Returns
    (GemmConfig, report dict)."""
    import json
    choice = GemmConfig()
    buf = C.create_string_buffer(16384)
    path = cache_path.encode() if cache_path else None
    check(load().db_gemm_tune(M, N, K, bits, epilogue, path, C.byref(choice), buf, len(buf)))
    return choice, json.loads(buf.value.decode())


def linear(x, w_codes, sw, N: int, weight_bits: int = 4, activation_bits: int = 8, fused: bool = True):
    """Matrix::apply (int8.rs:166-176): quantise + grouped GEMM (GEMV path for small M)."""
    import torch
    M, K = x.shape
    ws = torch.empty(load().db_linear_workspace_bytes(M, K), dtype=torch.uint8, device=x.device)
    y = torch.empty((M, N), dtype=torch.float32, device=x.device)
    check(load().db_linear_g64(_ptr(x), M, K, _ptr(w_codes), _ptr(sw), N, weight_bits, activation_bits, int(fused),
                               _ptr(y), _ptr(ws), _stream()))
    return y


def linear_noalloc(x, w_codes, sw, N: int, weight_bits: int = 4, activation_bits: int = 8, fused: bool = True,
                   out=None):
    """Matrix::apply without any device allocation by the library: for hosts that forbid it.  Uses
    the library's fixed scratch array (db_linear_noalloc_scratch_bytes()); see the C header for the
    sharing rules."""
    import torch
    M, K = x.shape
    y = torch.empty((M, N), dtype=torch.float32, device=x.device) if out is None else out
    check(load().db_linear_g64_noalloc(_ptr(x), M, K, _ptr(w_codes), _ptr(sw), N, weight_bits, activation_bits,
                                       int(fused), _ptr(y), _stream()))
    return y


def project_packed(x, w_codes, sw, outputs: int, bits: int):
    """packed::project (packed.rs:75-119) for one activation row."""
    import torch
    K = x.numel()
    ws = torch.empty(load().db_linear_workspace_bytes(1, K), dtype=torch.uint8, device=x.device)
    y = torch.empty(outputs, dtype=torch.float32, device=x.device)
    check(load().db_project_packed(_ptr(x), K, _ptr(w_codes), _ptr(sw), outputs, bits, _ptr(y), _ptr(ws), _stream()))
    return y


def interleave_gate_up(gate_codes, gate_scales, up_codes, up_scales, F: int, K: int, bits: int):
    import torch
    codes = torch.empty((2 * F, gate_codes.shape[1]), dtype=torch.uint8, device=gate_codes.device)
    scales = torch.empty((gate_scales.shape[0], scale_stride(2 * F)), dtype=torch.float32, device=gate_codes.device)
    check(load().db_interleave_gate_up(_ptr(gate_codes), _ptr(gate_scales), _ptr(up_codes), _ptr(up_scales), F, K,
                                       bits, _ptr(codes), _ptr(scales), _stream()))
    return codes, scales


def mlp(a_codes, sa, gu_codes, gu_scales, M: int, F: int, K: int, bits: int, fused: bool = True, nonfinite=None):
    """Fused gate/up + SiLU*up + re-quantisation (grouped_q4_mlp.wgsl) -> (codes [M, F], scales [F/64, M]).
    The code layout follows a_codes: f16 tensor-core codes (db_mlp_g64) or int8 natural codes
    (db_mlp_g64_natural, the kind::i8 path)."""
    import torch
    natural = a_codes.dtype == torch.int8
    codes = torch.zeros((M, F), dtype=torch.int8 if natural else torch.float16, device=a_codes.device)
    scales = torch.zeros((F // GROUP, scale_stride(M)), dtype=torch.float32, device=a_codes.device)
    fn = load().db_mlp_g64_natural if natural else load().db_mlp_g64
    check(fn(_ptr(a_codes), a_codes.stride(0), _ptr(sa), sa.stride(0), _ptr(gu_codes), _ptr(gu_scales),
             M, F, K, bits, int(fused), _ptr(codes), F, _ptr(scales), scale_stride(M), _ptr(nonfinite), _stream()))
    return codes, scales


def attention(q16, k16, v16, q_heads: int, kv_heads: int, scale: float | None = None):
    import torch
    T = q16.shape[0]
    out = torch.empty((T, q_heads * 128), dtype=torch.float32, device=q16.device)
    s = (1.0 / 128 ** 0.5) if scale is None else scale
    check(load().db_attention(_ptr(q16), _ptr(k16), _ptr(v16), T, q_heads, kv_heads, 128, s, _ptr(out),
                              q_heads * 128, _stream()))
    return out


def attention_decoder(q16, k16, v16, items: int, q_heads: int, kv_heads: int, kp16=None, vp16=None,
                      causal: bool = True, scale: float | None = None):
    """Decoder attention: `items` items of q16.shape[0] // items rows, each after the cached prefix
    keys kp16/vp16 [P, kv_heads, 128] (None: no prefix), causal own keys when asked."""
    import torch
    R = q16.shape[0]
    out = torch.empty((R, q_heads * 128), dtype=torch.float32, device=q16.device)
    s = (1.0 / 128 ** 0.5) if scale is None else scale
    P = 0 if kp16 is None else kp16.shape[0]
    check(load().db_attention_decoder(_ptr(q16), _ptr(k16), _ptr(v16), items, R // items,
                                      _ptr(kp16) if P else None, _ptr(vp16) if P else None, P, int(causal), q_heads,
                                      kv_heads, 128, s, _ptr(out), q_heads * 128, _stream()))
    return out


def synthetic_bf16(seed: int, tensor: int, shape, std: float, device="cuda"):
    import torch
    out = torch.empty(shape, dtype=torch.int16, device=device)
    check(load().db_synthetic_bf16(seed, tensor, out.numel(), std, _ptr(out), _stream()))
    return out


def device_error_word() -> int:
    return int(load().db_device_error_word())


# ------------------------------------------------------------------ model level (inference API mirror)
class Error(Exception):
    """inference::Error {code, message} (src/inference/mod.rs:44-85)."""

    def __init__(self, code: str, message: str):
        super().__init__(f"{code}: {message}")
        self.code, self.message = code, message

    @staticmethod
    def _from(e: _lib.DbError) -> "Error":
        return Error(e.code.decode(), e.message.decode())


class Cancellation:
    """inference::Cancellation (mod.rs:87-100): a shared flag the library polls."""

    def __init__(self):
        self._flag = C.c_uint8(0)  # the layout of Rust's AtomicBool

    def cancel(self):
        self._flag.value = 1

    def check(self):
        if self._flag.value:
            raise Error("CANCELLED", "Inference was cancelled")

    @property
    def ptr(self):
        return C.byref(self._flag)


@dataclass
class CacheOptions:
    """inference::CacheOptions (mod.rs:102-115)."""
    max_bytes: int = 64 * 1024 * 1024
    require_prefix: bool = False


@dataclass
class PplxParameters:
    """inference::PplxParameters (parameters.rs:81-103)."""
    max_sequence_tokens: int = 1024


@dataclass
class EncoderConfig:
    layers: int = 28
    hidden: int = 1024
    q_heads: int = 16
    kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 3072
    vocab: int = 151936
    weight_bits: int = 4
    rope_theta: float = 1e6
    eps: float = 1e-6
    max_sequence_tokens: int = 1024
    fused: bool = True
    causal: bool = False  # True: decoder (causal attention, prefix caches)

    def c(self) -> _lib.EncoderConfig:
        return _lib.EncoderConfig(self.layers, self.hidden, self.q_heads, self.kv_heads, self.head_dim, self.ffn,
                                  self.vocab, self.weight_bits, self.rope_theta, self.eps, self.max_sequence_tokens,
                                  int(self.fused), int(self.causal))


@dataclass
class Response:
    """inference::Response (mod.rs:127-132); `response` is the pooled embedding."""
    response: object
    model: str
    backend: str


@dataclass
class Outcome:
    """inference::Outcome (mod.rs:133-138)."""
    status: str
    result: Response | None = None
    error: Error | None = None


class Cache:
    def __init__(self, handle, model):
        self._h, self._model = handle, model

    def stats(self) -> dict:
        """Prefix reuse counters (kev/mod.rs Stats): hits, prefix tokens reused / computed."""
        v = (C.c_int64 * 3)()
        check(load().db_cache_stats(self._h, C.byref(v, 0), C.byref(v, 8), C.byref(v, 16)))
        return {"hits": v[0], "prefix_tokens_reused": v[1], "prefix_tokens_computed": v[2]}

    def __del__(self):
        if getattr(self, "_h", None):
            load().db_cache_destroy(self._h)
            self._h = None


class Model:
    """inference::Model<B> (mod.rs:156-273) over the CUDA encoder backend."""

    def __init__(self, handle, config: EncoderConfig):
        self._h, self.config = handle, config
        self.defaults = PplxParameters(config.max_sequence_tokens)

    @classmethod
    def synthetic(cls, config: EncoderConfig, seed: int = 0, std: float = 0.02, device: int = 0) -> "Model":
        err = _lib.DbError()
        cfg = config.c()
        h = load().db_model_create_synthetic(device, C.byref(cfg), seed, std, C.byref(err))
        if not h:
            raise Error._from(err)
        return cls(h, config)

    @classmethod
    def from_weights(cls, config: EncoderConfig, weights: dict, device: int = 0) -> "Model":
        """weights: 'embedding' bf16 bits [vocab, hidden]; per-layer lists 'q','k','v','o','gate','up','down'
        (bf16 bits [out, in]); per-layer f32 'input_norm','post_norm','q_norm','k_norm'; 'final_norm'."""
        import numpy as np
        keep = []

        def arr(a, dt):
            a = np.ascontiguousarray(a, dtype=dt)
            keep.append(a)
            return a.ctypes.data_as(C.POINTER(C.c_uint16 if dt == np.uint16 else C.c_float))

        w = _lib.EncoderWeights()
        w.embedding = arr(weights["embedding"], np.uint16)
        L = config.layers
        for n in ("q", "k", "v", "o", "gate", "up", "down"):
            p = (C.POINTER(C.c_uint16) * L)(*[arr(t, np.uint16) for t in weights[n]])
            keep.append(p)
            setattr(w, n, C.cast(p, _lib._u16pp))
        for n in ("input_norm", "post_norm", "q_norm", "k_norm"):
            p = (C.POINTER(C.c_float) * L)(*[arr(t, np.float32) for t in weights[n]])
            keep.append(p)
            setattr(w, n, C.cast(p, _lib._fpp))
        w.final_norm = arr(weights["final_norm"], np.float32)
        err = _lib.DbError()
        cfg = config.c()
        h = load().db_model_create(device, C.byref(cfg), C.byref(w), C.byref(err))
        if not h:
            raise Error._from(err)
        return cls(h, config)

    def close(self):
        if getattr(self, "_h", None):
            load().db_model_destroy(self._h)
            self._h = None

    __del__ = close

    def capabilities(self) -> dict:
        buf = C.create_string_buffer(512)
        check(load().db_model_capabilities(self._h, buf, 512))
        return json.loads(buf.value.decode())

    def synthetic_weight(self, name: str, layer: int = 0):
        import numpy as np
        n = load().db_model_synthetic_weight(self._h, name.encode(), layer, None, 0)
        if n < 0:
            raise CudaError(int(n))
        out = np.empty(n, dtype=np.uint16)
        got = load().db_model_synthetic_weight(self._h, name.encode(), layer, out.ctypes.data_as(C.c_void_p), n)
        if got != n:
            raise CudaError(int(got))
        return out

    def create_cache(self, options: CacheOptions | None = None) -> Cache:
        o = options or CacheOptions()
        err = _lib.DbError()
        h = load().db_cache_create(self._h, o.max_bytes, int(o.require_prefix), C.byref(err))
        if not h:
            raise Error._from(err)
        return Cache(h, self)

    def clear_cache(self, cache: Cache):
        err = _lib.DbError()
        if load().db_cache_clear(self._h, cache._h, C.byref(err)):
            raise Error._from(err)

    def _params(self, parameters):
        p = parameters or self.defaults
        return _lib.Parameters(p.max_sequence_tokens)

    def predict(self, ids, parameters: PplxParameters | None = None, cache: Cache | None = None,
                cancellation: Cancellation | None = None, out=None) -> Response:
        import numpy as np
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.empty(self.config.hidden, dtype=np.float32) if out is None else out
        err = _lib.DbError()
        p = self._params(parameters)
        rc = load().db_predict(self._h, ids.ctypes.data_as(C.c_void_p), ids.size, C.byref(p),
                               cache._h if cache else None, cancellation.ptr if cancellation else None,
                               out.ctypes.data_as(C.c_void_p), C.byref(err))
        if rc:
            raise Error._from(err)
        caps = self.capabilities()
        return Response(out, caps["model"], caps["backend"])

    def predict_continuations(self, prefix, continuations, cache: Cache | None = None,
                              cancellation: Cancellation | None = None):
        """Causal models: the final-normed hidden states [count, tokens, hidden] of each continuation
        (equal-length token lists) after a shared prefix, whose per-layer keys and values are
        computed once or reused from the cache (kev/mod.rs:163-300)."""
        import numpy as np
        pre = np.ascontiguousarray(prefix, dtype=np.int32)
        cont = np.ascontiguousarray(continuations, dtype=np.int32)
        if cont.ndim != 2:
            raise ValueError("continuations must be equal-length token lists")
        out = np.empty((cont.shape[0], cont.shape[1], self.config.hidden), dtype=np.float32)
        err = _lib.DbError()
        rc = load().db_predict_continuations(self._h, cache._h if cache else None, pre.ctypes.data_as(C.c_void_p),
                                             pre.size, cont.ctypes.data_as(C.c_void_p), cont.shape[0], cont.shape[1],
                                             cancellation.ptr if cancellation else None,
                                             out.ctypes.data_as(C.c_void_p), C.byref(err))
        if rc:
            raise Error._from(err)
        return out

    def score_continuations(self, prefix, continuations, cache: Cache | None = None,
                            cancellation: Cancellation | None = None, hidden: bool = False):
        """Causal models: per-token log-probabilities [count, tokens] of each continuation after the
        shared prefix, from an LM head tied to the embedding matrix (the continuation's score is
        the row sum).  With hidden=True also the LM head's input rows [1 + count*tokens, hidden]:
        the prefix's last final-normed state, then the continuations' states."""
        import numpy as np
        pre = np.ascontiguousarray(prefix, dtype=np.int32)
        cont = np.ascontiguousarray(continuations, dtype=np.int32)
        if cont.ndim != 2:
            raise ValueError("continuations must be equal-length token lists")
        out = np.empty(cont.shape, dtype=np.float32)
        h = np.empty((1 + cont.size, self.config.hidden), dtype=np.float32) if hidden else None
        err = _lib.DbError()
        rc = load().db_score_continuations(self._h, cache._h if cache else None, pre.ctypes.data_as(C.c_void_p),
                                           pre.size, cont.ctypes.data_as(C.c_void_p), cont.shape[0], cont.shape[1],
                                           cancellation.ptr if cancellation else None,
                                           out.ctypes.data_as(C.c_void_p),
                                           h.ctypes.data_as(C.c_void_p) if h is not None else None, C.byref(err))
        if rc:
            raise Error._from(err)
        return (out, h) if hidden else out

    def predict_batch(self, requests, parameters: PplxParameters | None = None, cache: Cache | None = None,
                      cancellation: Cancellation | None = None) -> list[Outcome]:
        import numpy as np
        reqs = [np.ascontiguousarray(r, dtype=np.int32) for r in requests]
        n = len(reqs)
        ptrs = (C.c_void_p * max(n, 1))(*[r.ctypes.data_as(C.c_void_p).value for r in reqs])
        lens = (C.c_size_t * max(n, 1))(*[r.size for r in reqs])
        outs = np.zeros((max(n, 1), self.config.hidden), dtype=np.float32)
        status = np.zeros(max(n, 1), dtype=np.int32)
        errs = (_lib.DbError * max(n, 1))()
        err = _lib.DbError()
        p = self._params(parameters)
        rc = load().db_predict_batch(self._h, ptrs, lens, n, C.byref(p), cache._h if cache else None,
                                     cancellation.ptr if cancellation else None, outs.ctypes.data_as(C.c_void_p),
                                     status.ctypes.data_as(C.c_void_p), errs, C.byref(err))
        if rc:
            raise Error._from(err)
        caps = self.capabilities()
        result = []
        for i in range(n):
            if status[i] == 0:
                result.append(Outcome("success", result=Response(outs[i].copy(), caps["model"], caps["backend"])))
            else:
                result.append(Outcome("error", error=Error._from(errs[i])))
        return result

    def use_graphs(self, enable: bool = True):
        """Forward as a captured CUDA graph per token count (default on); bit-identical either way."""
        check(load().db_model_use_graphs(self._h, int(enable)))

    def set_code_layout(self, layout: int):
        """CODES_NATURAL (int8 codes, kind::i8 GEMM; default) or CODES_TC (f16 codes, kind::f16 GEMM),
        bit-identical outputs either way; or CODES_DQ (dequantised f16 operands, full-K f32
        accumulation: within the contract's tolerance, not bit-identical)."""
        check(load().db_model_set_code_layout(self._h, int(layout)))

    def profile(self, enable: bool = True):
        check(load().db_model_profile(self._h, int(enable)))

    def profile_read(self, reset: bool = True) -> dict:
        """{kernel kind: (total ms, launches)} accumulated since the last reset."""
        import numpy as np
        n = 11
        ms = np.zeros(n, np.float64)
        cnt = np.zeros(n, np.int64)
        check(load().db_model_profile_read(self._h, ms.ctypes.data_as(C.c_void_p), cnt.ctypes.data_as(C.c_void_p), n,
                                           int(reset)))
        return {load().db_model_profile_name(k).decode(): (float(ms[k]), int(cnt[k])) for k in range(n)}

    @classmethod
    def from_packed(cls, config: EncoderConfig, manifest_path: str, verify: bool = True, device: int = 0) -> "Model":
        """Loads a packed checkpoint directory (packed-q4-e4.json / packed-q8-e8.json manifest, the
        reference's export_packed.rs format); verify checks every file's SHA-256."""
        err = _lib.DbError()
        cfg = config.c()
        h = load().db_model_create_packed(device, C.byref(cfg), manifest_path.encode(), int(verify), C.byref(err))
        if not h:
            raise Error._from(err)
        return cls(h, config)

    def set_streaming(self, enable: bool = True):
        """Two-bank layer streaming: weights in pinned host memory, two layers on the device."""
        err = _lib.DbError()
        if load().db_model_set_streaming(self._h, int(enable), C.byref(err)):
            raise Error._from(err)

    def export_packed(self, directory: str) -> str:
        """Writes this model's weights as a packed checkpoint into directory; returns the manifest path."""
        import os
        err = _lib.DbError()
        if load().db_model_export_packed(self._h, directory.encode(), C.byref(err)):
            raise Error._from(err)
        return os.path.join(directory, f"packed-q{self.config.weight_bits}-e{self.config.weight_bits}.json")

    def tune(self, tokens: int | None = None, cache_path: str | None = None) -> dict:
        """Tunes the four projection GEMMs at `tokens` rows (default: max_sequence_tokens) and uses
        the choices from then on; returns the per-projection reports."""
        import json
        err = _lib.DbError()
        buf = C.create_string_buffer(65536)
        n = tokens if tokens is not None else self.config.max_sequence_tokens
        rc = load().db_model_tune(self._h, n, cache_path.encode() if cache_path else None, buf, len(buf), C.byref(err))
        if rc:
            raise Error._from(err)
        return json.loads(buf.value.decode())

    def forward_device(self, ids_dev, out_dev, stream=None):
        """Device-resident forward (no host synchronisation) used for device-timed measurement."""
        check(load().db_forward_device(self._h, _ptr(ids_dev), ids_dev.numel(), _ptr(out_dev), _stream(stream)))


@dataclass
class BertConfig:
    """C4: the Decima-shaped (BERT) encoder on the Decima int8 kernels (db_bert_*)."""
    layers: int = 12
    hidden: int = 768
    heads: int = 12
    ffn: int = 3072
    vocab: int = 128100
    max_positions: int = 512
    block: int = 32
    eps: float = 1e-12
    fused: bool = True
    mode: int = 0  # 0: W8A8 (WeightsActivations), 1: W8A32 (Weights)

    def c(self) -> _lib.BertConfig:
        return _lib.BertConfig(self.layers, self.hidden, self.heads, self.ffn, self.vocab, self.max_positions,
                               self.block, self.eps, int(self.fused), int(self.mode))


class BertModel:
    """Synthetic-weight C4 encoder; predict returns (mean-pooled [hidden], states [n, hidden])."""

    def __init__(self, config: BertConfig, seed: int = 0, std: float = 0.02, device: int = 0):
        err = _lib.DbError()
        cfg = config.c()
        self._h = load().db_bert_create_synthetic(device, C.byref(cfg), seed, std, C.byref(err))
        if not self._h:
            raise Error._from(err)
        self.config, self.seed, self.std = config, seed, std

    def predict(self, ids, hidden: bool = False):
        import numpy as np
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        pooled = np.empty(self.config.hidden, np.float32)
        h = np.empty((ids.size, self.config.hidden), np.float32) if hidden else None
        err = _lib.DbError()
        rc = load().db_bert_predict(self._h, ids.ctypes.data_as(C.c_void_p), ids.size,
                                    pooled.ctypes.data_as(C.c_void_p),
                                    h.ctypes.data_as(C.c_void_p) if h is not None else None, C.byref(err))
        if rc:
            raise Error._from(err)
        return (pooled, h) if hidden else pooled

    HEAD_OUTPUTS = 3

    def score(self, state, choices, pooled: bool = False):
        """One cross-encoder request: logits [len(choices), 3] for the sequences state ++ choice,
        run packed in one pass (and their pooled states [len(choices), hidden] when asked)."""
        import numpy as np
        state = np.ascontiguousarray(state, dtype=np.int32)
        chs = [np.ascontiguousarray(c, dtype=np.int32) for c in choices]
        ptrs = (C.c_void_p * max(len(chs), 1))(*[c.ctypes.data for c in chs])
        lens = (C.c_size_t * max(len(chs), 1))(*[c.size for c in chs])
        logits = np.empty((len(chs), self.HEAD_OUTPUTS), np.float32)
        p = np.empty((len(chs), self.config.hidden), np.float32) if pooled else None
        err = _lib.DbError()
        rc = load().db_bert_score(self._h, state.ctypes.data_as(C.c_void_p), state.size, ptrs, lens, len(chs),
                                  logits.ctypes.data_as(C.c_void_p),
                                  p.ctypes.data_as(C.c_void_p) if p is not None else None, C.byref(err))
        if rc:
            raise Error._from(err)
        return (logits, p) if pooled else logits

    def close(self):
        if getattr(self, "_h", None):
            load().db_bert_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()
