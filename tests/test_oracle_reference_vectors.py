"""The reference crate's own unit tests for the quantised path, re-expressed against the oracle.

These pin oracle/oracle.c to the reference: every generator, shape list, tolerance and
bitwise assertion below is the one in the cited Rust test.  (The reference is Rust and cannot
be compiled in this image, so its tests are restated rather than run.)
"""
import numpy as np
import pytest

GROUP = 64
MIN_POSITIVE = np.float32(np.finfo(np.float32).tiny)


def f32(a):
    return np.asarray(a, dtype=np.float32)


def quant_ref(v, bits):
    """The closure of int8.rs:709-725 (and scale/quantize of int8.rs:291-298)."""
    limit = np.float32(7.0 if bits == 4 else 127.0)
    v = f32(v)
    scale = np.maximum(np.float32(np.max(np.abs(v), initial=np.float32(0))) / limit, MIN_POSITIVE)
    inv = np.float32(1.0) / scale
    q = np.clip(np.rint(v * inv), -limit, limit).astype(np.int64)
    return q, np.float32(scale)


# ---------------------------------------------------------------- int8.rs:678-772
SHAPES_678 = [(0, 7, 1), (1, 1, 1), (3, 63, 7), (7, 65, 9), (9, 129, 33), (15, 65, 9), (16, 65, 9),
              (17, 127, 32), (33, 1025, 65)]


@pytest.mark.parametrize("wb,ab", [(8, 8), (4, 8), (4, 4)])
@pytest.mark.parametrize("m,k,n", SHAPES_678)
def test_q4_and_q8_match_independent_grouped_dots(oracle, wb, ab, m, k, n):
    i = np.arange(k * n)
    weights = oracle.bf16_to_f32(oracle.f32_to_bf16(f32((i * 37 % 257).astype(np.float32) - 128) / np.float32(31)))
    bytes_ = oracle.f32_to_bf16(weights)
    xi = np.arange(m * k)
    x = f32((xi * 13 % 255).astype(np.float32) - 127) / np.float32(17)
    expected = np.zeros(m * n)
    G = -(-k // GROUP)
    for r in range(m):
        for c in range(n):
            tot = 0.0
            for g in range(G):
                end = min(g * GROUP + GROUP, k)
                a, sa = quant_ref(x[r * k + g * GROUP: r * k + end], ab)
                b, sb = quant_ref(weights[c * k + g * GROUP: c * k + end], wb)
                tot += float(np.dot(a, b)) * float(np.float32(sa * sb))
            expected[r * n + c] = tot
    w = oracle.Matrix(bytes_, k, n, wb, ab)
    assert w.bytes() == -(-n // 8) * 8 * G * (GROUP * wb // 8 + 4)
    a = w.apply(x, mode=0).reshape(-1)
    b = w.apply(x, mode=0).reshape(-1)
    assert np.array_equal(a, b)
    # buffered / AVX2 instruction path is bit-identical to the fused numerics (int8.rs:751-758)
    fused = w.apply(x, mode=2).reshape(-1)
    assert np.array_equal(a.view(np.uint32), fused.view(np.uint32)), f"panel cache changed W{wb}A{ab}"
    assert np.all(np.abs(a.astype(np.float64) - expected) <= 1e-4 + np.abs(expected) * 2e-6)
    # portable path (int8.rs:259-287) meets the same bound
    s = w.apply(x, mode=1).reshape(-1)
    assert np.all(np.abs(s.astype(np.float64) - expected) <= 1e-4 + np.abs(expected) * 2e-6)
    zero = w.apply(np.zeros(m * k, np.float32), mode=0)
    assert np.all(zero == 0)


# ---------------------------------------------------------------- int8.rs:774-798
def test_activation_rounding_matches_portable_at_boundaries(oracle):
    values = [0.0, -0.0, float(MIN_POSITIVE), -float(MIN_POSITIVE)]
    for i in range(-127, 127):
        half = np.float32(i + 0.5)
        values += [np.nextafter(half, np.float32(-np.inf)), half, np.nextafter(half, np.float32(np.inf))]
    values = f32(values)
    for s in [1.0, 0.0037, float(MIN_POSITIVE), 1e30]:
        s = np.float32(s)
        scaled = values * s
        for n in [1, 7, 8, 9, 63, 64, 65, scaled.size]:
            v = scaled[:n]
            sc = oracle.group_scale(v, 8)
            ref = np.maximum(np.float32(np.max(np.abs(v))) / np.float32(127), MIN_POSITIVE)
            assert sc == ref
            codes = oracle.pack_codes(v, s, 8)
            inv = np.float32(1) / s
            expect = np.clip(np.rint(v * inv), -127, 127).astype(np.int8)
            assert np.array_equal(codes, expect), (s, n)
            assert np.all(codes != -128)


# ---------------------------------------------------------------- int8.rs:877-949
@pytest.mark.parametrize("m,k,n", [(0, 1, 1), (1, 7, 1), (3, 64, 8), (4, 65, 9), (7, 127, 33), (13, 256, 65),
                                   (17, 1025, 9)])
def test_integer_extrema_tails_and_threads_match_scalar(oracle, m, k, n):
    i = np.arange(k * n)
    weights = np.where(i % 5 == 0, -127.0, np.where(i % 5 == 1, 127.0, np.where(i % 5 == 2, 0.0,
                                                                                 (i % 31) / 8.0))).astype(np.float32)
    xi = np.arange(m * k)
    x = np.where(xi % 7 == 0, 127.0, np.where(xi % 7 == 1, -127.0, np.where(xi % 7 == 2, 0.0,
                                                                          (xi % 13) - 6.0))).astype(np.float32)
    w = oracle.Matrix(oracle.f32_to_bf16(weights), k, n, 8, 8)
    for threads in (1, 3):
        oracle.set_threads(threads)
        a = w.apply(x, mode=1).reshape(-1)
        b = w.apply(x, mode=0).reshape(-1)
        for r in range(m):
            for c in range(n):
                tot = 0.0
                for g in range(-(-k // GROUP)):
                    end = min(g * GROUP + GROUP, k)
                    xv, wv = x[r * k + g * GROUP: r * k + end], weights[c * k + g * GROUP: c * k + end]
                    qa, sx = quant_ref(xv, 8)
                    qb, sw = quant_ref(wv, 8)
                    tot += float(np.dot(qa, qb)) * float(np.float32(sx * sw))
                assert abs(float(a[r * n + c]) - tot) <= 0.01 + abs(tot) * 1e-6
        assert np.all(np.abs(a - b) <= 0.02 + np.abs(a) * 1e-6)
    oracle.set_threads(0)


# ---------------------------------------------------------------- int8.rs:952-962
def test_invalid_weights_and_nonfinite_activations_are_rejected(oracle):
    with pytest.raises(ValueError):
        oracle.Matrix(np.zeros(0, np.uint16), 0, 1)
    with pytest.raises(ValueError):
        oracle.Matrix(np.array([0x7FC0], np.uint16), 1, 1)
    w = oracle.Matrix(np.zeros(1, np.uint16), 1, 1)
    assert np.isnan(w.apply(f32([np.nan]))[0, 0])
    assert w.apply(f32([0.0]))[0, 0] == 0.0


# ---------------------------------------------------------------- int8.rs:590-643
def test_affine_offsets_match_independent_dequantized_dot_products(oracle):
    k, n = 65, 9
    i = np.arange(k * n)
    vals = np.where((i // k) % 3 == 0, (i // k).astype(np.float32) + 3,
                    ((i * 31 % 97).astype(np.float32) - 48) / np.float32(17) + 9).astype(np.float32)
    bytes_ = oracle.f32_to_bf16(vals)
    G = -(-k // GROUP)
    for simd in (0, 1):
        w = oracle.Matrix(bytes_, k, n, 4, 8, fit=2, simd=simd)
        assert w.bytes() == -(-n // 8) * 8 * G * (GROUP // 2 + 8)
        codes = w.weight_codes().astype(np.float64)
        sc = w.weight_scales().astype(np.float64)
        off = w.weight_offsets().astype(np.float64)
        for m in (1, 15, 16, 17):
            xi = np.arange(m * k)
            x = ((xi * 13 % 255).astype(np.float32) - 127) / np.float32(17) + 3
            x = x.astype(np.float32)
            out = w.apply(x, mode=0)
            values, ascale, _ = w.prepare(x)
            values = values.reshape(m, G * GROUP).astype(np.float64)
            ascale = ascale.reshape(m, G).astype(np.float64)
            for r in range(m):
                for c in range(n):
                    j = np.arange(k)
                    g = j // GROUP
                    weight = codes[c, j] * sc[c, g] + off[c, g]
                    e = float(np.sum(weight * values[r, j] * ascale[r, g]))
                    assert abs(float(out[r, c]) - e) < 1e-3 + abs(e) * 4e-6


# ---------------------------------------------------------------- int8.rs:645-676
@pytest.mark.parametrize("k,n", [(65, 9), (128, 33)])
def test_fitted_q4_signed_scales_and_full_code_range_match_scalar(oracle, k, n):
    i = np.arange(k * n)
    bytes_ = oracle.f32_to_bf16(((i * 37 % 251).astype(np.float32) - 125) / np.float32(31))
    w = oracle.Matrix(bytes_, k, n, 4, 8, fit=1, simd=1)
    assert np.any(w.scales < 0)
    assert np.any(w.weight_codes() == -8)
    for m in (1, 15, 16, 17):
        xi = np.arange(m * k)
        x = (((xi * 13 % 255).astype(np.float32) - 127) / np.float32(17)).astype(np.float32)
        a = w.apply(x, mode=1)
        b = w.apply(x, mode=0)
        assert np.all(np.abs(a - b) < 1e-4 + np.abs(a) * 2e-6)


# ---------------------------------------------------------------- packed.rs:124-161
def test_grouped_codes_and_scale_match_native(oracle):
    i = np.arange(128)
    values = np.where(i < 64, (i - 32) / 16.0, (i - 96) * 8.0).astype(np.float32)
    bytes_ = oracle.bf16_truncate(values)
    for bits, group in [(4, 36), (8, 68)]:
        packed = oracle.packed_pack(bytes_, 1, 128, bits)
        assert packed.size == 2 * group
        for g in range(2):
            v = values[g * 64:(g + 1) * 64]
            scale = oracle.group_scale(v, bits)
            codes = oracle.pack_codes(v, scale, bits)
            p = packed[g * group:(g + 1) * group]
            assert p[group - 4:].tobytes() == np.float32(scale).tobytes()
            for kk in range(64):
                code = ((int(p[kk // 2]) >> (4 * (kk % 2))) & 15) - 8 if bits == 4 else int(np.int8(p[kk]))
                assert code == int(codes[kk])
        decoded = oracle.packed_unpack(packed, bits)
        assert decoded.size == 128
        assert np.isfinite(oracle.packed_project(packed, bits, 128, values, 1)[0])
    assert oracle.packed_size(1, 63, 4) == 0
    assert oracle.packed_size(1, 64, 2) == 0


# ---------------------------------------------------------------- packed.rs:162-208
def test_packed_projection_and_embeddings_match_native(oracle):
    n, k = 67, 128
    i = np.arange(n * k)
    values = np.where(i % 128 >= 64, 0.0, ((i * 23 % 127) - 63) / 32.0).astype(np.float32)
    bytes_ = oracle.bf16_truncate(values)
    j = np.arange(k)
    inp = np.where(j == 0, 127.0, ((j % 9) - 4.0) * 0.5).astype(np.float32)
    for bits in (4, 8):
        packed = oracle.packed_pack(bytes_, n, k, bits)
        native = oracle.Matrix(bytes_, k, n, bits, 8)
        reference = native.apply(inp, mode=1).reshape(-1)
        assert np.array_equal(oracle.packed_project(packed, bits, k, inp, 3).view(np.uint32),
                              reference[:3].view(np.uint32))
        assert np.array_equal(oracle.packed_project(packed, bits, k, inp, n).view(np.uint32),
                              reference.view(np.uint32))
        emb = oracle.Embedding(bytes_, k, bits, simd=0)
        ref = emb.append(5)
        row = oracle.packed_size(1, k, bits)
        decoded = oracle.packed_unpack(packed[5 * row:6 * row], bits)
        assert np.array_equal(decoded.view(np.uint32), ref.view(np.uint32))


# ---------------------------------------------------------------- quantized_rows.rs:117-208
def test_affine_embedding_offsets_and_storage(oracle):
    values = (np.arange(256) / 64.0).astype(np.float32)
    rows = oracle.Embedding(oracle.f32_to_bf16(values), 128, 4, fit=2, simd=0)
    assert rows.bytes() == 256 // 2 + 4 * 8
    for id_ in (1, 0, 1):
        actual = rows.append(id_)
        assert np.all(np.abs(actual - values[id_ * 128:(id_ + 1) * 128]) < 0.04)


def test_fitted_embedding_layout_matches_independent_block_decoding(oracle):
    i = np.arange(256)
    bytes_ = oracle.f32_to_bf16(((i * 37 % 101).astype(np.float32) - 50) / np.float32(37))
    for nf4 in (False, True):
        rows = oracle.Embedding(bytes_, 128, 4, fit=3 if nf4 else 1, simd=0)
        assert rows.bytes() == 256 // 2 + 256 // 64 * 4
        for id_ in (1, 0, 1):
            actual = rows.append(id_)
            for g in range(2):
                v = oracle.bf16_to_f32(bytes_[id_ * 128 + g * 64: id_ * 128 + (g + 1) * 64])
                if nf4:
                    s, codes = oracle.fit_nf4(v)
                    dec = oracle.NF4[codes.astype(np.int64) + 8] * s
                else:
                    s, codes = oracle.fit_mse(v, simd=0)
                    dec = codes.astype(np.float32) * s
                assert np.array_equal(actual[g * 64:(g + 1) * 64].view(np.uint32), dec.astype(np.float32).view(np.uint32))


@pytest.mark.parametrize("bits", [4, 8])
def test_packed_rows_preserve_signs_scales_and_random_access(oracle, bits):
    limit = 7 if bits == 4 else 127
    i = np.arange(3 * 128)
    values = ((i % (2 * limit + 1)) - limit).astype(np.float32)
    rows = oracle.Embedding(oracle.f32_to_bf16(values), 128, bits, simd=1)
    assert rows.bytes() == values.size * bits // 8 + values.size // 64 * 4
    for id_ in (2, 0, 1, 2):
        actual = rows.append(id_)
        assert np.all(np.abs(actual - values[id_ * 128:(id_ + 1) * 128]) <= 0.51)
    with pytest.raises(ValueError):
        oracle.Embedding(np.zeros(1, np.uint16), 1, 4)


# ---------------------------------------------------------------- quantization.rs:304-370
@pytest.mark.parametrize("simd", [0, 1])
def test_affine_preserves_constants_and_fits_offset_grids(oracle, simd):
    for n in (1, 7, 16, 63, 64):
        for v in (0.0, -3.25, 12.0):
            s, b, codes = oracle.fit_affine(np.full(n, v, np.float32), simd)
            assert np.all(codes.astype(np.float32) * s + b == np.float32(v))
        vals = (4 + (np.arange(n) * 15 // max(n - 1, 1)).astype(np.float32) * np.float32(0.25)).astype(np.float32)
        s, b, codes = oracle.fit_affine(vals, simd)
        assert np.all(np.abs(vals - (codes.astype(np.float32) * s + b)) < 1e-5)


@pytest.mark.parametrize("simd", [0, 1])
def test_fitting_reduces_reconstruction_error_and_handles_tails(oracle, simd):
    for n in (1, 7, 8, 31, 63, 64):
        for seed in range(32):
            i = np.arange(n)
            vals = (((i * 137 + seed * 19) % 101).astype(np.float32) - 50).astype(np.float32)
            vals[0] = vals[0] * np.float32(3.7)
            s = oracle.group_scale(vals, 4)
            base = oracle.pack_codes(vals, s, 4)
            fit, codes = oracle.fit_mse(vals, simd)

            def err(q, sc):
                return float(np.sum((vals.astype(np.float64) - q.astype(np.float64) * float(sc)) ** 2))

            assert err(codes, fit) <= err(base, s) + 1e-5
            assert np.all((codes >= -8) & (codes <= 7))
    s, codes = oracle.fit_mse(np.zeros(64, np.float32), simd)
    assert np.isfinite(s)
    assert np.all(codes == 0)


def test_nf4_roundtrips_codebook_and_zero(oracle):
    s, codes = oracle.fit_nf4(oracle.NF4)
    for i, c in enumerate(codes):
        assert abs(oracle.NF4[int(c) + 8] * s - oracle.NF4[i]) < 1e-6
    s, codes = oracle.fit_nf4(np.zeros(16, np.float32))
    assert np.isfinite(s)
    assert np.all(oracle.NF4[codes.astype(np.int64) + 8] == 0)


# ---------------------------------------------------------------- bf16 conversion (half 2.7.1)
def test_bf16_round_to_nearest_even(oracle):
    cases = {
        0x3F800000: 0x3F80,  # 1.0
        0x3F808000: 0x3F80,  # tie, even stays
        0x3F818000: 0x3F82,  # tie, odd rounds up
        0x3F808001: 0x3F81,  # above tie
        0x7F7FFFFF: 0x7F80,  # rounds to inf
        0xFFC00001: 0xFFC0,  # NaN stays NaN
    }
    for src, want in cases.items():
        got = int(oracle.f32_to_bf16(np.array([src], np.uint32).view(np.float32))[0])
        assert got == want, hex(src)
