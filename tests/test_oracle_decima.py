"""Pins the Decima int8 oracle (oracle_decima_*) to the reference's own unit tests for
src/models/decima/int8.rs (read as text; the Rust crate cannot be built here) and to an independent
numpy restatement of its quantiser: blocks of 16/32/64/128, scale = max|x|/127 (at least
f32::MIN_POSITIVE), codes = round-half-away-from-zero(x / scale) with true division, clamped to
+-127 (int8.rs:413-418); W8A8 apply in the AVX2 order (int8.rs:459-498) and the portable order
(int8.rs:380-420); y = sum + bias (or + 0)."""
import numpy as np
import pytest

from oracle import oracle

FLT_MIN = np.float32(np.finfo(np.float32).tiny)


def np_decima_quantize_rows(x, block):
    x = np.asarray(x, np.float32)
    rows, cols = x.shape
    groups = -(-cols // block)
    codes = np.zeros((rows, groups * block), np.int8)
    scales = np.zeros((rows, groups), np.float32)
    for g in range(groups):
        sl = x[:, g * block:min((g + 1) * block, cols)]
        s = np.maximum(np.max(np.abs(sl), axis=1) / np.float32(127), FLT_MIN).astype(np.float32)
        q = (sl / s[:, None]).astype(np.float32).astype(np.float64)   # f32 division, then exact rounding
        r = np.sign(q) * np.floor(np.abs(q) + 0.5)
        codes[:, g * block:g * block + sl.shape[1]] = np.clip(r, -127, 127).astype(np.int8)
        scales[:, g] = s
    return codes, scales


def test_rounding_is_half_away_from_zero_with_true_division():
    # pack_x86.rs vector_rounding_and_scales_match_scalar_bitwise: ties i + 0.5, their neighbours
    vals = [-127., 127., 0., -0., float(FLT_MIN), -float(FLT_MIN)]
    for i in range(-127, 127):
        h = np.float32(i + 0.5)
        vals += [float(np.nextafter(h, np.float32(-np.inf))), float(h), float(np.nextafter(h, np.float32(np.inf)))]
    for v in vals:
        q = oracle.lib().oracle_decima_quantize(np.float32(v), np.float32(1.0))
        t = np.float64(np.float32(v))
        expect = int(np.clip(np.sign(t) * np.floor(abs(t) + 0.5), -127, 127))
        assert q == expect, v
    rng = np.random.default_rng(4)
    bits = (np.arange(4096, dtype=np.uint64) * 747796405 + 2891336453) & 0xFF7FFFFF
    x = bits.astype(np.uint32).view(np.float32).reshape(64, 64)
    x = np.where(np.isfinite(x), x, 0).astype(np.float32)
    for block in (16, 32, 64, 128):
        c, s = oracle.decima_quantize_rows(x, block)
        c2, s2 = np_decima_quantize_rows(x, block)
        assert np.array_equal(s.view(np.uint32), s2.view(np.uint32))
        assert np.array_equal(c, c2)
    y = rng.normal(0, 3, (9, 77)).astype(np.float32)
    for block in (16, 32, 64, 128):
        c, s = oracle.decima_quantize_rows(y, block)
        c2, s2 = np_decima_quantize_rows(y, block)
        assert np.array_equal(c, c2) and np.array_equal(s, s2)


def test_imported_quantization_values_and_outputs():
    # int8.rs tests::imported_quantization_preserves_packed_values_scales_and_outputs
    n, k = 11, 64
    values = ((np.arange(n * k) * 17 % 129).astype(np.float32) - 64) / np.float32(65)
    quantized, scales = [], []
    for group in values.reshape(-1, 32):
        s = oracle.lib().oracle_decima_scale(np.ascontiguousarray(group).ctypes.data_as(oracle._f), 32)
        scales.append(np.float32(s))
        quantized += [oracle.lib().oracle_decima_quantize(np.float32(v), np.float32(s)) for v in group]
    m = oracle.DecimaMatrix(values.reshape(n, k), 32)
    assert np.array_equal(m.codes.reshape(-1), np.array(quantized, np.int8))
    assert np.array_equal(m.scales.reshape(-1), np.array(scales, np.float32))
    x = np.sin(np.arange(7 * k, dtype=np.float32) * np.float32(0.3)).astype(np.float32)
    for mode in (0, 1):
        y = m.apply(x, mode=mode)
        assert y.shape == (7, n) and np.all(np.isfinite(y))


@pytest.mark.parametrize("m,n,k", [(1, 1, 1), (3, 11, 33), (7, 17, 127), (8, 16, 64), (127, 9, 33),
                                   (128, 9, 33), (129, 9, 33), (511, 9, 33), (512, 9, 33), (513, 9, 33)])
def test_tails_extrema_zero_and_outliers(m, n, k):
    # int8.rs tests::tails_extrema_zero_and_outliers_match_portable
    i = np.arange(m * k)
    x = np.where(i % 11 == 0, 0., np.where(i % 7 == 0, 70., np.sin(i.astype(np.float32) * np.float32(0.31)))).astype(np.float32)
    v = np.where(np.arange(n * k) % 3 == 0, -127., 127.).astype(np.float32).reshape(n, k)
    for block in (16, 32, 64, 128):
        mat = oracle.DecimaMatrix(v, block)
        y = mat.apply(x, mode=1)
        z = mat.apply(x, mode=0)
        assert np.all(np.isfinite(y))
        assert np.all(np.abs(y - z) <= 0.02 + np.abs(y) * 1e-5)
        # the integer dot per block and the scale product are exact restatements: recompute in numpy
        a, sa = np_decima_quantize_rows(x.reshape(m, k), block)
        g = a.shape[1] // block
        dots = np.einsum("mgk,ngk->mng", a.reshape(m, g, block).astype(np.int64),
                         mat.codes.reshape(n, g, block).astype(np.int64))
        ref = np.zeros((m, n), np.float32)
        for gg in range(g):
            ref = (ref + dots[:, :, gg].astype(np.float32) * (mat.scales[None, :, gg] * sa[:, None, gg])).astype(np.float32)
        assert np.array_equal((ref + np.float32(0)).view(np.uint32), y.view(np.uint32))


def test_invalid_and_nonfinite_values_are_not_hidden():
    # int8.rs tests::invalid_and_nonfinite_values_are_not_hidden
    with pytest.raises(ValueError):
        oracle.DecimaMatrix(np.array([[np.nan]], np.float32), 32)
    with pytest.raises(ValueError):
        oracle.DecimaMatrix(np.array([[1.]], np.float32), 3)
    q = oracle.DecimaMatrix(np.array([[0.]], np.float32), 32)
    assert np.isnan(q.apply(np.array([np.inf], np.float32))[0, 0])
    assert q.apply(np.array([0.], np.float32), bias=np.array([2.], np.float32))[0, 0] == 2.0
