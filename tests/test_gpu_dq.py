"""GPU parity of the dequantised-operand GEMM (DB_CODES_DQ: weights unpacked to f16, tcgen05 kind::f16,
f32 accumulation over the whole K) against the CPU oracle, through the C ABI.

The reference CPU path folds exact per-group integer dots with the group scales (int8.rs:526-585);
this path multiplies f16(code * scale) operands instead, the numerics of the reference's WGSL GEMMs.
Tolerance, as the contract states it: max |y - y_ref| <= 2e-3 * rms(y_ref) against the oracle.
Two exact checks pin what the kernels compute: the DQ activation layout is f16(code * scale) of the
oracle's own codes and scales, bit for bit; the GEMM equals the f64 product of the dequantised
operands within f32 accumulation error (2^-16 of the sum of |terms|).  Every tile configuration
gives the same bits (store and residual epilogues).
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

GROUP = 64
TOL_RMS = 2e-3


@pytest.fixture(scope="module")
def db():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import decisive_b200 as d
    d.load()
    return d


def bits_equal(a, b):
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


def _inputs(oracle, m, k, n, seed=0):
    rng = np.random.default_rng(seed + 7 * k + n)
    x = rng.normal(0, 1, (m, k)).astype(np.float32)
    bf = oracle.f32_to_bf16(rng.normal(0, 0.02, (n, k)).astype(np.float32)).reshape(n, k)
    return x, bf


def _dequantised_weights(codes, scales, n, k, wb):
    """Host restatement of the unpack pass: fma(code, s_hi, f16(code * s_lo)) rounded to f16, with
    s_hi = f16(scale), s_lo = f16(scale - s_hi); natural k order, [n, Kp]."""
    c = codes.cpu().numpy()
    Kp = -(-k // GROUP) * GROUP
    if wb == 4:
        q = np.empty((n, Kp), np.int32)
        q[:, 0::2] = (c & 15).astype(np.int32) - 8
        q[:, 1::2] = (c >> 4).astype(np.int32) - 8
    else:
        q = c.view(np.int8).astype(np.int32)
    s32 = np.repeat(scales.cpu().numpy()[:, :n].T, GROUP, axis=1)  # [n, Kp]
    hi = s32.astype(np.float16)
    lo = (s32 - hi.astype(np.float32)).astype(np.float16)
    cc = q.astype(np.float16)
    t = cc * lo  # exact product in f32, one rounding to f16
    return (cc.astype(np.float64) * hi.astype(np.float64) + t.astype(np.float64)).astype(np.float16)


SHAPES = [(1, 1, 1), (3, 63, 7), (7, 65, 9), (65, 256, 33), (128, 128, 1024), (200, 1000, 300), (257, 130, 129),
          (1024, 1024, 3072), (128, 4096, 2560), (1024, 3072, 1024), (384, 2048, 256)]


@pytest.mark.parametrize("wb", [4, 8])
@pytest.mark.parametrize("m,k,n", SHAPES)
def test_dq_gemm_within_tolerance_of_oracle(db, oracle, m, k, n, wb):
    x, bf = _inputs(oracle, m, k, n)
    codes, scales = db.pack_weights(torch.from_numpy(bf.view(np.int16)).cuda(), wb)
    a, _, _ = db.quantize_activations(torch.from_numpy(x).cuda(), bits=8, layout=db.CODES_DQ)
    y = db.gemm(a, db.CODES_DQ, None, codes, scales, m, n, k, wb)
    torch.cuda.synchronize()
    assert db.device_error_word() == 0
    y = y.cpu().numpy()
    ref = oracle.Matrix(bf.reshape(-1), k, n, wb, 8).apply(x, mode=2 if m * n * k > 10 ** 7 else 0)
    rms = float(np.sqrt(np.mean(ref.astype(np.float64) ** 2)))
    err = float(np.max(np.abs(y.astype(np.float64) - ref)))
    print(f"dq max|d|/rms m={m} k={k} n={n} w{wb}: {err / max(rms, 1e-30):.3e}")
    assert err <= TOL_RMS * rms, f"max |d| = {err}, rms = {rms}"
    # what the kernels compute: the f64 product of the dequantised operands, up to f32 accumulation
    ad = a.cpu().numpy().astype(np.float64)
    wd = _dequantised_weights(codes, scales, n, k, wb).astype(np.float64)
    model = ad @ wd.T
    bound = 2.0 ** -16 * (np.abs(ad) @ np.abs(wd).T) + 1e-30
    assert np.all(np.abs(y - model) <= bound), f"max |y - model| = {np.max(np.abs(y - model))}"


@pytest.mark.parametrize("m,k", [(1, 1), (7, 65), (33, 1025), (256, 1024)])
def test_dq_activation_layout_is_dequantised_oracle_codes(db, oracle, m, k):
    """DB_CODES_DQ = f16(code * scale) of the reference quantiser's codes and scales, bit for bit, with
    zero padding up to Kp (a zero code is +0)."""
    x = np.random.default_rng(m + k).normal(0, 3, (m, k)).astype(np.float32)
    values, scales, _ = oracle.Matrix(np.zeros(k, np.uint16), k, 1, 8, 8).prepare(x.reshape(-1))
    G = -(-k // GROUP)
    codes = np.asarray(values, np.int8).reshape(m, G * GROUP).astype(np.float32)
    sa = np.asarray(scales, np.float32).reshape(m, G)
    expect = (codes * np.repeat(sa, GROUP, axis=1)).astype(np.float16)
    a, _, _ = db.quantize_activations(torch.from_numpy(x).cuda(), bits=8, layout=db.CODES_DQ)
    assert np.array_equal(a.cpu().numpy().view(np.uint16), expect.view(np.uint16))


DQ_CONFIGS = [(0, 0, 0), (256, 0, 0), (128, 0, 0), (64, 0, 0), (256, 5, 0), (128, 7, 0), (64, 3, 0), (64, 1, 0),
              (256, 0, 1), (128, 0, 1), (64, 0, 1), (256, 6, 1), (64, 3, 1)]


@pytest.mark.parametrize("m,k,n", [(200, 1000, 300), (1024, 1024, 3072), (257, 130, 129), (129, 3072, 1024),
                                   (37, 200, 70)])
@pytest.mark.parametrize("wb", [4, 8])
def test_dq_tile_configurations_are_bitwise_equal(db, oracle, m, k, n, wb):
    """Every tile width, grid cap and CTA pairing (M = 256 MMAs over two CTAs) gives the same bits,
    for the store and the residual (TMA reduce-add: y = base + acc, one f32 rounding) epilogues."""
    x, bf = _inputs(oracle, m, k, n, seed=1)
    codes, scales = db.pack_weights(torch.from_numpy(bf.view(np.int16)).cuda(), wb)
    a, _, _ = db.quantize_activations(torch.from_numpy(x).cuda(), bits=8, layout=db.CODES_DQ)
    base = torch.randn(m, n, device="cuda")
    first = None
    for bn, cap, pair in DQ_CONFIGS:
        cfg = db.GemmConfig(bn, cap, pair)
        y = db.gemm(a, db.CODES_DQ, None, codes, scales, m, n, k, wb, config=cfg)
        r = db.gemm(a, db.CODES_DQ, None, codes, scales, m, n, k, wb, residual=base.clone(), config=cfg)
        torch.cuda.synchronize()
        assert db.device_error_word() == 0
        y, r = y.cpu().numpy(), r.cpu().numpy()
        if first is None:
            first = y
        assert bits_equal(y, first), f"store epilogue differs for config {(bn, cap, pair)}"
        assert bits_equal(r, (base.cpu().numpy() + y).astype(np.float32)), f"residual differs for {(bn, cap, pair)}"


def test_dq_nonfinite_input_gives_nan(db, oracle):
    x, bf = _inputs(oracle, 64, 256, 128)
    x[3, 17] = np.inf
    codes, scales = db.pack_weights(torch.from_numpy(bf.view(np.int16)).cuda(), 4)
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    a, _, _ = db.quantize_activations(torch.from_numpy(x).cuda(), bits=8, layout=db.CODES_DQ, nonfinite=flag)
    y = db.gemm(a, db.CODES_DQ, None, codes, scales, 64, 128, 256, 4, nonfinite=flag)
    torch.cuda.synchronize()
    assert int(flag.item()) == 1 and bool(torch.isnan(y).all())
