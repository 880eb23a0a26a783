"""GPU parity of the Decima int8 path (C4 scheme, src/models/decima/int8.rs) against the CPU
oracle, through the C ABI: the block quantiser (round half away from zero of x / scale) for
weights and activations, and the W8A8 grouped GEMM in blocks of 32 and 64 with the bias epilogue,
in the AVX2 (fma) and portable accumulation orders.  All comparisons are bit-exact."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def db():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import decisive_b200 as d
    d.load()
    return d


@pytest.fixture(scope="module")
def oracle():
    from oracle import oracle as o
    o.lib()
    return o


def bits_equal(a, b):
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


def x_pattern(m, k):
    # decima/int8.rs tails_extrema_zero_and_outliers_match_portable: zeros, outliers, sines
    i = np.arange(m * k)
    return np.where(i % 11 == 0, 0., np.where(i % 7 == 0, 70., np.sin(i.astype(np.float32) * np.float32(0.31)))
                    ).astype(np.float32).reshape(m, k)


@pytest.mark.parametrize("block", [16, 32, 64, 128])
@pytest.mark.parametrize("m,k", [(1, 1), (3, 33), (7, 127), (130, 96), (257, 768)])
def test_decima_activation_quantiser_bit_exact(db, oracle, block, m, k):
    x = x_pattern(m, k) * np.float32(0.9)
    codes, scales, flag = db.decima_quantize_activations(torch.from_numpy(x).cuda(), block, db.CODES_NATURAL)
    ref_c, ref_s = oracle.decima_quantize_rows(x, block)
    g = ref_s.shape[1]
    got = codes.cpu().numpy()
    assert np.array_equal(got[:, :g * block][:, :k], ref_c[:, :k])
    assert not np.any(got[:, k:])  # padding codes are 0
    assert bits_equal(scales.cpu().numpy()[:g, :m].T, ref_s)
    assert int(flag.item()) == 0


@pytest.mark.parametrize("block", [32, 64])
@pytest.mark.parametrize("n,k", [(9, 33), (64, 768), (130, 3072), (768, 100)])
def test_decima_weight_quantiser_bit_exact(db, oracle, block, n, k):
    v = np.random.default_rng(n + k).normal(0, 0.05, (n, k)).astype(np.float32)
    v[0, :min(k, 5)] = [-127., 127., 0., 1e-39, 3.][:min(k, 5)]
    codes, scales = db.decima_quantize_weights(torch.from_numpy(v).cuda(), block)
    ref = oracle.DecimaMatrix(v, block)
    g = ref.scales.shape[1]
    assert np.array_equal(codes.cpu().numpy().view(np.int8)[:, :k], ref.codes[:, :k])
    assert bits_equal(scales.cpu().numpy()[:g, :n].T, ref.scales)


@pytest.mark.parametrize("block", [32, 64])
@pytest.mark.parametrize("m,n,k", [(1, 9, 33), (7, 17, 127), (129, 9, 33), (200, 300, 768), (513, 768, 3072),
                                   (256, 1024, 96)])
def test_decima_linear_bit_exact(db, oracle, block, m, n, k):
    x = x_pattern(m, k)
    v = np.where(np.arange(n * k) % 3 == 0, -127., 127.).astype(np.float32).reshape(n, k)
    v = (v * np.random.default_rng(k).uniform(0.001, 0.02, (n, k))).astype(np.float32)
    bias = np.random.default_rng(n).normal(0, 1, n).astype(np.float32)
    ref = oracle.DecimaMatrix(v, block)
    codes, scales = db.decima_quantize_weights(torch.from_numpy(v).cuda(), block)
    xd = torch.from_numpy(x).cuda()
    bd = torch.from_numpy(bias).cuda()
    for fused, mode in ((True, 0), (False, 1)):
        y = db.decima_linear(xd, codes, scales, n, block, fused, bd).cpu().numpy()
        assert bits_equal(y, ref.apply(x, bias=bias, mode=mode)), (fused, np.max(np.abs(y - ref.apply(x, bias=bias, mode=mode))))
        y0 = db.decima_linear(xd, codes, scales, n, block, fused, None).cpu().numpy()
        assert bits_equal(y0, ref.apply(x, mode=mode))  # sum + 0 (a -0 sum becomes +0)
    torch.cuda.synchronize()
    assert db.device_error_word() == 0


def test_decima_nonfinite_input_gives_nan_and_bias_only(db):
    # decima/int8.rs invalid_and_nonfinite_values_are_not_hidden
    codes, scales = db.decima_quantize_weights(torch.zeros((1, 1), device="cuda"), 32)
    y = db.decima_linear(torch.tensor([[float("inf")]], device="cuda"), codes, scales, 1, 32)
    assert torch.isnan(y).all()
    y = db.decima_linear(torch.zeros((1, 1), device="cuda"), codes, scales, 1, 32, True,
                         torch.tensor([2.0], device="cuda"))
    assert y.item() == 2.0
    with pytest.raises(Exception):
        db.decima_quantize_weights(torch.tensor([[float("nan")]], device="cuda"), 32)
    with pytest.raises(Exception):
        db.decima_linear(torch.zeros((1, 1), device="cuda"), codes, scales, 1, 16)  # GEMM takes 32 or 64


# ------------------------------------------------------------------ Weights mode (W8A32)
@pytest.mark.parametrize("block", [32, 64, 128])
@pytest.mark.parametrize("m,n,k", [(1, 9, 33), (7, 17, 127), (65, 70, 96), (200, 300, 768), (130, 768, 3072)])
def test_decima_w8a32_bit_exact(db, oracle, block, m, n, k):
    """Matrix::apply_with_rows in Weights mode: f32 activations against the int8 weight codes, in
    the AVX2 order (decoded weights, one fma chain over k: decima/int8/weights_x86.rs) and the
    portable order (per-block dot, then sum += dot * scale: decima/int8.rs:384-407)."""
    x = x_pattern(m, k)
    v = (np.random.default_rng(k + n).normal(0, 0.05, (n, k))).astype(np.float32)
    bias = np.random.default_rng(n).normal(0, 1, n).astype(np.float32)
    ref = oracle.DecimaMatrix(v, block, weights_only=True)
    codes, scales = db.decima_quantize_weights(torch.from_numpy(v).cuda(), block)
    xd = torch.from_numpy(x).cuda()
    bd = torch.from_numpy(bias).cuda()
    for fused, mode in ((True, 0), (False, 1)):
        y = db.decima_linear_w8a32(xd, codes, scales, n, block, fused, bd).cpu().numpy()
        want = ref.apply(x, bias=bias, mode=mode)
        assert bits_equal(y, want), (fused, np.max(np.abs(y - want)))
        y0 = db.decima_linear_w8a32(xd, codes, scales, n, block, fused, None).cpu().numpy()
        assert bits_equal(y0, ref.apply(x, mode=mode))


def test_decima_w8a32_nonfinite_and_blocks(db):
    codes, scales = db.decima_quantize_weights(torch.ones((3, 40), device="cuda"), 32)
    x = torch.ones((2, 40), device="cuda")
    x[1, 7] = float("nan")
    assert torch.isnan(db.decima_linear_w8a32(x, codes, scales, 3, 32)).all()
    y = db.decima_linear_w8a32(torch.ones((2, 40), device="cuda"), codes, scales, 3, 32)
    assert torch.equal(y, torch.full((2, 3), 40.0, device="cuda"))
    c16, s16 = db.decima_quantize_weights(torch.ones((3, 40), device="cuda"), 16)
    with pytest.raises(Exception):
        db.decima_linear_w8a32(torch.ones((2, 40), device="cuda"), c16, s16, 3, 16)
