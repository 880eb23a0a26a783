"""GPU parity of the CUDA kernels against the CPU oracle, through the C ABI.

Bit-exact: activation quantiser, weight packer, packed import/export, row dequantisation, the
tensor-core GEMM and the GEMV path (both accumulation modes).  Tolerance (stated per test):
the fused SwiGLU re-quantisation (exp differs by <= 2 ulp between libm and CUDA) and the f16
attention.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

GROUP = 64


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


def ref_weights(k, n, seed=0, kind="ramp"):
    i = np.arange(k * n)
    if kind == "ramp":  # int8.rs:691-693
        v = ((i * 37 % 257).astype(np.float32) - 128) / np.float32(31)
    else:
        v = np.random.default_rng(seed).normal(0, 0.02, k * n).astype(np.float32)
    return v


def ref_x(m, k, seed=0, kind="ramp"):
    i = np.arange(m * k)
    if kind == "ramp":  # int8.rs:698-700
        return (((i * 13 % 255).astype(np.float32) - 127) / np.float32(17)).astype(np.float32)
    return np.random.default_rng(seed).normal(0, 1, m * k).astype(np.float32)


def dev_bf16(oracle, w, n, k):
    bf = oracle.f32_to_bf16(w).reshape(n, k)
    return bf, torch.from_numpy(bf.view(np.int16)).cuda()


# ------------------------------------------------------------------ quantiser
@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("m,k", [(1, 1), (3, 63), (7, 65), (17, 127), (33, 1025), (256, 1024)])
def test_activation_quantiser_matches_oracle(db, oracle, bits, m, k):
    x = ref_x(m, k, kind="normal") * 3
    w = oracle.Matrix(np.zeros(k, np.uint16), k, 1, 8, bits)
    values, scales, sums = w.prepare(x)
    G = -(-k // GROUP)
    xt = torch.from_numpy(x.reshape(m, k)).cuda()
    for layout in (db.CODES_NATURAL, db.CODES_GEMV, db.CODES_TC):
        codes, sc, s = db.quantize_activations(xt, bits=bits, layout=layout, sums=True)
        nat = torch.empty((m, G * GROUP), dtype=torch.int8, device="cuda")
        # decode to natural order through the library's own converter via the GEMV/TC position maps
        c = codes.cpu().numpy().astype(np.int64)
        if layout == db.CODES_TC:
            perm = np.array([0, 4, 1, 5, 2, 6, 3, 7])
        elif layout == db.CODES_GEMV:
            perm = np.array([0, 2, 4, 6, 1, 3, 5, 7])
        else:
            perm = np.arange(8)
        natural = np.zeros_like(c)
        for b in range(0, G * GROUP, 8):
            natural[:, b + perm] = c[:, b:b + 8]
        del nat
        assert np.array_equal(natural.reshape(-1), values.astype(np.int64)), layout
        assert bits_equal(sc.cpu().numpy()[:, :m].T.reshape(-1), scales)
        assert np.array_equal(s.cpu().numpy()[:, :m].T.reshape(-1), sums)


def test_activation_rounding_at_ties(db, oracle):
    vals = []
    for i in range(-127, 127):
        h = np.float32(i + 0.5)
        vals += [np.nextafter(h, np.float32(-np.inf)), h, np.nextafter(h, np.float32(np.inf))]
    base = np.array(vals, np.float32)
    for s in (1.0, 0.0037, float(np.finfo(np.float32).tiny), 1e30):
        x = (base * np.float32(s)).astype(np.float32)
        x = np.concatenate([x, np.zeros((-x.size) % 64, np.float32)]).reshape(-1, 64)
        codes, sc, _ = db.quantize_activations(torch.from_numpy(x).cuda(), bits=8, layout=db.CODES_NATURAL)
        w = oracle.Matrix(np.zeros(64, np.uint16), 64, 1)
        values, scales, _ = w.prepare(x)
        assert np.array_equal(codes.cpu().numpy().reshape(-1), values)
        assert bits_equal(sc.cpu().numpy()[:, :x.shape[0]].T.reshape(-1), scales)


# ------------------------------------------------------------------ weights
@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("n,k", [(1, 64), (7, 128), (67, 128), (33, 1024), (3072, 1024)])
def test_weight_packer_matches_packed_pack(db, oracle, bits, n, k):
    w = ref_weights(k, n, kind="normal")
    bf, dbf = dev_bf16(oracle, w, n, k)
    codes, scales = db.pack_weights(dbf, bits)
    packed = db.export_packed(codes, scales, n, k, bits).cpu().numpy()
    ref = oracle.packed_pack(bf.reshape(-1), n, k, bits)
    assert np.array_equal(packed, ref)
    c2, s2 = db.import_packed(torch.from_numpy(ref).cuda(), n, k, bits)
    assert torch.equal(c2, codes) and torch.equal(s2, scales)
    # dequantised weights bit-for-bit vs packed::unpack (packed.rs:59-73)
    deq = db.dequant_rows(codes, scales, n, k, bits).cpu().numpy().reshape(-1)
    assert bits_equal(deq, oracle.packed_unpack(ref, bits))


@pytest.mark.parametrize("bits", [4, 8])
def test_weight_packer_ragged_k_matches_matrix_layout(db, oracle, bits):
    for n, k in [(9, 65), (33, 129), (65, 1025)]:
        w = ref_weights(k, n)
        bf, dbf = dev_bf16(oracle, w, n, k)
        codes, scales = db.pack_weights(dbf, bits)
        mat = oracle.Matrix(bf.reshape(-1), k, n, bits, 8)
        G = -(-k // GROUP)
        c = codes.cpu().numpy()
        if bits == 4:
            dense = np.zeros((n, G * GROUP), np.int64)
            dense[:, 0::2] = (c & 15).astype(np.int64) - 8
            dense[:, 1::2] = (c >> 4).astype(np.int64) - 8
        else:
            dense = c.view(np.int8).astype(np.int64)
        assert np.array_equal(dense, mat.weight_codes().astype(np.int64))
        assert bits_equal(scales.cpu().numpy()[:, :n].T, mat.weight_scales())
        assert np.all(scales.cpu().numpy()[:, n:] == 0)


def test_embedding_rows_match_append(db, oracle):
    rows, cols = 300, 256
    w = ref_weights(cols, rows, kind="normal")
    bf, dbf = dev_bf16(oracle, w, rows, cols)
    for bits in (4, 8):
        codes, scales = db.pack_weights(dbf, bits)
        emb = oracle.Embedding(bf.reshape(-1), cols, bits, simd=1)
        ids = np.array([5, 0, 299, 5, 17], np.int32)
        out = db.dequant_rows(codes, scales, rows, cols, bits, torch.from_numpy(ids).cuda()).cpu().numpy()
        for i, r in enumerate(ids):
            assert bits_equal(out[i], emb.append(int(r)))
    with pytest.raises(db.CudaError):
        db.dequant_rows(codes, scales, rows, cols, 8, torch.tensor([300], dtype=torch.int32, device="cuda"))


def test_nonfinite_weight_rejected(db):
    bad = torch.zeros((2, 64), dtype=torch.int16, device="cuda")
    bad[1, 3] = 0x7FC0
    with pytest.raises(db.CudaError):
        db.pack_weights(bad, 4)


# ------------------------------------------------------------------ grouped GEMM
SHAPES = [(1, 1, 1), (3, 63, 7), (7, 65, 9), (9, 129, 33), (15, 65, 9), (16, 65, 9), (17, 127, 32), (33, 1025, 65),
          # webgpu/grouped_q4.rs:227 check shapes (m, n, k) reordered to (m, k, n)
          (1, 64, 7), (5, 128, 67), (65, 256, 33), (7, 192, 11), (3, 128, 5),
          (128, 1024, 128), (200, 512, 300), (1024, 1024, 3072)]


def _gpu_gemm(db, oracle, x, m, k, n, wbits, abits, fused, path):
    w = ref_weights(k, n, kind="ramp" if n * k < 100000 else "normal")
    bf, dbf = dev_bf16(oracle, w, n, k)
    codes, scales = db.pack_weights(dbf, wbits)
    xt = torch.from_numpy(x.reshape(m, k)).cuda()
    if path == "linear":
        y = db.linear(xt, codes, scales, n, wbits, abits, fused)
    else:
        layout = db.CODES_NATURAL if path == "i8" else db.CODES_TC
        a, sa, s = db.quantize_activations(xt, bits=abits, layout=layout)
        y = db.gemm(a, layout, sa, codes, scales, m, n, k, wbits, fused)
    torch.cuda.synchronize()
    assert db.device_error_word() == 0
    mat = oracle.Matrix(bf.reshape(-1), k, n, wbits, abits)
    return y.cpu().numpy(), mat


@pytest.mark.parametrize("path", ["tc", "i8"])
@pytest.mark.parametrize("wb,ab", [(4, 8), (8, 8), (4, 4)])
@pytest.mark.parametrize("m,k,n", SHAPES)
def test_tensor_core_gemm_bit_exact(db, oracle, wb, ab, m, k, n, path):
    x = ref_x(m, k, kind="ramp" if m * k < 100000 else "normal")
    y, mat = _gpu_gemm(db, oracle, x, m, k, n, wb, ab, True, path)
    ref = mat.apply(x, mode=2 if m * n * k > 10 ** 7 else 0)
    assert bits_equal(y, ref), f"max |d| = {np.max(np.abs(y - ref))}"


I8_CONFIGS = [(256, 0, 1), (256, 0, 0), (128, 0, 1), (128, 0, 0), (64, 0, 1), (64, 0, 0), (256, 5, 1), (64, 3, 0),
              (128, 7, 1), (32, 0, 0), (32, 5, 0), (32, 0, 1)]


@pytest.mark.parametrize("m,k,n", [(200, 1000, 300), (1024, 1024, 3072), (257, 130, 129), (384, 2048, 256),
                                   (300, 64, 64), (129, 3072, 1024), (128, 4096, 2560), (37, 200, 70)])
@pytest.mark.parametrize("wb", [4, 8])
def test_i8_tile_configurations_are_bitwise_equal(db, oracle, m, k, n, wb):
    """kind::i8 path: every tile width / pairing / grid cap gives the oracle's bits, for the store
    and the residual (TMA reduce-add) epilogues and both accumulation orders."""
    x = ref_x(m, k, kind="normal")
    bf = oracle.f32_to_bf16(np.random.default_rng(k + n).normal(0, 0.02, (n, k)).astype(np.float32))
    codes, scales = db.pack_weights(torch.from_numpy(bf.view(np.int16)).cuda(), wb)
    a, sa, _ = db.quantize_activations(torch.from_numpy(x.reshape(m, k)).cuda(), bits=8, layout=db.CODES_NATURAL)
    mat = oracle.Matrix(bf.reshape(-1), k, n, wb, 8)
    ref, ref_p = mat.apply(x, mode=0), mat.apply(x, mode=1)
    base = torch.randn(m, n, device="cuda")
    expect_res = (base.cpu().numpy() + ref).astype(np.float32)
    for bn, cap, pair in I8_CONFIGS:
        cfg = db.GemmConfig(bn, cap, pair)
        y = db.gemm(a, db.CODES_NATURAL, sa, codes, scales, m, n, k, wb, True, config=cfg)
        r = db.gemm(a, db.CODES_NATURAL, sa, codes, scales, m, n, k, wb, True, residual=base.clone(), config=cfg)
        p = db.gemm(a, db.CODES_NATURAL, sa, codes, scales, m, n, k, wb, False, config=cfg)
        torch.cuda.synchronize()
        assert db.device_error_word() == 0
        assert bits_equal(y.cpu().numpy(), ref), f"store epilogue differs for config {(bn, cap, pair)}"
        assert bits_equal(r.cpu().numpy(), expect_res), f"residual epilogue differs for config {(bn, cap, pair)}"
        assert bits_equal(p.cpu().numpy(), ref_p), f"portable numerics differ for config {(bn, cap, pair)}"


TILE_CONFIGS = [(0, 0, 0), (64, 0, 0), (128, 0, 1), (128, 16, 0), (128, 7, 1), (64, 3, 0), (256, 0, 0), (256, 5, 0)]


@pytest.mark.parametrize("m,k,n", [(200, 1000, 300), (1024, 1024, 3072), (257, 130, 129), (384, 2048, 256)])
@pytest.mark.parametrize("wb", [4, 8])
def test_tile_configurations_are_bitwise_equal(db, oracle, m, k, n, wb):
    """The tuner's candidate space (checkpoint.rs:279-294): every tile configuration -- tile width,
    persistent grid cap, CTA pairs with M = 256 MMAs -- gives the same bits, equal to the oracle."""
    x = ref_x(m, k, kind="normal")
    bf = oracle.f32_to_bf16(np.random.default_rng(k + n).normal(0, 0.02, (n, k)).astype(np.float32))
    codes, scales = db.pack_weights(torch.from_numpy(bf.view(np.int16)).cuda(), wb)
    a, sa, _ = db.quantize_activations(torch.from_numpy(x.reshape(m, k)).cuda(), bits=8, layout=db.CODES_TC)
    ref = oracle.Matrix(bf.reshape(-1), k, n, wb, 8).apply(x, mode=0)
    base = torch.randn(m, n, device="cuda")
    outs = []
    for bn, cap, pair in TILE_CONFIGS:
        cfg = db.GemmConfig(bn, cap, pair)
        y = db.gemm(a, db.CODES_TC, sa, codes, scales, m, n, k, wb, True, config=cfg)
        r = db.gemm(a, db.CODES_TC, sa, codes, scales, m, n, k, wb, True, residual=base.clone(), config=cfg)
        torch.cuda.synchronize()
        assert db.device_error_word() == 0
        outs.append((y.cpu().numpy(), r.cpu().numpy()))
    assert bits_equal(outs[0][0], ref)
    expect_res = (base.cpu().numpy() + ref).astype(np.float32)
    for (y, r), c in zip(outs, TILE_CONFIGS):
        assert bits_equal(y, outs[0][0]), f"store epilogue differs for config {c}"
        assert bits_equal(r, expect_res), f"residual epilogue differs for config {c}"


@pytest.mark.parametrize("m,k,n", [(7, 65, 9), (65, 256, 33), (256, 1024, 512)])
def test_tensor_core_gemm_portable_mode_bit_exact(db, oracle, m, k, n):
    x = ref_x(m, k)
    y, mat = _gpu_gemm(db, oracle, x, m, k, n, 4, 8, False, "tc")
    assert bits_equal(y, mat.apply(x, mode=1))


@pytest.mark.parametrize("wb", [4, 8])
@pytest.mark.parametrize("m", [1, 2, 3, 4, 5, 8])
@pytest.mark.parametrize("k,n", [(64, 7), (1025, 65), (1024, 3072), (3072, 1024), (9728, 40), (10240, 9)])
def test_gemv_path_bit_exact(db, oracle, wb, m, k, n):
    x = ref_x(m, k, kind="normal")
    for fused, mode in ((True, 0), (False, 1)):
        y, mat = _gpu_gemm(db, oracle, x, m, k, n, wb, 8, fused, "linear")
        assert bits_equal(y, mat.apply(x, mode=mode))


def test_linear_nonfinite_input_gives_nan(db, oracle):
    for m in (1, 40):
        x = ref_x(m, 128)
        x[5] = np.nan
        w = ref_weights(128, 16)
        bf, dbf = dev_bf16(oracle, w, 16, 128)
        codes, scales = db.pack_weights(dbf, 4)
        y = db.linear(torch.from_numpy(x.reshape(m, 128)).cuda(), codes, scales, 16).cpu().numpy()
        assert np.all(np.isnan(y))
        z = db.linear(torch.zeros((m, 128), device="cuda"), codes, scales, 16).cpu().numpy()
        assert np.all(z == 0)


def test_project_packed_matches_packed_project(db, oracle):
    n, k = 67, 128  # packed.rs:163-208
    i = np.arange(n * k)
    values = np.where(i % 128 >= 64, 0.0, ((i * 23 % 127) - 63) / 32.0).astype(np.float32)
    bf = oracle.bf16_truncate(values)
    j = np.arange(k)
    inp = np.where(j == 0, 127.0, ((j % 9) - 4.0) * 0.5).astype(np.float32)
    for bits in (4, 8):
        codes, scales = db.pack_weights(torch.from_numpy(bf.view(np.int16).reshape(n, k)).cuda(), bits)
        y = db.project_packed(torch.from_numpy(inp).cuda(), codes, scales, n, bits).cpu().numpy()
        ref = oracle.packed_project(oracle.packed_pack(bf, n, k, bits), bits, k, inp, n)
        assert bits_equal(y, ref)
    bad = inp.copy()
    bad[3] = np.inf
    with pytest.raises(db.CudaError):
        db.project_packed(torch.from_numpy(bad).cuda(), codes, scales, n, 8)


# ------------------------------------------------------------------ fused MLP
@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("m,f,k", [(67, 192, 256), (256, 512, 1024), (1024, 3072, 1024)])
@pytest.mark.parametrize("layout", ["tc", "i8"])
def test_fused_mlp_matches_unfused_oracle(db, oracle, bits, m, f, k, layout):
    # webgpu/grouped_q4.rs:313-354 shape and generators for the first case
    def weight(seed):
        i = np.arange(f * k)
        return (((i * seed % 251).astype(np.float32) - 125) / np.float32(400)).astype(np.float32)
    x = ((np.arange(m * k) * 29 % 509).astype(np.float32) - 254) / np.float32(97)
    bg, dg = dev_bf16(oracle, weight(37), f, k)
    bu, du = dev_bf16(oracle, weight(53), f, k)
    gc, gs = db.pack_weights(dg, bits)
    uc, us = db.pack_weights(du, bits)
    guc, gus = db.interleave_gate_up(gc, gs, uc, us, f, k, bits)
    lay = db.CODES_NATURAL if layout == "i8" else db.CODES_TC
    a, sa, _ = db.quantize_activations(torch.from_numpy(x.reshape(m, k)).cuda(), bits=8, layout=lay)
    codes, scales = db.mlp(a, sa, guc, gus, m, f, k, bits)
    torch.cuda.synchronize()
    assert db.device_error_word() == 0
    g = oracle.Matrix(bg.reshape(-1), k, f, bits, 8).apply(x, mode=0)
    u = oracle.Matrix(bu.reshape(-1), k, f, bits, 8).apply(x, mode=0)
    h = oracle.silu_mul(g, u)
    values, ref_scales, _ = oracle.Matrix(np.zeros(f, np.uint16), f, 1).prepare(h)
    c = codes.cpu().numpy().astype(np.int64)
    if layout == "i8":
        natural = c
    else:
        perm = np.array([0, 4, 1, 5, 2, 6, 3, 7])
        natural = np.zeros_like(c)
        for b in range(0, f, 8):
            natural[:, b + perm] = c[:, b:b + 8]
    diff = np.abs(natural.reshape(-1) - values.astype(np.int64))
    # exp() of CUDA and libm differ by <= 2 ulp; a code may flip only at a rounding boundary
    assert diff.max() <= 1 and np.count_nonzero(diff) <= max(2, diff.size // 10000)
    rel = np.abs(scales.cpu().numpy()[:, :m].T.reshape(-1) - ref_scales) / ref_scales
    assert rel.max() <= 4e-7


# ------------------------------------------------------------------ attention
# Key-tile counts 1 to 16 (tiles of 128 keys: even and odd counts, ragged last tiles), GQA ratios
# 1, 2 and 4, and sharper softmaxes (scale 0.25: scores with a standard deviation of ~2.8).
@pytest.mark.parametrize("t,hq,hk,scale", [(1, 2, 1, None), (65, 4, 2, None), (128, 2, 2, None),
                                           (129, 2, 1, None), (200, 4, 4, None), (300, 8, 2, None),
                                           (300, 4, 1, 0.25), (1024, 16, 8, None), (1000, 4, 2, 0.25),
                                           (2048, 4, 1, 0.25)])
def test_attention_matches_oracle(db, oracle, t, hq, hk, scale):
    rng = np.random.default_rng(t)
    q = rng.normal(0, 1, (t, hq, 128)).astype(np.float16)
    k = rng.normal(0, 1, (t, hk, 128)).astype(np.float16)
    v = rng.normal(0, 1, (t, hk, 128)).astype(np.float16)
    out = db.attention(torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), hq, hk,
                       scale)
    assert db.device_error_word() == 0
    ref = oracle.attention(q.astype(np.float32), k.astype(np.float32), v.astype(np.float32), hq, hk, 128, scale)
    o = out.cpu().numpy().reshape(-1)
    r = ref.reshape(-1)
    # f16 probabilities (11-bit mantissa) into an f32 accumulator: error ~1e-3 of the output RMS
    assert np.max(np.abs(o - r)) <= 5e-3 * np.sqrt(np.mean(r ** 2)) + 1e-6


def decoder_attention_ref(q, k, v, kp, vp, items, hq, hk, causal, scale):
    """float64 restatement: each item's rows see the prefix keys, then their own keys (causal: up
    to themselves); scale * q.k, softmax, P.v per head."""
    R = q.shape[0]
    T = R // items
    out = np.zeros((R, hq * 128))
    for b in range(items):
        rows = slice(b * T, (b + 1) * T)
        for h in range(hq):
            kh = h // (hq // hk)
            keys = np.concatenate([kp[:, kh], k[rows, kh]]) if kp is not None else k[rows, kh]
            vals = np.concatenate([vp[:, kh], v[rows, kh]]) if vp is not None else v[rows, kh]
            s = q[rows, h] @ keys.T * scale
            if causal:
                P = keys.shape[0] - T  # own key j sits at column P + j
                s[(np.arange(keys.shape[0])[None, :] - P) > np.arange(T)[:, None]] = -np.inf
            s -= s.max(axis=1, keepdims=True)
            p = np.exp(s)
            out[rows, h * 128:(h + 1) * 128] = (p / p.sum(axis=1, keepdims=True)) @ vals
    return out


# (items, T, P, causal, Hq, Hk, scale): C5-shaped continuations (4 x 32 after 512), the prefix pass
# (causal, no prefix, many tiles), ragged prefixes and items, single-token decode steps, GQA 1/2/4.
@pytest.mark.parametrize("items,t,p,causal,hq,hk,scale", [
    (4, 32, 512, 1, 8, 2, None), (1, 300, 0, 1, 4, 2, None), (3, 17, 100, 1, 4, 4, 0.25), (2, 129, 1, 0, 4, 1, None),
    (1, 1, 1, 1, 2, 1, None), (5, 1, 300, 1, 4, 2, 0.25), (1, 1000, 0, 1, 4, 2, None), (2, 200, 257, 0, 2, 2, None)])
def test_decoder_attention_matches_reference(db, items, t, p, causal, hq, hk, scale):
    rng = np.random.default_rng(items * 1000 + t + p)
    q = rng.normal(0, 1, (items * t, hq, 128)).astype(np.float16)
    k = rng.normal(0, 1, (items * t, hk, 128)).astype(np.float16)
    v = rng.normal(0, 1, (items * t, hk, 128)).astype(np.float16)
    kp = rng.normal(0, 1, (p, hk, 128)).astype(np.float16) if p else None
    vp = rng.normal(0, 1, (p, hk, 128)).astype(np.float16) if p else None
    cu = lambda a: torch.from_numpy(a).cuda() if a is not None else None
    out = db.attention_decoder(cu(q), cu(k), cu(v), items, hq, hk, cu(kp), cu(vp), bool(causal), scale)
    assert db.device_error_word() == 0
    s = (1.0 / 128 ** 0.5) if scale is None else scale
    f64 = lambda a: a.astype(np.float64) if a is not None else None
    ref = decoder_attention_ref(f64(q), f64(k), f64(v), f64(kp), f64(vp), items, hq, hk, causal, s)
    o = out.cpu().numpy()
    assert np.max(np.abs(o - ref)) <= 5e-3 * np.sqrt(np.mean(ref ** 2)) + 1e-6
    # an item's result does not depend on the other items of the batch
    last = db.attention_decoder(cu(q[-t:]), cu(k[-t:]), cu(v[-t:]), 1, hq, hk, cu(kp), cu(vp), bool(causal), scale)
    assert np.array_equal(last.cpu().numpy().view(np.uint32), o[-t:].view(np.uint32))
