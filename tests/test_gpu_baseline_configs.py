"""Parity at the BASELINE configurations' own inputs and dimensions.

C1  the single W4A8 GEMM on config 1's exact inputs: activations f16 N(0,1) from seed 0
    [1024, 1024], weights f32 N(0,0.02) from seed 1 [N=3072, K=1024] rounded to bf16 (RNE) and
    quantised Q4 g64.  Dequantised weights bitwise equal to packed::unpack (packed.rs:59-73); the
    output bitwise equal to the oracle (int8.rs:526-585 numerics) and, as the north-star bound,
    within 2e-3 x RMS of it.
C2  all 28 layers of the Pplx-shaped encoder at 1024 tokens against the composed oracle:
    pooled cosine >= 0.9999 (the north-star bound for final embeddings), with the exact grouped
    GEMMs and with the dequantised ones (DB_CODES_DQ).
C4  the Decima-shaped encoder at its real width (hidden 768, 12 heads, FFN 3072, vocab 128100,
    blocks of 32), 2 layers, one 384 + 32-token sequence: pooled cosine >= 0.9999.
C5  the Qwen3-4B-shaped decoder at its real width (hidden 2560, 32q/8kv x 128, FFN 9728), 2
    layers, a 512-token prefix and 4 continuations of 32 tokens: per-token cosine >= 0.999 and
    continuation-mean cosine >= 0.9999 against one causal oracle pass over prefix + continuation,
    with the exact and with the dequantised projections.
"""
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


def cosine(a, b):
    a, b = a.astype(np.float64).ravel(), b.astype(np.float64).ravel()
    return float(a @ b / np.linalg.norm(a) / np.linalg.norm(b))


def bits_equal(a, b):
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_c1_exact_inputs(db, oracle):
    m, k, n = 1024, 1024, 3072
    x16 = np.random.default_rng(0).normal(0, 1, (m, k)).astype(np.float16)
    w32 = np.random.default_rng(1).normal(0, 0.02, (n, k)).astype(np.float32)
    bf = oracle.f32_to_bf16(w32)
    codes, scales = db.pack_weights(torch.from_numpy(bf.view(np.int16)).cuda(), 4)
    # dequantised weights: bitwise packed::unpack of the reference's packed rows
    ref_packed = oracle.packed_pack(bf.reshape(-1), n, k, 4)
    deq = db.dequant_rows(codes, scales, n, k, 4).cpu().numpy().reshape(-1)
    assert bits_equal(deq, oracle.packed_unpack(ref_packed, 4))
    # the GEMM through the public projection call (f16 activations quantised on the device)
    xt = torch.from_numpy(x16).cuda()
    a, sa, _ = db.quantize_activations(xt, bits=8, layout=db.CODES_TC)
    y = db.gemm(a, db.CODES_TC, sa, codes, scales, m, n, k, 4, True).cpu().numpy()
    torch.cuda.synchronize()
    assert db.device_error_word() == 0
    ref = oracle.Matrix(bf.reshape(-1), k, n, 4, 8).apply(x16.astype(np.float32), mode=2)
    assert bits_equal(y, ref), f"max |d| = {np.max(np.abs(y - ref))}"
    rms = float(np.sqrt(np.mean(ref.astype(np.float64) ** 2)))
    assert float(np.max(np.abs(y.astype(np.float64) - ref))) <= 2e-3 * rms


C2_CFG = dict(layers=28, hidden=1024, q_heads=16, kv_heads=8, head_dim=128, ffn=3072, vocab=151936, weight_bits=4)


@pytest.fixture(scope="module")
def c2_oracle(db, oracle):
    """The synthetic C2 weights, 1024 token ids and the composed oracle's pooled embedding."""
    model = db.Model.synthetic(db.EncoderConfig(**C2_CFG), seed=11)
    D, F, L = 1024, 3072, 28
    shapes = {"q": (2048, D), "k": (1024, D), "v": (1024, D), "o": (D, 2048), "gate": (F, D), "up": (F, D),
              "down": (D, F)}
    w = {"embedding": model.synthetic_weight("embedding")}
    for name, shape in shapes.items():
        w[name] = [model.synthetic_weight(name, l).reshape(shape) for l in range(L)]
    for name, size in (("input_norm", D), ("post_norm", D), ("q_norm", 128), ("k_norm", 128)):
        w[name] = [np.ones(size, np.float32) for _ in range(L)]
    w["final_norm"] = np.ones(D, np.float32)
    model.close()
    ids = np.random.default_rng(2).integers(0, C2_CFG["vocab"], 1024).astype(np.int32)
    return ids, oracle.Encoder(C2_CFG, w).forward(ids, mode=2)


def test_c2_all_28_layers_match_oracle(db, c2_oracle):
    ids, want = c2_oracle
    model = db.Model.synthetic(db.EncoderConfig(**C2_CFG), seed=11)
    got = model.predict(ids).response
    model.close()
    assert cosine(got, want) >= 0.9999, cosine(got, want)


def test_c2_dequantised_mode_matches_oracle(db, c2_oracle):
    """The same 28 layers with the dequantised projections (f16(code * scale) operands, full-K f32
    accumulation, separate SwiGLU re-quantisation): pooled cosine >= 0.9999 against the oracle's
    exact grouped fold, and repeatable bit for bit."""
    ids, want = c2_oracle
    model = db.Model.synthetic(db.EncoderConfig(**C2_CFG), seed=11)
    model.set_code_layout(db.CODES_DQ)
    got = model.predict(ids).response
    again = model.predict(ids).response
    model.close()
    assert np.array_equal(got.view(np.uint32), again.view(np.uint32))
    assert cosine(got, want) >= 0.9999, cosine(got, want)


def test_c4_full_width_matches_oracle(db):
    """BASELINE config 4 dimensions (768 hidden, 12 heads, FF 3072, vocab 128100, W8A8 blocks of
    32) on one request as the config states it: a 384-token state and 8 choices of U(16..48)
    tokens, scored as 8 packed state+choice sequences into 3-way logits."""
    from test_gpu_bert import check_score
    cfg = dict(layers=2, hidden=768, heads=12, ffn=3072, vocab=128100, max_positions=512, block=32, eps=1e-12)
    seed, std = 3, 0.05
    model = db.BertModel(db.BertConfig(**cfg), seed=seed, std=std)
    rng = np.random.default_rng(4)
    state = rng.integers(0, cfg["vocab"], 384).astype(np.int32)
    choices = [rng.integers(0, cfg["vocab"], int(rng.integers(16, 49))).astype(np.int32) for _ in range(8)]
    check_score(db, model, cfg, seed, std, state, choices, oracle_seqs=(0, 5))
    model.close()


@pytest.mark.parametrize("numerics", ["exact", "dequantised"])
def test_c5_full_width_continuations_match_causal_oracle(db, oracle, numerics):
    cfg = dict(layers=2, hidden=2560, q_heads=32, kv_heads=8, head_dim=128, ffn=9728, vocab=151936, weight_bits=4)
    model = db.Model.synthetic(db.EncoderConfig(**cfg, max_sequence_tokens=1024, causal=True), seed=5)
    if numerics == "dequantised":
        model.set_code_layout(db.CODES_DQ)
    D, F, L, Nq, Nk = 2560, 9728, 2, 4096, 1024
    shapes = {"q": (Nq, D), "k": (Nk, D), "v": (Nk, D), "o": (D, Nq), "gate": (F, D), "up": (F, D), "down": (D, F)}
    w = {"embedding": model.synthetic_weight("embedding")}
    for name, shape in shapes.items():
        w[name] = [model.synthetic_weight(name, l).reshape(shape) for l in range(L)]
    for name, size in (("input_norm", D), ("post_norm", D), ("q_norm", 128), ("k_norm", 128)):
        w[name] = [np.ones(size, np.float32) for _ in range(L)]
    w["final_norm"] = np.ones(D, np.float32)
    rng = np.random.default_rng(5)
    prefix = rng.integers(0, cfg["vocab"], 512).astype(np.int32)
    conts = rng.integers(0, cfg["vocab"], (4, 32)).astype(np.int32)
    cache = model.create_cache(db.CacheOptions(max_bytes=256 << 20, require_prefix=True))
    got = model.predict_continuations(prefix, conts, cache=cache)
    again = model.predict_continuations(prefix, conts, cache=cache)  # prefix reused from the cache
    assert np.array_equal(again.view(np.uint32), got.view(np.uint32))
    # scored by log-probability over the 151,936-token vocabulary (LM head tied to the embedding)
    lp, rows = model.score_continuations(prefix, conts, cache=cache, hidden=True)
    model.close()
    assert np.array_equal(rows[1:].view(np.uint32), got.reshape(-1, D).view(np.uint32))
    want = oracle.lm_logprobs(w["embedding"], rows, conts, 4, mode=2)
    assert np.abs(lp - want).max() <= 5e-5, np.abs(lp - want).max()
    ref = oracle.Encoder(dict(cfg, causal=1), w)
    for c in range(4):
        _, h = ref.forward(np.concatenate([prefix, conts[c]]), mode=2, hidden=True)
        per_token = [cosine(got[c, t], h[512 + t]) for t in range(32)]
        assert min(per_token) >= 0.999, (c, min(per_token))
        assert cosine(got[c].mean(0), h[512:].mean(0)) >= 0.9999
        if c == 0:
            e2e = oracle.lm_logprobs(w["embedding"], np.concatenate([h[511:512], h[512:544]]), conts[:1], 4,
                                     mode=2)[0]
            err = np.abs(lp[0] - e2e)
            assert err.max() <= 0.1 and err.mean() <= 0.03, (err.max(), err.mean())
