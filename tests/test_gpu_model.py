"""Model-level GPU tests: the encoder forward against the composed CPU oracle, and the
inference-API contract (src/inference/tests.rs:58-140) through the C ABI."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

SMALL = dict(layers=2, hidden=256, q_heads=4, kv_heads=2, head_dim=128, ffn=512, vocab=1000)


@pytest.fixture(scope="module")
def db():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import decisive_b200 as d
    d.load()
    return d


def random_weights(oracle, cfg, seed=0, std=0.02):
    rng = np.random.default_rng(seed)
    D, F, V = cfg["hidden"], cfg["ffn"], cfg["vocab"]
    Nq, Nk = cfg["q_heads"] * 128, cfg["kv_heads"] * 128
    L = cfg["layers"]

    def bf(shape):
        return oracle.f32_to_bf16(rng.normal(0, std, shape).astype(np.float32))

    def norm(n):
        return (1 + rng.normal(0, 0.1, n)).astype(np.float32)

    w = {"embedding": bf((V, D))}
    for name, shape in (("q", (Nq, D)), ("k", (Nk, D)), ("v", (Nk, D)), ("o", (D, Nq)), ("gate", (F, D)),
                        ("up", (F, D)), ("down", (D, F))):
        w[name] = [bf(shape) for _ in range(L)]
    for name, n in (("input_norm", D), ("post_norm", D), ("q_norm", 128), ("k_norm", 128)):
        w[name] = [norm(n) for _ in range(L)]
    w["final_norm"] = norm(D)
    return w


def cosine(a, b):
    a, b = a.astype(np.float64), b.astype(np.float64)
    return float(a @ b / np.linalg.norm(a) / np.linalg.norm(b))


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("tokens", [1, 37, 300])
def test_encoder_matches_composed_oracle(db, oracle, bits, tokens):
    cfg = dict(SMALL, weight_bits=bits)
    w = random_weights(oracle, cfg, seed=bits)
    model = db.Model.from_weights(db.EncoderConfig(**cfg, max_sequence_tokens=512), w)
    ref = oracle.Encoder(cfg, w)
    ids = np.random.default_rng(tokens).integers(0, cfg["vocab"], tokens).astype(np.int32)
    got = model.predict(ids).response
    want = ref.forward(ids, mode=2)
    # north_star: final embeddings within cosine >= 0.9999 of the reference CPU path
    assert cosine(got, want) >= 0.9999, cosine(got, want)
    model.close()


def test_full_shape_layers_match_oracle(db, oracle):
    # BASELINE config 2 dimensions (2 of the 28 layers), synthetic weights exported for the oracle
    cfg = dict(layers=2, hidden=1024, q_heads=16, kv_heads=8, head_dim=128, ffn=3072, vocab=151936, weight_bits=4)
    model = db.Model.synthetic(db.EncoderConfig(**cfg), seed=7)
    w = {"embedding": model.synthetic_weight("embedding")}
    D, F = 1024, 3072
    shapes = {"q": (2048, D), "k": (1024, D), "v": (1024, D), "o": (D, 2048), "gate": (F, D), "up": (F, D),
              "down": (D, F)}
    for n in shapes:
        w[n] = [model.synthetic_weight(n, l).reshape(shapes[n]) for l in range(2)]
    for n, size in (("input_norm", D), ("post_norm", D), ("q_norm", 128), ("k_norm", 128)):
        w[n] = [np.ones(size, np.float32) for _ in range(2)]
    w["final_norm"] = np.ones(D, np.float32)
    ids = np.random.default_rng(2).integers(0, cfg["vocab"], 1024).astype(np.int32)
    got = model.predict(ids).response
    want = oracle.Encoder(cfg, w).forward(ids, mode=2)
    assert cosine(got, want) >= 0.9999, cosine(got, want)
    model.close()


# ------------------------------------------------------------------ inference API contract
@pytest.fixture(scope="module")
def small_model(db):
    m = db.Model.synthetic(db.EncoderConfig(**dict(SMALL, weight_bits=4), max_sequence_tokens=64), seed=1)
    yield m
    m.close()


def test_capabilities_and_unsupported_prefix_cache(db, small_model):
    caps = small_model.capabilities()
    assert caps["model"] == "pplx-flash" and caps["backend"] == "cuda" and caps["caches"] == []
    with pytest.raises(db.Error) as e:
        small_model.create_cache(db.CacheOptions(require_prefix=True))
    assert e.value.code == "UNSUPPORTED_CACHE"


def test_batches_keep_order_and_per_item_failures(db, small_model):
    ids = [np.arange(5), np.arange(10) + 3, np.array([], np.int32), np.arange(100), np.array([999999]), np.arange(7)]
    cache = small_model.create_cache()
    out = small_model.predict_batch(ids, cache=cache)
    assert [o.status for o in out] == ["success", "success", "error", "error", "error", "success"]
    assert out[2].error.code == "INVALID_REQUEST"
    assert out[3].error.code == "INPUT_TOO_LONG" and "exceeds token limit" in out[3].error.message
    assert out[4].error.code == "INVALID_REQUEST"
    # ordering: each success equals the single-request prediction
    for i in (0, 1, 5):
        single = small_model.predict(ids[i]).response
        assert np.array_equal(single, out[i].result.response)


def test_cache_ownership_ephemeral_calls_and_cancellation(db, small_model):
    other = db.Model.synthetic(db.EncoderConfig(**dict(SMALL, weight_bits=4), max_sequence_tokens=64), seed=2)
    foreign = other.create_cache()
    with pytest.raises(db.Error) as e:
        small_model.predict(np.arange(4), cache=foreign)
    assert e.value.code == "CACHE_OWNER"
    with pytest.raises(db.Error) as e:
        small_model.clear_cache(foreign)
    assert e.value.code == "CACHE_OWNER"
    with pytest.raises(db.Error) as e:
        small_model.predict_batch([np.arange(4)], cache=foreign)
    assert e.value.code == "CACHE_OWNER"
    for _ in range(2):
        small_model.predict(np.arange(4))
    c = db.Cancellation()
    c.cancel()
    batch = small_model.predict_batch([np.arange(3), np.arange(4)], cancellation=c)
    assert all(o.status == "error" and o.error.code == "CANCELLED" for o in batch)
    other.close()


def test_parameters_are_validated(db, small_model):
    with pytest.raises(db.Error) as e:
        small_model.predict(np.arange(4), parameters=db.PplxParameters(0))
    assert e.value.code == "INVALID_PARAMETERS"
    with pytest.raises(db.Error) as e:
        small_model.predict(np.arange(20), parameters=db.PplxParameters(16))
    assert e.value.code == "INPUT_TOO_LONG"
    # a larger per-call limit than the model's default grows the workspace instead of truncating
    r = small_model.predict(np.arange(80), parameters=db.PplxParameters(128))
    assert np.all(np.isfinite(r.response))


def test_predictions_are_deterministic(db, small_model):
    ids = np.random.default_rng(0).integers(0, 1000, 50)
    a = small_model.predict(ids).response
    b = small_model.predict(ids).response
    assert np.array_equal(a, b)


def test_models_on_two_devices_in_one_process(db):
    """One model per device from one process (the multi-GPU integration without collectives):
    every kernel's launch settings are made per device."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    cfg = db.EncoderConfig(**SMALL, weight_bits=4, max_sequence_tokens=256)
    a = db.Model.synthetic(cfg, seed=4, device=0)
    b = db.Model.synthetic(cfg, seed=4, device=1)
    ids = np.random.default_rng(0).integers(0, SMALL["vocab"], 200).astype(np.int32)
    ra, rb = np.asarray(a.predict(ids).response), np.asarray(b.predict(ids).response)
    assert np.array_equal(ra.view(np.uint32), rb.view(np.uint32))
    a.close()
    b.close()


def test_graph_forward_is_bit_identical(db):
    """The plain forward runs as a captured CUDA graph from its second call for a token count on;
    graph and layer-by-layer results are identical, also after the workspace grows."""
    cfg = db.EncoderConfig(**SMALL, weight_bits=4, max_sequence_tokens=128)
    m = db.Model.synthetic(cfg, seed=8)
    rng = np.random.default_rng(5)
    reqs = [rng.integers(0, SMALL["vocab"], n).astype(np.int32) for n in (64, 64, 64, 17, 17, 17, 200, 200)]
    m.use_graphs(False)
    want = [np.asarray(m.predict(r, parameters=db.PplxParameters(256)).response).copy() for r in reqs]
    m.use_graphs(True)
    for _ in range(2):
        got = [np.asarray(m.predict(r, parameters=db.PplxParameters(256)).response).copy() for r in reqs]
        for a, b in zip(want, got):
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    m.close()


@pytest.mark.parametrize("bits", [4, 8])
def test_code_layouts_are_bit_identical(db, oracle, bits):
    """int8 codes through the kind::i8 GEMM and f16 codes through the kind::f16 GEMM compute the
    same integer dots and fold them in the same order: the encoder's outputs agree bit for bit."""
    cfg = dict(SMALL, weight_bits=bits)
    model = db.Model.from_weights(db.EncoderConfig(**cfg, max_sequence_tokens=512), random_weights(oracle, cfg, 3))
    ids = np.random.default_rng(9).integers(0, cfg["vocab"], 300).astype(np.int32)
    a = np.asarray(model.predict(ids).response)
    model.set_code_layout(db.CODES_TC)
    b = np.asarray(model.predict(ids).response)
    model.set_code_layout(db.CODES_NATURAL)
    c = np.asarray(model.predict(ids).response)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32)) and np.array_equal(a.view(np.uint32), c.view(np.uint32))
    model.close()


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("tokens", [1, 37, 300])
def test_dequantised_mode_matches_composed_oracle(db, oracle, bits, tokens):
    """DB_CODES_DQ (f16(code * scale) operands, full-K f32 accumulation, separate SwiGLU
    re-quantisation): final embeddings within cosine >= 0.9999 of the oracle's exact grouped fold."""
    cfg = dict(SMALL, weight_bits=bits)
    w = random_weights(oracle, cfg, seed=bits)
    model = db.Model.from_weights(db.EncoderConfig(**cfg, max_sequence_tokens=512), w)
    model.set_code_layout(db.CODES_DQ)
    ids = np.random.default_rng(tokens).integers(0, cfg["vocab"], tokens).astype(np.int32)
    got = model.predict(ids).response
    want = oracle.Encoder(cfg, w).forward(ids, mode=2)
    assert cosine(got, want) >= 0.9999, cosine(got, want)
    model.close()
    assert db.device_error_word() == 0
