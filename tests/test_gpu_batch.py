"""C3: a ragged batch of encoder requests run as packed passes (int8 weights,
64 sequences with lengths drawn uniformly from 16 to 1024).

predict_batch concatenates the requests' tokens, runs every projection once over all rows and the
attention per sequence over its own keys, then pools each sequence.  Every kernel computes a row
(or one sequence's attention) as the one-request forward does, so each outcome equals predict's
bit for bit; the composed CPU oracle bounds the result (pooled cosine >= 0.9999).  Outcomes keep
the reference's order (src/inference/mod.rs:250-273)."""
import numpy as np
import pytest

from test_gpu_model import cosine

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

C2 = dict(hidden=1024, q_heads=16, kv_heads=8, head_dim=128, ffn=3072, vocab=151936)


@pytest.fixture(scope="module")
def db():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import decisive_b200 as d
    d.load()
    return d


def c3_requests(n=64, seed=3):
    rng = np.random.default_rng(seed)
    lens = rng.integers(16, 1025, n)
    return [rng.integers(0, C2["vocab"], int(L)).astype(np.int32) for L in lens]


def synthetic_oracle_weights(model, cfg):
    D, F, L = cfg["hidden"], cfg["ffn"], cfg["layers"]
    Nq, Nk = cfg["q_heads"] * 128, cfg["kv_heads"] * 128
    shapes = {"q": (Nq, D), "k": (Nk, D), "v": (Nk, D), "o": (D, Nq), "gate": (F, D), "up": (F, D), "down": (D, F)}
    w = {"embedding": model.synthetic_weight("embedding")}
    for name, shape in shapes.items():
        w[name] = [model.synthetic_weight(name, l).reshape(shape) for l in range(L)]
    for name, size in (("input_norm", D), ("post_norm", D), ("q_norm", 128), ("k_norm", 128)):
        w[name] = [np.ones(size, np.float32) for _ in range(L)]
    w["final_norm"] = np.ones(D, np.float32)
    return w


def test_c3_packed_batch_matches_oracle_and_single_requests(db, oracle):
    cfg = dict(C2, layers=2, weight_bits=8)
    model = db.Model.synthetic(db.EncoderConfig(**cfg, max_sequence_tokens=1024), seed=21)
    reqs = c3_requests()
    out = model.predict_batch(reqs)
    assert all(o.status == "success" for o in out)
    ref = oracle.Encoder(cfg, synthetic_oracle_weights(model, cfg))
    for i, r in enumerate(reqs):
        got = np.asarray(out[i].result.response)
        single = np.asarray(model.predict(r).response)
        assert np.array_equal(got.view(np.uint32), single.view(np.uint32)), i
        assert cosine(got, ref.forward(r, mode=2)) >= 0.9999, i
    model.close()
    assert db.device_error_word() == 0


def test_c3_packed_batch_dequantised_mode(db, oracle):
    """The packed pass with the dequantised projections (DB_CODES_DQ): every request equals its own
    single pass bit for bit (each output row is its own full-K sum) and the oracle within cosine
    >= 0.9999."""
    cfg = dict(C2, layers=2, weight_bits=8)
    model = db.Model.synthetic(db.EncoderConfig(**cfg, max_sequence_tokens=1024), seed=21)
    model.set_code_layout(db.CODES_DQ)
    reqs = c3_requests()[:16]
    out = model.predict_batch(reqs)
    assert all(o.status == "success" for o in out)
    ref = oracle.Encoder(cfg, synthetic_oracle_weights(model, cfg))
    for i, r in enumerate(reqs):
        got = np.asarray(out[i].result.response)
        single = np.asarray(model.predict(r).response)
        assert np.array_equal(got.view(np.uint32), single.view(np.uint32)), i
        assert cosine(got, ref.forward(r, mode=2)) >= 0.9999, i
    model.close()
    assert db.device_error_word() == 0


def test_c3_full_depth_packed_equals_single(db):
    cfg = dict(C2, layers=28, weight_bits=8)
    model = db.Model.synthetic(db.EncoderConfig(**cfg, max_sequence_tokens=1024), seed=22)
    reqs = c3_requests(seed=4)
    out = model.predict_batch(reqs)
    for i in (0, 1, 17, 40, 63):
        single = np.asarray(model.predict(reqs[i]).response)
        got = np.asarray(out[i].result.response)
        assert np.all(np.isfinite(got)) and np.array_equal(got.view(np.uint32), single.view(np.uint32)), i
    model.close()


def test_ragged_batch_mixed_outcomes_and_lengths(db, oracle):
    """Invalid requests keep their place; valid ones of every length (1, tile-ragged, 128-exact)
    come out as single predicts."""
    from test_gpu_model import SMALL, random_weights
    cfg = dict(SMALL, weight_bits=4)
    model = db.Model.from_weights(db.EncoderConfig(**cfg, max_sequence_tokens=300), random_weights(oracle, cfg, 8))
    rng = np.random.default_rng(6)
    reqs = [rng.integers(0, 1000, n).astype(np.int32) for n in (1, 129, 128, 300, 77, 2)]
    reqs.insert(2, np.array([], np.int32))
    reqs.insert(4, np.arange(301) % 1000)
    out = model.predict_batch(reqs)
    assert [o.status for o in out] == ["success", "success", "error", "success", "error", "success", "success",
                                       "success"]
    assert out[2].error.code == "INVALID_REQUEST" and out[4].error.code == "INPUT_TOO_LONG"
    for i in (0, 1, 3, 5, 6, 7):
        single = np.asarray(model.predict(reqs[i]).response)
        assert np.array_equal(np.asarray(out[i].result.response).view(np.uint32), single.view(np.uint32)), i
    model.close()
