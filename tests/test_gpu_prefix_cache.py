"""C5 decoder path: a causal model's prefix keys/values computed once and reused, and continuations
run batched after it (kev/mod.rs:163-300 semantics).  Checked against the composed CPU oracle
with causal attention: a continuation's hidden states equal the tail of one causal pass over
prefix + continuation (cosine >= 0.9999 per token, the encoder's bar; the attention runs in
f16), and the cached, recomputed and batched results agree with each other bit for bit."""
import numpy as np
import pytest

from test_gpu_model import SMALL, cosine, random_weights

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def db():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import decisive_b200 as d
    d.load()
    return d


def decoder(db, oracle, bits=4, seed=5):
    cfg = dict(SMALL, weight_bits=bits)
    w = random_weights(oracle, cfg, seed=seed)
    model = db.Model.from_weights(db.EncoderConfig(**cfg, max_sequence_tokens=512, causal=True), w)
    ref = oracle.Encoder(dict(cfg, causal=1), w)
    return cfg, model, ref


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("prefix_len,tokens,count", [(64, 32, 4), (100, 17, 3), (1, 5, 2), (300, 70, 2)])
def test_continuations_match_causal_oracle(db, oracle, bits, prefix_len, tokens, count):
    cfg, model, ref = decoder(db, oracle, bits)
    rng = np.random.default_rng(prefix_len * 7 + tokens)
    prefix = rng.integers(0, cfg["vocab"], prefix_len).astype(np.int32)
    conts = rng.integers(0, cfg["vocab"], (count, tokens)).astype(np.int32)
    cache = model.create_cache(db.CacheOptions(max_bytes=64 << 20, require_prefix=True))
    got = model.predict_continuations(prefix, conts, cache=cache)
    assert got.shape == (count, tokens, cfg["hidden"])
    for c in range(count):
        _, h = ref.forward(np.concatenate([prefix, conts[c]]), mode=2, hidden=True)
        per_token = [cosine(got[c, t], h[prefix_len + t]) for t in range(tokens)]
        # single token states carry the activation-quantisation noise that pooling averages out:
        # 0.999 per token, 0.9999 for the continuation's mean state (the encoder's bar)
        assert min(per_token) >= 0.999, (c, min(per_token))
        assert cosine(got[c].mean(0), h[prefix_len:].mean(0)) >= 0.9999
        if c == 0 and prefix_len > 1:
            # the test sees the prefix: the same tokens without it are far off
            _, alone = ref.forward(conts[c], mode=2, hidden=True)
            assert cosine(got[c].mean(0), alone.mean(0)) < 0.999
    st = cache.stats()
    assert st["hits"] == 0 and st["prefix_tokens_computed"] == prefix_len
    # the same prefix again: reused, identical bits; one continuation alone: identical bits
    again = model.predict_continuations(prefix, conts, cache=cache)
    assert np.array_equal(again.view(np.uint32), got.view(np.uint32))
    st = cache.stats()
    assert st["hits"] == 1 and st["prefix_tokens_reused"] == prefix_len
    one = model.predict_continuations(prefix, conts[-1:], cache=None)
    assert np.array_equal(one[0].view(np.uint32), got[-1].view(np.uint32))
    model.close()


def test_prefill_predict_is_causal(db, oracle):
    cfg, model, ref = decoder(db, oracle, 4, seed=9)
    ids = np.random.default_rng(1).integers(0, cfg["vocab"], 90).astype(np.int32)
    got = np.asarray(model.predict(ids).response)
    want = ref.forward(ids, mode=2)
    assert cosine(got, want) >= 0.9999
    enc = oracle.Encoder(dict(SMALL, weight_bits=4), random_weights(oracle, dict(SMALL, weight_bits=4), seed=9))
    assert cosine(enc.forward(ids, mode=2), want) < 0.99999  # the mask matters
    model.close()


def test_prefix_cache_contract(db, oracle):
    cfg, model, _ = decoder(db, oracle, 4)
    caps = model.capabilities()
    assert caps["model"] == "decoder" and caps["caches"] == ["prefix"]
    small = model.create_cache(db.CacheOptions(max_bytes=1024, require_prefix=True))  # too small to keep
    prefix = np.arange(50, dtype=np.int32)
    conts = np.ones((2, 8), np.int32)
    a = model.predict_continuations(prefix, conts, cache=small)
    b = model.predict_continuations(prefix, conts, cache=small)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    assert small.stats()["hits"] == 0 and small.stats()["prefix_tokens_computed"] == 100
    with pytest.raises(db.Error) as e:
        model.predict_continuations(np.arange(500, dtype=np.int32), np.ones((1, 20), np.int32))
    assert e.value.code == "INPUT_TOO_LONG"
    with pytest.raises(db.Error) as e:
        model.predict_continuations(prefix, np.full((1, 4), cfg["vocab"], np.int32))
    assert e.value.code == "INVALID_REQUEST"
    other = db.Model.synthetic(db.EncoderConfig(**SMALL, weight_bits=4, max_sequence_tokens=512, causal=True), seed=1)
    with pytest.raises(db.Error) as e:
        other.predict_continuations(prefix, conts, cache=small)
    assert e.value.code == "CACHE_OWNER"
    enc = db.Model.synthetic(db.EncoderConfig(**SMALL, weight_bits=4, max_sequence_tokens=512), seed=1)
    with pytest.raises(db.Error) as e:
        enc.create_cache(db.CacheOptions(require_prefix=True))
    assert e.value.code == "UNSUPPORTED_CACHE"
    model.close()
    other.close()
    enc.close()


def lm_rows(h, prefix_len, tokens):
    """The LM head's input rows for one continuation from a causal pass's final states h."""
    return np.concatenate([h[prefix_len - 1:prefix_len], h[prefix_len:prefix_len + tokens]])


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("prefix_len,tokens,count", [(50, 9, 3), (1, 1, 1), (200, 33, 2)])
def test_scored_continuations(db, oracle, bits, prefix_len, tokens, count):
    """Log-probability scoring: the LM head (tied embedding, W*A8 g64) and the f32 log-softmax on
    the GPU's own rows agree with the oracle's f64 log-softmax over the oracle GEMM's logits to
    2e-5; end to end against the causal oracle, per-token log-probs agree to 0.1 (mean 0.03: the
    states carry the f16 attention's noise, cosine >= 0.999 per token)."""
    cfg, model, ref = decoder(db, oracle, bits)
    w = random_weights(oracle, cfg, seed=5)
    rng = np.random.default_rng(prefix_len + 11 * tokens)
    prefix = rng.integers(0, cfg["vocab"], prefix_len).astype(np.int32)
    conts = rng.integers(0, cfg["vocab"], (count, tokens)).astype(np.int32)
    cache = model.create_cache(db.CacheOptions(max_bytes=64 << 20, require_prefix=True))
    lp, rows = model.score_continuations(prefix, conts, cache=cache, hidden=True)
    assert lp.shape == (count, tokens) and rows.shape == (1 + count * tokens, cfg["hidden"])
    assert np.all(lp < 0)
    want = oracle.lm_logprobs(w["embedding"], rows, conts, bits)
    assert np.abs(lp - want).max() <= 2e-5, np.abs(lp - want).max()
    # the rows after the first are the continuation states predict_continuations returns
    states = model.predict_continuations(prefix, conts, cache=cache)
    assert np.array_equal(rows[1:].view(np.uint32), states.reshape(-1, cfg["hidden"]).view(np.uint32))
    for c in range(count):
        _, h = ref.forward(np.concatenate([prefix, conts[c]]), mode=2, hidden=True)
        e2e = oracle.lm_logprobs(w["embedding"], lm_rows(h, prefix_len, tokens), conts[c:c + 1], bits)[0]
        err = np.abs(lp[c] - e2e)
        assert err.max() <= 0.1 and err.mean() <= 0.03, (c, err.max(), err.mean())
    # a reused prefix (its last state kept with its keys and values) and no cache give the same bits
    again = model.score_continuations(prefix, conts, cache=cache)
    assert np.array_equal(again.view(np.uint32), lp.view(np.uint32))
    st = cache.stats()
    assert st["hits"] == 2 and st["prefix_tokens_computed"] == prefix_len
    alone = model.score_continuations(prefix, conts[-1:])
    assert np.array_equal(alone[0].view(np.uint32), lp[-1].view(np.uint32))
    model.close()


def test_scoring_rejects_bad_requests(db, oracle):
    cfg, model, _ = decoder(db, oracle, 4)
    with pytest.raises(db.Error) as e:
        model.score_continuations([1, 2], np.zeros((2, 0), np.int32))
    assert e.value.code == "INVALID_REQUEST"
    with pytest.raises(db.Error) as e:
        model.score_continuations(np.arange(500) % 1000, np.zeros((1, 13), np.int32))
    assert e.value.code == "INPUT_TOO_LONG"
    with pytest.raises(db.Error) as e:
        model.score_continuations([1, 2], [[3, 1000]])
    assert e.value.code == "INVALID_REQUEST"
    assert model.score_continuations([1, 2], [[3, 4]]).shape == (1, 2)
    model.close()
