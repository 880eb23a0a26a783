"""C4: the Decima-shaped (BERT) encoder on the Decima int8 kernels against the composed CPU oracle
(oracle.bert_forward: decima/mod.rs:492-556 with the W8A8 block projections of decima/int8.rs,
LayerNorm and erf GELU of decima/cpu.rs).  The attention runs in f16 on the GPU and in f32 on the
CPU, and CUDA's erff differs from libm's by an ulp or so, so the bar is the encoder's: mean-pooled
state cosine >= 0.9999, every token's state >= 0.999.  Relative-position attention is not part of
this model (the reference's Decima uses absolute positions).

The cross-encoder request (score: one state with several choices, run as packed state+choice
sequences) computes every row, every sequence's attention and every pool as a one-sequence predict
does, so its pooled states equal predict's bit for bit, and its scorer head equals the oracle's
sequential f32 linear bit for bit on the same pooled state."""
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


def oracle_weights(db, cfg, seed, std):
    def f32(tensor, shape):
        bits = db.synthetic_bf16(seed, tensor, shape, std).cpu().numpy().view(np.uint16).astype(np.uint32) << 16
        return bits.view(np.float32).reshape(shape)

    D, F = cfg["hidden"], cfg["ffn"]
    w = {"word": f32(0, (cfg["vocab"], D)), "pos": f32(1, (cfg["max_positions"], D)), "type": f32(2, (2, D)),
         "emb_ln_w": np.ones(D, np.float32), "emb_ln_b": np.zeros(D, np.float32), "layers": []}
    for l in range(cfg["layers"]):
        t = lambda k: 16 + 16 * l + k
        w["layers"].append({"q": f32(t(0), (D, D)), "k": f32(t(1), (D, D)), "v": f32(t(2), (D, D)),
                            "o": f32(t(3), (D, D)), "ff1": f32(t(4), (F, D)), "ff2": f32(t(5), (D, F)),
                            "bq": f32(t(6), (D,)), "bk": f32(t(7), (D,)), "bv": f32(t(8), (D,)),
                            "bo": f32(t(9), (D,)), "b1": f32(t(10), (F,)), "b2": f32(t(11), (D,)),
                            "ln1_w": np.ones(D, np.float32), "ln1_b": np.zeros(D, np.float32),
                            "ln2_w": np.ones(D, np.float32), "ln2_b": np.zeros(D, np.float32)})
    return w


@pytest.mark.parametrize("hidden,heads,block,tokens", [(256, 4, 32, 100), (256, 4, 32, 1), (512, 4, 64, 128),
                                                       (384, 6, 32, 77)])
def test_c4_encoder_matches_composed_oracle(db, hidden, heads, block, tokens):
    from oracle import oracle
    cfg = dict(layers=2, hidden=hidden, heads=heads, ffn=2 * hidden, vocab=1000, max_positions=128, block=block,
               eps=1e-12)
    seed, std = 7, 0.05
    model = db.BertModel(db.BertConfig(**cfg), seed=seed, std=std)
    ids = np.random.default_rng(tokens).integers(0, cfg["vocab"], tokens).astype(np.int32)
    pooled, states = model.predict(ids, hidden=True)
    want_pooled, want_states = oracle.bert_forward(cfg, oracle_weights(db, cfg, seed, std), ids)
    assert cosine(pooled, want_pooled) >= 0.9999, cosine(pooled, want_pooled)
    per_token = [cosine(states[t], want_states[t]) for t in range(tokens)]
    assert min(per_token) >= 0.999, min(per_token)
    model.close()
    assert db.device_error_word() == 0


@pytest.mark.parametrize("fused", [True, False])
def test_c4_encoder_weights_mode_matches_oracle(db, fused):
    """The same encoder with Weights-mode (W8A32) projections: f32 activations against the int8
    weight codes (decima/int8.rs:166-283, weights_x86.rs), in either accumulation order."""
    from oracle import oracle
    cfg = dict(layers=2, hidden=256, heads=4, ffn=512, vocab=1000, max_positions=128, block=32, eps=1e-12)
    seed, std = 11, 0.05
    model = db.BertModel(db.BertConfig(**cfg, fused=fused, mode=1), seed=seed, std=std)
    ids = np.random.default_rng(5).integers(0, cfg["vocab"], 90).astype(np.int32)
    pooled, states = model.predict(ids, hidden=True)
    want_pooled, want_states = oracle.bert_forward(dict(cfg, mode=1), oracle_weights(db, cfg, seed, std), ids,
                                                   mode=0 if fused else 1)
    assert cosine(pooled, want_pooled) >= 0.9999, cosine(pooled, want_pooled)
    assert min(cosine(states[t], want_states[t]) for t in range(len(ids))) >= 0.999
    # W8A32 keeps the activations in f32: closer to the oracle than the W8A8 model is
    w8a8 = db.BertModel(db.BertConfig(**cfg, fused=fused), seed=seed, std=std)
    assert cosine(pooled, want_pooled) >= cosine(w8a8.predict(ids), want_pooled)
    logits = model.score(ids[:40], [ids[40:50], ids[50:52]])
    assert logits.shape == (2, 3) and np.all(np.isfinite(logits))
    model.close()
    w8a8.close()


def test_c4_encoder_rejects_bad_requests(db):
    cfg = db.BertConfig(layers=1, hidden=256, heads=4, ffn=512, vocab=100, max_positions=64)
    model = db.BertModel(cfg)
    with pytest.raises(db.Error) as e:
        model.predict(np.arange(65) % 100)
    assert e.value.code == "INPUT_TOO_LONG"
    with pytest.raises(db.Error) as e:
        model.predict([100])
    assert e.value.code == "INVALID_REQUEST"
    with pytest.raises(db.Error):
        db.BertModel(db.BertConfig(layers=1, hidden=250, heads=4, ffn=512, vocab=100, max_positions=64))
    model.close()


def head_weights(db, cfg, seed, std):
    def f32(tensor, shape):
        bits = db.synthetic_bf16(seed, tensor, shape, std).cpu().numpy().view(np.uint16).astype(np.uint32) << 16
        return bits.view(np.float32).reshape(shape)
    return f32(3, (3, cfg["hidden"])), f32(4, (3,))


def check_score(db, model, cfg, seed, std, state, choices, oracle_seqs=()):
    from oracle import oracle
    logits, pooled = model.score(state, choices, pooled=True)
    assert logits.shape == (len(choices), 3) and pooled.shape == (len(choices), cfg["hidden"])
    hw, hb = head_weights(db, cfg, seed, std)
    # the head on the GPU's pooled states: bit-exact against the sequential f32 linear
    assert np.array_equal(logits.view(np.uint32), oracle.bert_score_head(pooled, hw, hb).view(np.uint32))
    for i, ch in enumerate(choices):
        single = model.predict(np.concatenate([state, ch]))
        assert np.array_equal(pooled[i].view(np.uint32), single.view(np.uint32)), i
    if oracle_seqs:
        w = oracle_weights(db, cfg, seed, std)
        for i in oracle_seqs:
            want_pooled, _ = oracle.bert_forward(cfg, w, np.concatenate([state, choices[i]]))
            assert cosine(pooled[i], want_pooled) >= 0.9999, (i, cosine(pooled[i], want_pooled))
            want = oracle.bert_score_head(want_pooled[None, :], hw, hb)[0]
            # pooled cosine >= 0.9999 puts |pooled - want| within ~0.0142 |want|, so by Cauchy-Schwarz
            # each logit is within 0.02 |w_o| |want| of the oracle's
            bound = 0.02 * np.linalg.norm(hw, axis=1) * np.linalg.norm(want_pooled)
            assert np.all(np.abs(logits[i] - want) <= bound), (logits[i], want, bound)


@pytest.mark.parametrize("block,nstate,lens", [(32, 40, (5, 17, 1, 33, 9)), (64, 1, (3,)), (32, 0, (7, 64, 2)),
                                               (32, 60, (0, 4))])
def test_c4_score_packed_request(db, block, nstate, lens):
    cfg = dict(layers=2, hidden=256, heads=4, ffn=512, vocab=1000, max_positions=128, block=block, eps=1e-12)
    seed, std = 9, 0.05
    model = db.BertModel(db.BertConfig(**cfg), seed=seed, std=std)
    rng = np.random.default_rng(nstate)
    state = rng.integers(0, cfg["vocab"], nstate).astype(np.int32)
    choices = [rng.integers(0, cfg["vocab"], n).astype(np.int32) for n in lens]
    check_score(db, model, cfg, seed, std, state, choices, oracle_seqs=(0, len(lens) - 1))
    model.close()
    assert db.device_error_word() == 0


def test_c4_score_rejects_bad_requests(db):
    cfg = db.BertConfig(layers=1, hidden=256, heads=4, ffn=512, vocab=100, max_positions=64)
    model = db.BertModel(cfg)
    state = np.arange(40) % 100
    for choices, code in (([], "INVALID_REQUEST"), ([[1]] * 17, "INVALID_REQUEST"), ([[1], [2] * 25], "INPUT_TOO_LONG"),
                          ([[1], [100]], "INVALID_REQUEST")):
        with pytest.raises(db.Error) as e:
            model.score(state, choices)
        assert e.value.code == code, choices
    with pytest.raises(db.Error) as e:
        model.score([], [[]])
    assert e.value.code == "INVALID_REQUEST"
    assert model.score(state, [[1]] * 16).shape == (16, 3)  # the model still serves
    model.close()
