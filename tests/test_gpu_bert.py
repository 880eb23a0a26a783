"""C4: the Decima-shaped (BERT) encoder on the Decima int8 kernels against the composed CPU oracle
(oracle.bert_forward: decima/mod.rs:492-556 with the W8A8 block projections of decima/int8.rs,
LayerNorm and erf GELU of decima/cpu.rs).  The attention runs in f16 on the GPU and in f32 on the
CPU, and CUDA's erff differs from libm's by an ulp or so, so the bar is the encoder's: mean-pooled
state cosine >= 0.9999, every token's state >= 0.999.  Relative-position attention is not part of
this model (the reference's Decima uses absolute positions)."""
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
