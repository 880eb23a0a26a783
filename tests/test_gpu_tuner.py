"""Kernel-selection tuner (the reference's rule, webgpu/checkpoint.rs:420-565): every candidate
is checked for bitwise equality with the default configuration, the choice is cached under a key
of device, build and shape, a cached choice is re-checked, and a tuned model's outputs are
bitwise those of the untuned model."""
import numpy as np
import pytest

import decisive_b200 as db

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K,bits,epi", [(1024, 4096, 1024, 4, db.EPILOGUE_STORE),
                                            (1024, 1024, 2048, 8, db.EPILOGUE_RESIDUAL),
                                            (1024, 6144, 1024, 4, db.EPILOGUE_SWIGLU),
                                            (100, 384, 320, 4, db.EPILOGUE_STORE)])
def test_tune_gemm_candidates_equal_and_cached(tmp_path, M, N, K, bits, epi):
    cache = str(tmp_path / "tuning.txt")
    choice, rep = db.tune_gemm(M, N, K, bits, epi, cache)
    assert rep["cached"] is False
    cands = rep["candidates"]
    # the baseline is the int8 path's default configuration for the shape
    base_cfg = cands[0]["config"]
    assert base_cfg[0] in (32, 64, 128, 256) and base_cfg[1] == 0 and base_cfg[2] in (0, 1)
    assert len(cands) == len({tuple(c["config"]) for c in cands}) >= (1 if epi == db.EPILOGUE_SWIGLU else 3)
    assert all(c["equal"] for c in cands)  # every tile configuration is bitwise equal by design
    assert all(c["ms"] > 0 for c in cands)
    got = [choice.block_n, choice.max_ctas, choice.pair_ctas]
    assert got in [c["config"] for c in cands]
    if got != base_cfg:
        base = cands[0]["ms"]
        assert min(c["ms"] for c in cands if c["config"] == got) <= 0.99 * base
    choice2, rep2 = db.tune_gemm(M, N, K, bits, epi, cache)
    assert rep2["cached"] is True and rep2["key"] == rep["key"]
    assert [choice2.block_n, choice2.max_ctas, choice2.pair_ctas] == got


def test_tune_cache_ignores_malformed_entries(tmp_path):
    cache = tmp_path / "tuning.txt"
    _, rep = db.tune_gemm(512, 1024, 512, 4, db.EPILOGUE_STORE, str(cache))
    with open(cache, "a") as f:
        f.write(f"{rep['key']} 96 0 0\n")  # not a valid tile width
    choice, rep2 = db.tune_gemm(512, 1024, 512, 4, db.EPILOGUE_STORE, str(cache))
    assert rep2["cached"] is True and rep2["choice"] in [[bn, 0, p] for bn in (32, 64, 128, 256) for p in (0, 1)]
    cache.write_text(f"{rep['key']} 96 0 0\n")  # only a malformed entry: tuned again
    _, rep3 = db.tune_gemm(512, 1024, 512, 4, db.EPILOGUE_STORE, str(cache))
    assert rep3["cached"] is False


def test_tune_rejects_bad_arguments():
    with pytest.raises(db.CudaError):
        db.tune_gemm(128, 100, 128, 4, db.EPILOGUE_SWIGLU)  # SwiGLU needs N % 128 == 0
    with pytest.raises(db.CudaError):
        db.tune_gemm(128, 128, 128, 5)


def test_tuned_model_outputs_bitwise_equal(tmp_path):
    cfg = db.EncoderConfig(layers=2, hidden=512, q_heads=8, kv_heads=4, head_dim=128, ffn=1536, vocab=1000,
                           weight_bits=4, max_sequence_tokens=512)
    m = db.Model.synthetic(cfg, seed=7)
    rng = np.random.default_rng(1)
    ids = [rng.integers(0, 1000, n).tolist() for n in (512, 300, 129)]
    before = [np.array(m.predict(x).response, copy=True) for x in ids]
    rep = m.tune(512, str(tmp_path / "t.txt"))
    assert set(rep) == {"qkv", "o", "gate_up", "down"}
    after = [np.asarray(m.predict(x).response) for x in ids]
    for a, b in zip(before, after):
        assert np.array_equal(a, b)
    rep2 = m.tune(512, str(tmp_path / "t.txt"))
    assert all(r["cached"] for r in rep2.values())
