"""Packed checkpoints in the reference's export format (export_packed.rs:13-103): a model's weights
are written as one file per layer plus embedding and final norm, with a JSON manifest giving every
tensor's name, shape and byte range and every file's size and SHA-256.  The 2-D tensors must be
byte-identical to packed::pack (packed.rs:10-56) of the same bf16 weights (checked against the
oracle), and a model loaded back must predict bit-identically to the one exported.  Corrupted files
and checkpoints that do not match the configuration are rejected."""
import hashlib
import json
import os

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


def small_cfg(db, bits):
    return db.EncoderConfig(layers=2, hidden=256, q_heads=4, kv_heads=2, head_dim=128, ffn=512, vocab=1000,
                            weight_bits=bits, max_sequence_tokens=256)


@pytest.mark.parametrize("bits", [4, 8])
def test_export_matches_reference_format_and_round_trips(db, tmp_path, bits):
    from oracle import oracle
    cfg = small_cfg(db, bits)
    m = db.Model.synthetic(cfg, seed=11)
    path = m.export_packed(str(tmp_path))
    man = json.loads(open(path).read())
    assert man["schema_version"] == 1 and man["group_size"] == 64
    assert man["scheme"] == f"q{bits}-w{bits}a8-e{bits}-r{bits}-g64"
    assert man["group_bytes"] == (36 if bits == 4 else 68)
    assert man["embedding_row_bytes"] == 256 // 64 * man["group_bytes"] and man["readout"] is None
    assert len(man["layers"]) == 2
    for name, info in man["files"].items():
        data = open(tmp_path / name, "rb").read()
        assert len(data) == info["bytes"]
        assert hashlib.sha256(data).hexdigest() == info["sha256"]
    assert man["decoder_bytes"] == sum(l["bytes"] for l in man["layers"])
    # the packed bytes are packed::pack of the model's bf16 weights
    names = {"q": "self_attn.q_proj.weight", "k": "self_attn.k_proj.weight", "v": "self_attn.v_proj.weight",
             "o": "self_attn.o_proj.weight", "gate": "mlp.gate_proj.weight", "up": "mlp.up_proj.weight",
             "down": "mlp.down_proj.weight"}
    for layer in range(2):
        entry = man["layers"][layer]
        blob = open(tmp_path / entry["file"], "rb").read()
        tensors = {t["name"]: t for t in entry["tensors"]}
        pos = 0
        for t in entry["tensors"]:  # contiguous, in order
            assert t["start"] == pos
            pos = t["end"]
        assert pos == entry["bytes"]
        for short, suffix in names.items():
            t = tensors[f"language_model.layers.{layer}.{suffix}"]
            rows, cols = t["shape"]
            bf = m.synthetic_weight(short, layer)
            want = oracle.packed_pack(bf, rows, cols, bits)
            assert np.array_equal(np.frombuffer(blob[t["start"]:t["end"]], np.uint8), want), (layer, short)
        norm = tensors[f"language_model.layers.{layer}.input_layernorm.weight"]
        assert norm["shape"] == [256]
        assert np.all(np.frombuffer(blob[norm["start"]:norm["end"]], np.uint16) == 0x3F80)  # bf16 1.0
    emb = np.frombuffer(open(tmp_path / man["embedding"], "rb").read(), np.uint8)
    assert np.array_equal(emb, oracle.packed_pack(m.synthetic_weight("embedding"), 1000, 256, bits))
    # loaded back: bit-identical predictions
    loaded = db.Model.from_packed(cfg, path, verify=True)
    rng = np.random.default_rng(2)
    for n in (1, 37, 256):
        ids = rng.integers(0, 1000, n).tolist()
        a = np.asarray(m.predict(ids).response)
        b = np.asarray(loaded.predict(ids).response)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_corrupt_or_mismatched_checkpoints_are_rejected(db, tmp_path):
    cfg = small_cfg(db, 4)
    m = db.Model.synthetic(cfg, seed=3)
    path = m.export_packed(str(tmp_path))
    man = json.loads(open(path).read())
    layer_file = tmp_path / man["layers"][1]["file"]
    blob = bytearray(open(layer_file, "rb").read())
    blob[100] ^= 0x11
    open(layer_file, "wb").write(bytes(blob))
    with pytest.raises(db.Error) as e:
        db.Model.from_packed(cfg, path, verify=True)
    assert e.value.code == "INVALID_WEIGHTS" and "sha256" in e.value.message
    db.Model.from_packed(cfg, path, verify=False)  # the digest check is what caught it
    other = db.EncoderConfig(layers=2, hidden=256, q_heads=4, kv_heads=2, head_dim=128, ffn=448, vocab=1000,
                             weight_bits=4, max_sequence_tokens=256)
    with pytest.raises(db.Error) as e:
        db.Model.from_packed(other, path, verify=False)
    assert e.value.code == "INVALID_WEIGHTS"
    with pytest.raises(db.Error) as e:
        db.Model.from_packed(small_cfg(db, 8), path, verify=False)
    assert e.value.code == "INVALID_WEIGHTS"
    with pytest.raises(db.Error):
        db.Model.from_packed(cfg, str(tmp_path / "missing.json"))


@pytest.mark.parametrize("bits", [4, 8])
def test_layer_streaming_is_bit_identical(db, tmp_path, bits):
    """Two-bank layer streaming (webgpu/streaming.rs scheme): weights in pinned host memory, each
    layer copied on a copy stream while the previous one computes; outputs equal resident ones."""
    cfg = db.EncoderConfig(layers=5, hidden=256, q_heads=4, kv_heads=2, head_dim=128, ffn=512, vocab=1000,
                           weight_bits=bits, max_sequence_tokens=256)
    m = db.Model.synthetic(cfg, seed=21)
    rng = np.random.default_rng(3)
    reqs = [rng.integers(0, 1000, n).tolist() for n in (1, 64, 256, 77)]
    want = [np.asarray(m.predict(r).response).copy() for r in reqs]
    m.set_streaming(True)
    for _ in range(2):  # consecutive forwards reuse the banks
        got = [np.asarray(m.predict(r).response).copy() for r in reqs]
        for a, b in zip(want, got):
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    with pytest.raises(db.Error):
        m.export_packed(str(tmp_path))
    m.set_streaming(False)
    got = np.asarray(m.predict(reqs[2]).response)
    assert np.array_equal(want[2].view(np.uint32), got.view(np.uint32))
    m.close()
