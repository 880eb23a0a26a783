"""CPU checks of the C-ABI boundary: the library loads without a GPU and exports every entry
point include/decisive_b200.h declares; argument validation that runs before any device work."""
import ctypes as C
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "decisive_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"\b(db_[a-z0-9_]+)\s*\(", text)
    return sorted(set(names))


@pytest.fixture(scope="module")
def lib():
    from decisive_b200 import build, _lib
    build.build()
    return _lib.load()


def test_header_declares_the_boundary():
    names = declared_functions()
    for must in ("db_quantize_activations_g64", "db_pack_weights_g64", "db_gemm_g64", "db_linear_g64",
                 "db_mlp_g64", "db_attention", "db_predict", "db_predict_batch", "db_cache_create"):
        assert must in names


def test_library_exports_every_declared_symbol(lib):
    raw = C.CDLL(os.path.join(ROOT, "decisive_b200", "libdecisive_b200.so"))
    missing = [n for n in declared_functions() if not hasattr(raw, n)]
    assert not missing, missing


def test_bindings_cover_the_header(lib):
    from decisive_b200 import _lib
    bound = {s[0] for s in _lib.SIGNATURES}
    assert set(declared_functions()) <= bound


def test_abi_version_and_argument_validation_without_gpu(lib):
    assert lib.db_abi_version() == 1
    # shape errors are rejected on the host before any CUDA call
    rc = lib.db_quantize_activations_g64(None, 0, 0, 1, 0, 8, None, 2, 0, None, None, 1, None, None)
    assert rc == -1
    assert lib.db_last_error_code().decode() == "INVALID_ARGUMENT"
    rc = lib.db_gemm_g64(None, 2, 64, None, None, 1, None, None, 1, 0, 64, 4, 1, 0, None, 0, None, None)
    assert rc == -1
    rc = lib.db_attention(None, None, None, 8, 4, 3, 128, 1.0, None, 512, None)
    assert rc == -5 and lib.db_last_error_code().decode() == "UNSUPPORTED"


def test_code_layout_constants_match_the_header(lib):
    """The activation layouts the header defines (DB_CODES_*) are the binding's constants; a layout
    past the last one is refused on the host."""
    import decisive_b200 as db
    text = open(HEADER).read()
    defined = {k: int(v) for k, v in re.findall(r"#define DB_CODES_([A-Z]+) (\d+)", text)}
    assert defined == {"NATURAL": db.CODES_NATURAL, "GEMV": db.CODES_GEMV, "TC": db.CODES_TC, "DQ": db.CODES_DQ}
    rc = lib.db_quantize_activations_g64(None, 0, 64, 1, 64, 8, None, max(defined.values()) + 1, 64, None, None, 128,
                                         None, None)
    assert rc == -1 and lib.db_last_error_code().decode() == "INVALID_ARGUMENT"
    # the dequantised GEMM validates its shape before any device work as well
    rc = lib.db_gemm_g64(None, db.CODES_DQ, 64, None, None, 0, None, None, 1, 0, 64, 4, 1, 0, None, 0, None, None)
    assert rc == -1


def test_model_creation_without_device_reports_gpu_unavailable(lib):
    import decisive_b200 as db
    if lib.db_device_count() > 0:
        pytest.skip("a device is present")
    with pytest.raises(db.Error) as e:
        db.Model.synthetic(db.EncoderConfig(layers=1, hidden=128, q_heads=1, kv_heads=1, ffn=64, vocab=10))
    assert e.value.code == "GPU_UNAVAILABLE"


def test_invalid_config_rejected_before_device(lib):
    import decisive_b200 as db
    with pytest.raises(db.Error) as e:
        db.Model.synthetic(db.EncoderConfig(head_dim=64))
    assert e.value.code == "INVALID_PARAMETERS"


def test_missing_library_fails_loudly(tmp_path):
    from decisive_b200 import _lib
    with pytest.raises(RuntimeError):
        _lib._lib, saved = None, _lib._lib
        try:
            _lib.load(str(tmp_path / "nope.so"))
        finally:
            _lib._lib = saved
