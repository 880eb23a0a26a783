"""GPU test of the allocation-free projection entry point (db_linear_g64_noalloc).

Some callers may not let this library allocate device memory -- a host engine that owns a fixed
device-memory budget, or a latency-critical caller that must never reach cudaMalloc and its
implicit device synchronisation.  For them the library offers a variant of the full projection
whose scratch is a fixed array compiled into the library.  This file checks it through the C ABI
against the allocating entry point (db_linear_g64), bit for bit, on consecutive calls that reuse
the shared array, at the largest shape the array holds and one past it, and checks that calls
after the first allocate no device memory and leave the entry point's own error word clear.  The
file is collected last on purpose; it also passes when run on its own.
"""
import ctypes as C

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


def _weights(db, n, k, bits, seed):
    from oracle import oracle
    w = oracle.f32_to_bf16(np.random.default_rng(seed).normal(0, 0.02, (n, k)).astype(np.float32))
    return db.pack_weights(torch.from_numpy(w.view(np.int16)).cuda(), bits)


def _both(db, x, codes, scales, n, bits):
    lib = db.load()
    m, k = x.shape
    y_alloc = db.linear(x, codes, scales, n, bits)
    y_free = torch.full((m, n), 7.0, dtype=torch.float32, device="cuda")
    rc = lib.db_linear_g64_noalloc(C.c_void_p(x.data_ptr()), m, k, C.c_void_p(codes.data_ptr()),
                                   C.c_void_p(scales.data_ptr()), n, bits, 8, 1, C.c_void_p(y_free.data_ptr()),
                                   C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, db._lib.last_error()
    torch.cuda.synchronize()
    return y_alloc.cpu().numpy(), y_free.cpu().numpy()


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("m,k,n", [(200, 1024, 3072), (3, 1024, 512), (1024, 1000, 300)])
def test_noalloc_matches_allocating_entry_point_on_consecutive_calls(db, m, k, n, bits):
    codes, scales = _weights(db, n, k, bits, seed=m + k)
    rng = np.random.default_rng(n)
    for call in range(2):  # the second call reuses the array the first one left behind
        x = torch.from_numpy(rng.normal(0, 1 + call, (m, k)).astype(np.float32)).cuda()
        a, b = _both(db, x, codes, scales, n, bits)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), f"call {call}"


def test_noalloc_clears_the_nonfinite_flag_between_calls(db):
    m, k, n = 64, 256, 128
    codes, scales = _weights(db, n, k, 4, seed=1)
    bad = torch.randn(m, k, device="cuda")
    bad[3, 5] = float("nan")
    a, b = _both(db, bad, codes, scales, n, 4)
    assert np.all(np.isnan(a)) and np.all(np.isnan(b))
    good = torch.randn(m, k, device="cuda")
    a, b = _both(db, good, codes, scales, n, 4)
    assert np.all(np.isfinite(b)) and np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_noalloc_rejects_shapes_beyond_its_scratch(db):
    lib = db.load()
    cap = lib.db_linear_noalloc_scratch_bytes()
    m, k, n = 4096, 4096, 64  # f16 codes alone need 32 MiB
    assert m * k * 2 > cap
    x = torch.empty((1, 1), device="cuda")
    rc = lib.db_linear_g64_noalloc(C.c_void_p(x.data_ptr()), m, k, C.c_void_p(x.data_ptr()),
                                   C.c_void_p(x.data_ptr()), n, 4, 8, 1, C.c_void_p(x.data_ptr()), None)
    assert rc == -1
    assert lib.db_last_error_code().decode() == "SCRATCH_LIMIT"


CODE_BYTES = 2  # bytes per activation code in the tensor-core layout the entry point quantises into


def _need(m, k):
    """Scratch bytes of one call, as the header documents the carve: codes, scales, sums, flag."""
    up = lambda b: (b + 255) // 256 * 256
    g = (k + 63) // 64
    lds = (m + 127) // 128 * 128
    return up(m * g * 64 * CODE_BYTES) + 2 * up(g * lds * 4) + 256


def test_noalloc_at_the_end_of_its_scratch(db):
    lib = db.load()
    cap = lib.db_linear_noalloc_scratch_bytes()
    k, n = 960, 256
    m = 4096
    while _need(m + 128, k) <= cap:
        m += 128
    assert _need(m, k) <= cap < _need(m + 128, k)
    codes, scales = _weights(db, n, k, 4, seed=9)
    x = torch.from_numpy(np.random.default_rng(9).normal(0, 1, (m, k)).astype(np.float32)).cuda()
    a, b = _both(db, x, codes, scales, n, 4)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    # the first shape past the array is refused
    m2 = m + 1
    while _need(m2, k) <= cap:
        m2 += 1
    x2 = torch.zeros((m2, k), device="cuda")
    y2 = torch.zeros((m2, n), device="cuda")
    rc = lib.db_linear_g64_noalloc(C.c_void_p(x2.data_ptr()), m2, k, C.c_void_p(codes.data_ptr()),
                                   C.c_void_p(scales.data_ptr()), n, 4, 8, 1, C.c_void_p(y2.data_ptr()), None)
    assert rc == -1 and lib.db_last_error_code().decode() == "SCRATCH_LIMIT"


def test_noalloc_allocates_nothing_after_the_first_call_and_reports_no_expiry(db):
    lib = db.load()
    m, k, n = 512, 1024, 1024
    codes, scales = _weights(db, n, k, 8, seed=4)
    x = torch.randn(m, k, device="cuda")
    y = torch.empty((m, n), device="cuda")
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)

    def call():
        rc = lib.db_linear_g64_noalloc(C.c_void_p(x.data_ptr()), m, k, C.c_void_p(codes.data_ptr()),
                                       C.c_void_p(scales.data_ptr()), n, 8, 8, 1, C.c_void_p(y.data_ptr()), stream)
        assert rc == 0, db._lib.last_error()

    call()  # set-up: looks up the array's address on this device
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    for _ in range(5):
        call()
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free_before
    assert lib.db_linear_noalloc_error_word() == 0
