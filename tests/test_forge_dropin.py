"""The forge:: C++ API (include/forge/*.hpp) as a drop-in for the reference's.

The reference's own unit tests — tests/test_matmul.cpp, test_kv_cache.cpp,
test_mtp.cpp, test_layer_skip.cpp of tundefund0-gif/pocketforge — are compiled
unchanged against this repository's forge headers and linked to
libforge_b200.so (recipe: oracle/Makefile, target forge_tests; the binaries
are built where the reference checkout exists and travel in oracle/_ref).
On a GPU they must pass as they do against the reference's CPU library.

The device kernels behind the classes keep the reference's summation order;
their parity with the oracle is checked here through the C ABI.
"""
import ctypes as C
import os
import re
import subprocess

import numpy as np
import pytest

from pocketforge_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "oracle", "_ref", "forge_tests")
REF_TESTS = ["test_matmul", "test_kv_cache", "test_mtp", "test_layer_skip"]


def test_forge_symbols_exported():
    """Every forge:: entry point the headers declare is exported by the library."""
    out = subprocess.run(["nm", "-D", "--defined-only", "-C", _lib.LIB_PATH], capture_output=True, text=True).stdout
    for sym in ["forge::matmul_int8(", "forge::matmul_quantized(", "forge::quantize_activation_row(",
                "forge::dequant_q4_to_int8(", "forge::dequant_q2_to_int8(", "forge::dequant_ternary_to_int8(",
                "forge::dot_product(", "forge::softmax(", "forge::rmsnorm(",
                "forge::KVCache::KVCache(", "forge::KVCache::store(", "forge::KVCache::attention_scores(",
                "forge::KVCache::attention_weighted_sum(", "forge::KVCache::clear(", "forge::KVCache::memory_usage(",
                "forge::MTPHeads::MTPHeads(", "forge::MTPHeads::init_weights(", "forge::MTPHeads::forward(",
                "forge::MTPHeads::speculative_accept(", "forge::MTPHeads::argmax(", "forge::MTPHeads::memory_usage(",
                "forge::LayerSkipController::LayerSkipController(", "forge::LayerSkipController::should_skip_ffn(",
                "forge::LayerSkipController::record_layer_output(", "forge::LayerSkipController::new_token(",
                "forge::LayerSkipController::reset(", "forge::LayerSkipController::reset_anchor(",
                "forge::ModelConfig::check_memory_budget("]:
        assert sym in out, sym


@pytest.mark.gpu
@pytest.mark.parametrize("name", REF_TESTS)
def test_reference_unit_test_passes(name):
    exe = os.path.join(BIN, name)
    if not os.path.exists(exe):
        pytest.skip("reference unit tests not built (no reference checkout where the repository was built)")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    res = re.search(r"Results: (\d+) passed, (\d+) failed", r.stdout)
    assert r.returncode == 0 and res and int(res.group(2)) == 0, r.stdout[-3000:] + r.stderr[-2000:]


def _call(name, *args):
    _lib.check(getattr(_lib.lib(), name)(*args), name)


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _p(t):
    return C.c_void_p(t.data_ptr())


@pytest.mark.gpu
def test_sequential_kernels_match_host_order():
    """dot / q4 row product / skip delta: the reference's loops, bit for bit."""
    import torch
    L = _lib.lib()
    rng = np.random.default_rng(3)
    n = 777
    a = rng.standard_normal(n).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    out = torch.zeros(1, device="cuda")
    L.pf_dot_f32.argtypes = [C.c_void_p, C.c_void_p, C.c_uint32, C.c_void_p, C.c_void_p]
    L.pf_dot_f32.restype = C.c_int
    da, db = _dev(a), _dev(b)
    _lib.check(L.pf_dot_f32(_p(da), _p(db), n, _p(out), None), "pf_dot_f32")
    s = np.float32(0)
    for i in range(n):
        s = np.float32(s + np.float32(a[i] * b[i]))
    assert out.item() == s

    rows, cols = 9, 64
    w = rng.integers(0, 256, (rows, cols // 2), dtype=np.uint8)
    sc = rng.uniform(0.01, 0.1, rows).astype(np.float32)
    x = rng.standard_normal(cols).astype(np.float32)
    y = torch.zeros(rows, device="cuda")
    L.pf_gemv_q4_rows.argtypes = [C.c_void_p] * 4 + [C.c_uint32, C.c_uint32, C.c_void_p]
    L.pf_gemv_q4_rows.restype = C.c_int
    dx, dw, ds = _dev(x), _dev(w), _dev(sc)
    _lib.check(L.pf_gemv_q4_rows(_p(dx), _p(dw), _p(ds), _p(y), rows, cols, None), "pf_gemv_q4_rows")
    want = np.zeros(rows, np.float32)
    for r in range(rows):
        s = np.float32(0)
        for i in range(0, cols, 2):
            byte = int(w[r, i // 2])
            s = np.float32(s + np.float32(x[i] * np.float32(np.float32((byte & 15) - 8) * sc[r])))
            s = np.float32(s + np.float32(x[i + 1] * np.float32(np.float32((byte >> 4) - 8) * sc[r])))
        want[r] = s
    np.testing.assert_array_equal(y.cpu().numpy(), want)

    L.pf_skip_delta.argtypes = [C.c_void_p, C.c_void_p, C.c_uint32, C.c_void_p, C.c_void_p]
    L.pf_skip_delta.restype = C.c_int
    _lib.check(L.pf_skip_delta(_p(da), _p(db), n, _p(out), None), "pf_skip_delta")
    s = np.float32(0)
    for i in range(n):
        d = np.float32(a[i] - b[i])
        s = np.float32(s + np.float32(d * d))
    assert out.item() == np.float32(np.sqrt(np.float32(s / np.float32(n))))
