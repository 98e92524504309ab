"""CPU-side checks of the product library: it loads, exports every entry point
include/pf_b200.h declares, refuses to run kernels without an sm_100 device,
and its synthetic-model generator matches the oracle's and the reference's."""
import ctypes as C
import os
import re

import numpy as np
import pytest

import pocketforge_b200 as pf
from pocketforge_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    hdr = open(os.path.join(ROOT, "include", "pf_b200.h")).read()
    return sorted(set(re.findall(r"^PF_API\s+[\w\s\*]+?\b(pf_\w+)\(", hdr, re.M)))


def test_library_exports_every_declared_symbol():
    lib = C.CDLL(_lib.LIB_PATH)
    names = declared_symbols()
    assert len(names) >= 35
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_no_device_is_an_error_not_a_fallback():
    if pf.device_count() > 0:
        pytest.skip("a device is present")
    L = _lib.lib()
    st = L.pf_argmax_rows(None, 1, 4, None, None)
    assert st in (_lib.PF_ERR_NO_DEVICE, _lib.PF_ERR_INVALID)
    h = C.c_void_p()
    c = pf.ModelConfig(n_layers=1, n_embd=128, n_heads=2, n_kv_heads=1, n_ff=256, n_vocab=256).to_c()
    assert L.pf_engine_create(C.byref(c), 1, 64, 0, C.byref(h)) == _lib.PF_ERR_NO_DEVICE


def test_packed_sizes():
    L = _lib.lib()
    assert L.pf_packed_weight_bytes(2048, 2048, 1) == 2048 * 2048 // 2
    assert L.pf_packed_weight_bytes(2048, 5632, 2) == 2048 * 5632 // 4
    assert L.pf_packed_weight_bytes(2048, 5632, 3) == 2048 * 5632 // 4
    assert L.pf_packed_weight_bytes(64, 128, 0) == 64 * 128
    assert L.pf_packed_weight_bytes(3, 5, 1) == 3 * 64  # K padded to one 128-wide block


@pytest.mark.parametrize("qtype,rows,cols", [(1, 64, 128), (2, 40, 96), (3, 32, 64), (0, 16, 64), (1, 7, 33)])
def test_synth_matches_oracle(olib, qtype, rows, cols):
    w, rs, gs = pf.synth_matrix(5, 2, 4, rows, cols, qtype)
    a = np.zeros(rows * cols, np.int8)
    b = np.zeros(rows, np.float32)
    g = np.zeros(1, np.float32)
    olib.po_synth_matrix(5, 2, 4, rows, cols, qtype, a, b, g)
    np.testing.assert_array_equal(w.ravel(), a)
    np.testing.assert_array_equal(rs, b)
    assert gs == g[0]


def test_synth_matches_reference_quantizer(olib, rlib):
    """The generator's int8 values are what the reference's Quantizer +
    WeightLoader produce from the same floats (zstd round trip included)."""
    import tempfile
    rows, cols = 48, 128
    for qtype in (1, 2, 3):
        f = np.zeros(rows * cols, np.float32)
        olib.po_synth_normals(0, 1, 6, rows * cols, f)
        w, rs, gs = pf.synth_matrix(0, 1, 6, rows, cols, qtype)
        out = np.zeros(rows * cols, np.int8)
        r2 = np.zeros(rows, np.float32)
        g2 = np.zeros(1, np.float32)
        with tempfile.TemporaryDirectory() as td:
            assert rlib.pfref_squeeze_roundtrip(os.path.join(td, "s.squeeze").encode(), f, rows, cols, qtype,
                                                out, r2, g2) == 0
        np.testing.assert_array_equal(w.ravel(), out)
        np.testing.assert_array_equal(rs, r2)


def test_synth_mtp_matches_oracle_and_reference(olib, rlib):
    d = 64
    q, s = pf.synth_mtp_matrix(3, 1, 2, d)
    a = np.zeros(d * d // 2, np.uint8)
    b = np.zeros(d, np.float32)
    olib.po_synth_mtp_matrix(3, 1, 2, d, a, b)
    np.testing.assert_array_equal(q.ravel(), a)
    np.testing.assert_array_equal(s, b)
