"""Pins the CPU oracle (oracle/pf_oracle.cpp) to the reference.

Two kinds of pins:
  * the known-answer cases of the reference's own tests
    (tests/test_matmul.cpp, tests/test_mtp.cpp, tests/test_layer_skip.cpp,
    tests/test_kv_cache.cpp of tundefund0-gif/pocketforge), restated as data;
  * bit-for-bit comparison with the reference's functions compiled from its
    sources (oracle/_ref/libpfref.so) on seeded random inputs.
"""
import ctypes as C
import os
import tempfile

import numpy as np
import pytest

import oracle


def f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


# --------------------------------------------------------------------------
# Known answers from the reference's tests
# --------------------------------------------------------------------------
def test_kat_matmul_int8(olib):
    # tests/test_matmul.cpp:53-81
    A = np.array([[1, 2, 3, 4, 5], [0, -1, -2, 1, 0], [2, -3, 1, -1, 2]], np.int8)
    B = np.array([[1, 0, -1, 2, 1], [-1, 2, 0, 1, -2], [0, 1, 2, -1, 0], [2, -1, 1, 0, -1]],
                 np.int8)
    Cm = np.zeros((3, 4), np.int32)
    olib.po_matmul_int8(A.ravel(), B.ravel(), Cm.ravel(), 3, 4, 5)
    np.testing.assert_array_equal(Cm, A.astype(np.int32) @ B.astype(np.int32).T)


def test_kat_dequant(olib):
    # tests/test_matmul.cpp:158-166 (Q4) and :180-189 (ternary)
    q4 = np.array([0x12, 0x34, 0x56, 0x78], np.uint8)
    out = np.zeros(8, np.int8)
    olib.po_dequant_q4_to_int8(q4, out, 8)
    assert list(out[:4]) == [-6, -7, -4, -5]
    t = np.array([0x00, 0x09, 0, 0], np.uint8)
    out = np.zeros(8, np.int8)
    olib.po_dequant_ternary_to_int8(t, out, 8)
    assert list(out[:4]) == [-1, -1, 0, 1]
    # Q2: codes 00,01,10,11 -> -2,-1,0,1 (comment block of tests/test_matmul.cpp:172-176)
    q2 = np.array([0xE4, 0x1B], np.uint8)
    out = np.zeros(8, np.int8)
    olib.po_dequant_q2_to_int8(q2, out, 8)
    assert list(out) == [-2, -1, 0, 1, 1, 0, -1, -2]


def test_kat_quantize_and_rmsnorm(olib):
    # tests/test_matmul.cpp:29-49
    src = f32([0.5, -1.0, 0.0, 0.75, -0.25, 1.0, -0.5, 0.1])
    dst = np.zeros(8, np.int8)
    sc = np.zeros(1, np.float32)
    olib.po_quantize_activation_row(src, dst, sc, 8)
    assert sc[0] > 0 and dst[2] == 0 and dst[0] > 0 and dst[1] < 0
    assert np.all(np.abs(dst * sc[0] - src) < 0.02)
    # tests/test_matmul.cpp:139-153
    x = f32([1, 2, 3, 4])
    w = f32([0.5, 1.0, 1.5, 2.0])
    out = np.zeros(4, np.float32)
    olib.po_rmsnorm(out, x, w, 4, 1e-6, 0)
    rms = np.sqrt(7.5)
    assert abs(out[0] - 0.5 / rms) < 0.01 and abs(out[3] - 8.0 / rms) < 0.01


def test_kat_softmax_argmax(olib):
    # tests/test_matmul.cpp:123-136 and tests/test_mtp.cpp:55-58
    v = f32([2.0, 1.0, 0.1, 0.5, 3.0])
    olib.po_softmax(v, 5)
    assert abs(v.sum() - 1.0) < 1e-3 and v[4] > v[0] > v[1] > v[3] > v[2]
    assert olib.po_argmax(f32([-1.0, 3.0, 0.5, -0.2, 2.0]), 5) == 1


def test_kat_layer_skip(olib, rlib):
    # tests/test_layer_skip.cpp:21-95 against both implementations
    L, d = 12, 8
    h1 = np.ones(d, np.float32)
    hd = np.full(d, 100.0, np.float32)
    o = olib.po_skip_create(L, d, 0.5)
    r = rlib.pfref_skip_create(L, d, 0.5, 4)
    try:
        seq = [(0, h1, False), (1, h1, False), (5, h1, None), (5, h1, True), (10, h1, False),
               (5, hd, False)]
        for layer, x, want in seq:
            a = olib.po_skip_should_skip(o, layer, x, 0)
            b = rlib.pfref_skip_should_skip(r, layer, x, d)
            assert a == b
            if want is not None:
                assert bool(a) == want
        assert rlib.pfref_skip_total(r) == 0  # skipped_count_ never increments
    finally:
        olib.po_skip_destroy(o)
        rlib.pfref_skip_destroy(r)


def test_kat_speculative_accept(rlib):
    # tests/test_mtp.cpp:61-69: MTPHeads::speculative_accept (unused by the engine)
    m = rlib.pfref_mtp_create(4, 64, 128)
    try:
        tl = np.full((4, 128), -1.0, np.float32)
        tl[0, 5] = tl[1, 5] = tl[3, 5] = 10.0
        tl[2, 7] = 10.0
        assert rlib.pfref_mtp_speculative_accept(m, 5, tl.ravel(), 4) == 2
    finally:
        rlib.pfref_mtp_destroy(m)


# --------------------------------------------------------------------------
# Bit-for-bit against the reference build
# --------------------------------------------------------------------------
@pytest.mark.parametrize("n", [1, 7, 64, 2048, 5632])
def test_pin_quantize_activation_row(olib, rlib, n):
    rng = np.random.default_rng(n)
    for scale in (1e-3, 1.0, 1e5):
        x = f32(rng.standard_normal(n) * scale)
        if n > 3:
            x[3] = 0.0
        a, b = np.zeros(n, np.int8), np.zeros(n, np.int8)
        sa, sb = np.zeros(1, np.float32), np.zeros(1, np.float32)
        olib.po_quantize_activation_row(x, a, sa, n)
        rlib.pfref_quantize_activation_row(x, b, sb, n)
        np.testing.assert_array_equal(a, b)
        assert sa.view(np.uint32)[0] == sb.view(np.uint32)[0]
    z = np.zeros(n, np.float32)
    a, sa = np.zeros(n, np.int8), np.zeros(1, np.float32)
    olib.po_quantize_activation_row(z, a, sa, n)
    assert sa[0] == 1.0 and not a.any()


@pytest.mark.parametrize("n", [1, 2, 3, 31, 32, 33, 1000, 4096])
def test_pin_dequant(olib, rlib, n):
    rng = np.random.default_rng(n)
    src = rng.integers(0, 256, n, dtype=np.uint8)
    for po_fn, ref_fn in (("po_dequant_q4_to_int8", "pfref_dequant_q4_to_int8"),
                          ("po_dequant_q2_to_int8", "pfref_dequant_q2_to_int8"),
                          ("po_dequant_ternary_to_int8", "pfref_dequant_ternary_to_int8")):
        a, b = np.zeros(n, np.int8), np.zeros(n, np.int8)
        getattr(olib, po_fn)(src, a, n)
        getattr(rlib, ref_fn)(src, b, n)
        np.testing.assert_array_equal(a, b)


@pytest.mark.parametrize("M,N,K", [(1, 64, 64), (5, 96, 160), (3, 17, 33)])
def test_pin_matmul(olib, rlib, M, N, K):
    rng = np.random.default_rng(M * N * K)
    A = rng.integers(-127, 128, (M, K), dtype=np.int8)
    B = rng.integers(-8, 8, (N, K), dtype=np.int8)
    c1, c2 = np.zeros(M * N, np.int32), np.zeros(M * N, np.int32)
    olib.po_matmul_int8(A.ravel(), B.ravel(), c1, M, N, K)
    rlib.pfref_matmul_int8(A.ravel(), B.ravel(), c2, M, N, K)
    np.testing.assert_array_equal(c1, c2)
    Af = f32(rng.standard_normal((M, K)) * 3)
    ws = f32(rng.uniform(0.5, 2.0, N))
    f1, f2 = np.zeros(M * N, np.float32), np.zeros(M * N, np.float32)
    olib.po_matmul_quantized(Af.ravel(), B.ravel(), f1, M, N, K, ws, None)
    rlib.pfref_matmul_quantized(Af.ravel(), B.ravel(), f2, M, N, K, ws, None)
    np.testing.assert_array_equal(f1.view(np.uint32), f2.view(np.uint32))


@pytest.mark.parametrize("n", [4, 64, 2048])
def test_pin_rmsnorm_softmax(olib, rlib, n):
    rng = np.random.default_rng(n)
    x = f32(rng.standard_normal(n) * 50)
    w = f32(rng.uniform(0.5, 1.5, n))
    a, b = np.zeros(n, np.float32), np.zeros(n, np.float32)
    olib.po_rmsnorm(a, x, w, n, 1e-6, 0)
    rlib.pfref_rmsnorm(b, x, w, n)
    np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))
    v1 = f32(rng.standard_normal(n) * 4)
    v2 = v1.copy()
    olib.po_softmax(v1, n)
    rlib.pfref_softmax(v2, n)
    np.testing.assert_array_equal(v1.view(np.uint32), v2.view(np.uint32))


@pytest.mark.parametrize("window,pool,n_pos,max_ctx", [(16, 4, 30, 128), (8, 3, 61, 64),
                                                      (32, 64, 200, 300), (2048, 64, 40, 4096)])
def test_pin_kv_cache(olib, rlib, window, pool, n_pos, max_ctx):
    """3-tier cache: sink, window eviction, fp64 pooling, scores and sums."""
    L, H, hd, sink = 2, 2, 8, 4
    rng = np.random.default_rng(window * 7 + n_pos)
    o = olib.po_kv_create(L, H, hd, sink, window, pool, max_ctx)
    r = rlib.pfref_kv_create(L, H, hd, sink, window, pool, max_ctx)
    try:
        for p in range(n_pos):
            for l in range(L):
                for h in range(H):
                    k = f32(rng.standard_normal(hd) * 3)
                    v = f32(rng.standard_normal(hd) * 3)
                    olib.po_kv_store(o, l, h, p, k, v)
                    rlib.pfref_kv_store(r, l, h, p, k, v)
            if p % 5 == 4 or p == n_pos - 1:
                for l in range(L):
                    for h in range(H):
                        q = f32(rng.standard_normal(hd))
                        s1 = np.zeros(max_ctx + 16, np.float32)
                        s2 = np.zeros(max_ctx + 16, np.float32)
                        n1 = olib.po_kv_scores(o, l, h, q, s1)
                        n2 = rlib.pfref_kv_scores(r, l, h, q, s2)
                        assert n1 == n2
                        np.testing.assert_array_equal(s1[:n1].view(np.uint32), s2[:n2].view(np.uint32))
                        p1 = f32(rng.uniform(0, 1, n1))
                        w1, w2 = np.zeros(hd, np.float32), np.zeros(hd, np.float32)
                        olib.po_kv_weighted_sum(o, l, h, p1, w1, n1)
                        rlib.pfref_kv_weighted_sum(r, l, h, p1, w2, n1)
                        np.testing.assert_array_equal(w1.view(np.uint32), w2.view(np.uint32))
        assert olib.po_kv_size(o) == rlib.pfref_kv_size(r)
    finally:
        olib.po_kv_destroy(o)
        rlib.pfref_kv_destroy(r)


def test_pin_layer_skip_sequence(olib, rlib):
    L, d = 22, 64
    rng = np.random.default_rng(5)
    o = olib.po_skip_create(L, d, 0.3)
    r = rlib.pfref_skip_create(L, d, 0.3, 4)
    try:
        base = f32(rng.standard_normal(d))
        for t in range(40):
            for l in range(L):
                x = f32(base + rng.standard_normal(d) * rng.choice([0.01, 0.2, 1.0]))
                assert olib.po_skip_should_skip(o, l, x, 0) == rlib.pfref_skip_should_skip(r, l, x, d)
    finally:
        olib.po_skip_destroy(o)
        rlib.pfref_skip_destroy(r)


@pytest.mark.parametrize("qtype", [0, 1, 2, 3])
def test_pin_quantizer_and_loader(olib, rlib, qtype):
    rows, cols = 24, 64 + 32 * (qtype == 0)
    rng = np.random.default_rng(qtype)
    data = f32(rng.standard_normal(rows * cols) * (0.02 if qtype else 0.5))
    if qtype == 3:
        data = f32(rng.standard_normal(rows * cols) * 0.5)  # ternary threshold is 0.35
    n = olib.po_quantize_matrix(data, rows, cols, qtype, None)
    assert n == rlib.pfref_quantize_matrix(data, rows, cols, qtype, None)
    a, b = np.zeros(n, np.uint8), np.zeros(n, np.uint8)
    olib.po_quantize_matrix(data, rows, cols, qtype, a.ctypes.data)
    rlib.pfref_quantize_matrix(data, rows, cols, qtype, b.ctypes.data)
    np.testing.assert_array_equal(a, b)
    w1 = np.zeros(rows * cols, np.int8)
    rs1 = np.zeros(rows, np.float32)
    g1 = np.zeros(1, np.float32)
    olib.po_loader_decode(a, n, rows, cols, qtype, w1, rs1, g1)
    w2 = np.zeros(rows * cols, np.int8)
    rs2 = np.zeros(rows, np.float32)
    g2 = np.zeros(1, np.float32)
    with tempfile.TemporaryDirectory() as td:
        rc = rlib.pfref_squeeze_roundtrip(os.path.join(td, "m.squeeze").encode(), data, rows, cols,
                                          qtype, w2, rs2, g2)
    assert rc == 0
    np.testing.assert_array_equal(w1, w2)
    np.testing.assert_array_equal(rs1, rs2)
    assert g1[0] == g2[0]


def test_pin_mtp(olib, rlib):
    H, d, V = 4, 64, 96
    rng = np.random.default_rng(11)
    q4 = np.zeros((H, 3, d, d // 2), np.uint8)
    sc = np.zeros((H, 3, d), np.float32)
    for h in range(H):
        for j in range(3):
            w = f32(rng.uniform(-1, 1, d * d) / np.sqrt(d))
            a, s = np.zeros(d * d // 2, np.uint8), np.zeros(d, np.float32)
            b, t = np.zeros(d * d // 2, np.uint8), np.zeros(d, np.float32)
            olib.po_mtp_quantize_q4(w, a, s, d, d)
            rlib.pfref_mtp_quantize_q4(w, b, t, d, d)
            np.testing.assert_array_equal(a, b)
            np.testing.assert_array_equal(s, t)
            q4[h, j] = a.reshape(d, d // 2)
            sc[h, j] = s
    emb = f32(rng.integers(-8, 8, (V, d)))
    hid = f32(rng.standard_normal(d))
    l1 = np.zeros(H * V, np.float32)
    l2 = np.zeros(H * V, np.float32)
    olib.po_mtp_forward(H, d, q4.ravel(), sc.ravel(), hid, emb.ravel(), V, l1, None)
    m = rlib.pfref_mtp_create(H, d, V)
    try:
        for h in range(H):
            rlib.pfref_mtp_set_head(m, h, q4[h, 0].ravel(), sc[h, 0], q4[h, 1].ravel(), sc[h, 1],
                                    q4[h, 2].ravel(), sc[h, 2])
        rlib.pfref_mtp_forward(m, hid, emb.ravel(), emb.size, l2)
    finally:
        rlib.pfref_mtp_destroy(m)
    np.testing.assert_array_equal(l1.view(np.uint32), l2.view(np.uint32))


@pytest.mark.parametrize("mode", ["top_p", "top_k", "temp", "greedy", "dispatch"])
def test_pin_sampling(olib, rlib, mode):
    rng = np.random.default_rng(3)
    eng = rlib.pfref_engine_create()
    try:
        for trial in range(40):
            n = int(rng.choice([5, 100, 16384]))
            lg = f32(rng.standard_normal(n) * rng.choice([0.5, 3.0, 20.0]))
            seed = int(rng.integers(0, 2**31))
            u = np.zeros(1, np.float32)
            olib.po_uniforms(seed, 1, u)
            rlib.pfref_seed_sampler(seed)
            T = float(rng.choice([0.3, 0.8, 1.5]))
            if mode == "top_p":
                p = float(rng.choice([0.5, 0.9, 0.95]))
                assert olib.po_sample_top_p(lg, n, p, T, u[0]) == rlib.pfref_sample_top_p(eng, lg, n, p, T)
            elif mode == "top_k":
                k = int(rng.choice([1, 5, 40]))
                assert olib.po_sample_top_k(lg, n, k, T, u[0]) == rlib.pfref_sample_top_k(eng, lg, n, k, T)
            elif mode == "greedy":
                assert olib.po_argmax(lg, n) == rlib.pfref_sample_greedy(eng, lg, n)
            else:
                cfg = oracle.PfSamplingConfig(T, 1.0 if mode == "temp" else float(rng.choice([0.9, 1.0])),
                                              40 if mode == "dispatch" else 0, 0)
                want = rlib.pfref_sample(eng, lg, n, cfg.temperature, cfg.top_p, cfg.top_k, 0)
                assert olib.po_sample(lg, n, C.byref(cfg), u[0]) == want
    finally:
        rlib.pfref_engine_destroy(eng)


def test_uniform_stream_matches_reference(olib, rlib):
    """po_uniforms reproduces the reference's draws: the k-th draw of
    std::mt19937(seed) through uniform_real_distribution<float>."""
    eng = rlib.pfref_engine_create()
    try:
        u = np.zeros(64, np.float32)
        olib.po_uniforms(1234, 64, u)
        # Reconstruct draw k via top-p over a 2-token distribution whose cut is
        # the whole vocabulary: token 0 is returned iff u <= p0.
        rlib.pfref_seed_sampler(1234)
        for k in range(64):
            lg = f32([0.0, 0.0])  # p0 = 0.5 after normalisation
            got = rlib.pfref_sample_top_p(eng, lg, 2, 0.999, 1.0)
            assert got == (0 if u[k] <= 0.5 else 1)
    finally:
        rlib.pfref_engine_destroy(eng)
