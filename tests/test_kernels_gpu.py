"""Kernel-level parity on the GPU, called through the C ABI (include/pf_b200.h)
and compared with the CPU oracle on identical seeded inputs.

Integer results (int8 quantization, int32 accumulators) must be bit-exact,
and so must fp32 results whose operation order the kernels reproduce
(matmul_quantized's two-rounding epilogue).  Reductions whose order differs
are checked against a tolerance stated in each test."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

import pocketforge_b200 as pf  # noqa: E402
from pocketforge_b200 import _lib  # noqa: E402


@pytest.fixture(scope="module", autouse=True)
def need_device():
    if not torch.cuda.is_available() or pf.device_count() == 0:
        pytest.skip("no sm_100 device")


_alive = []  # device tensors must outlive the asynchronous calls that use them


@pytest.fixture(autouse=True)
def _release():
    yield
    torch.cuda.synchronize()
    _alive.clear()


def dev(a):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    _alive.append(t)
    return t


def p(t):
    return C.c_void_p(t.data_ptr())


def call(name, *args):
    _lib.check(getattr(_lib.lib(), name)(*args), name)
    torch.cuda.synchronize()


@pytest.mark.parametrize("M,K", [(1, 7), (5, 2048), (320, 2048), (64, 5632)])
def test_quantize_activation_rows_bitexact(olib, M, K):
    rng = np.random.default_rng(M + K)
    x = (rng.standard_normal((M, K)) * rng.choice([1e-3, 1.0, 1e6], (M, 1))).astype(np.float32)
    x[0, : min(3, K)] = 0
    if M > 1:
        x[1] = 0
    q, s = torch.zeros((M, K), dtype=torch.int8, device="cuda"), torch.zeros(M, device="cuda")
    call("pf_quantize_activation_rows", p(dev(x)), p(q), p(s), M, K, None)
    qh, sh = q.cpu().numpy(), s.cpu().numpy()
    for i in range(M):
        a, b = np.zeros(K, np.int8), np.zeros(1, np.float32)
        olib.po_quantize_activation_row(np.ascontiguousarray(x[i]), a, b, K)
        np.testing.assert_array_equal(qh[i], a)
        assert sh[i].view(np.uint32) == b.view(np.uint32)[0]


@pytest.mark.parametrize("n", [1, 33, 4096, 100001])
def test_dequant_bitexact(olib, n):
    src = np.random.default_rng(n).integers(0, 256, n, dtype=np.uint8)
    for fn, ofn in (("pf_dequant_q4_to_int8", "po_dequant_q4_to_int8"),
                    ("pf_dequant_q2_to_int8", "po_dequant_q2_to_int8"),
                    ("pf_dequant_ternary_to_int8", "po_dequant_ternary_to_int8")):
        out = torch.zeros(n, dtype=torch.int8, device="cuda")
        if fn == "pf_dequant_ternary_to_int8":
            call(fn, p(dev(src)), p(out), n, None)
        else:
            call(fn, p(dev(src)), p(out), C.c_float(1.0), n, None)
        want = np.zeros(n, np.int8)
        getattr(olib, ofn)(src, want, n)
        np.testing.assert_array_equal(out.cpu().numpy(), want)


@pytest.mark.parametrize("M,N,K", [(3, 4, 5), (1, 64, 128), (5, 96, 160), (64, 3072, 2048), (320, 2048, 5632),
                                   (333, 130, 300)])
def test_matmul_int8_bitexact(M, N, K):
    rng = np.random.default_rng(M * 7 + N + K)
    A = rng.integers(-127, 128, (M, K), dtype=np.int8)
    B = rng.integers(-128, 128, (N, K), dtype=np.int8)
    Cd = torch.zeros((M, N), dtype=torch.int32, device="cuda")
    call("pf_matmul_int8", p(dev(A)), p(dev(B)), p(Cd), M, N, K, None)
    np.testing.assert_array_equal(Cd.cpu().numpy(), A.astype(np.int64) @ B.astype(np.int64).T)


@pytest.mark.parametrize("M,N,K,given", [(2, 3, 4, False), (5, 3072, 2048, False), (17, 200, 384, True)])
def test_matmul_quantized_bitexact(olib, M, N, K, given):
    rng = np.random.default_rng(K)
    A = (rng.standard_normal((M, K)) * 5).astype(np.float32)
    B = rng.integers(-8, 8, (N, K), dtype=np.int8)
    ws = rng.uniform(0.5, 2, N).astype(np.float32)
    asc = (np.abs(A).max(1) / 127).astype(np.float32) if given else None
    Cd = torch.zeros((M, N), device="cuda")
    call("pf_matmul_quantized", p(dev(A)), p(dev(B)), p(Cd), M, N, K, p(dev(ws)),
         p(dev(asc)) if given else None, None)
    want = np.zeros(M * N, np.float32)
    olib.po_matmul_quantized(A.ravel(), B.ravel(), want, M, N, K, ws, asc.ctypes.data if given else None)
    np.testing.assert_array_equal(Cd.cpu().numpy().ravel().view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("qtype,lo,hi", [(1, -8, 8), (2, -2, 2), (3, -1, 2), (0, -128, 128)])
@pytest.mark.parametrize("M,N,K", [(5, 128, 2048), (320, 3072, 2048), (70, 64, 5632)])
def test_packed_projection_bitexact(qtype, lo, hi, M, N, K):
    """The engine's projection kernel over each packed weight format."""
    rng = np.random.default_rng(qtype * 100 + M)
    W = rng.integers(lo, hi, (N, K), dtype=np.int8)
    A = rng.integers(-127, 128, (M, K), dtype=np.int8)
    a_s = rng.uniform(1e-3, 1, M).astype(np.float32)
    w_s = rng.uniform(0.5, 2, N).astype(np.float32)
    nbytes = _lib.lib().pf_packed_weight_bytes(N, K, qtype)
    packed = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    call("pf_pack_weights", p(dev(W)), N, K, qtype, p(packed), None)
    Cd = torch.zeros((M, N), device="cuda")
    call("pf_gemm_packed", p(dev(A)), p(dev(a_s)), p(packed), p(dev(w_s)), qtype, p(Cd), M, N, K, None)
    acc = (A.astype(np.int64) @ W.astype(np.int64).T).astype(np.float32)
    want = (acc * a_s[:, None]).astype(np.float32) * w_s[None, :]
    np.testing.assert_array_equal(Cd.cpu().numpy().view(np.uint32), want.astype(np.float32).view(np.uint32))


@pytest.mark.parametrize("qtype,lo,hi", [(1, -8, 8), (2, -2, 2), (0, -128, 128)])
@pytest.mark.parametrize("M", [1, 5, 16])
@pytest.mark.parametrize("N,K", [(2048, 2048), (3072, 2048), (2048, 5632), (11264, 2048)])
def test_few_row_projection_bitexact(olib, qtype, lo, hi, M, N, K):
    """At most 16 activation rows run on the dp4a path (gemv.cu): the same
    int32 sums and matmul_quantized epilogue as the oracle, bit for bit."""
    rng = np.random.default_rng(qtype * 1000 + M * 7 + N + K)
    W = rng.integers(lo, hi, (N, K), dtype=np.int8)
    Af = (rng.standard_normal((M, K)) * 3).astype(np.float32)
    ws = rng.uniform(0.5, 2, N).astype(np.float32)
    A = np.zeros((M, K), np.int8)
    a_s = np.zeros(M, np.float32)
    for i in range(M):
        q, s = np.zeros(K, np.int8), np.zeros(1, np.float32)
        olib.po_quantize_activation_row(np.ascontiguousarray(Af[i]), q, s, K)
        A[i], a_s[i] = q, s[0]
    packed = torch.zeros(_lib.lib().pf_packed_weight_bytes(N, K, qtype), dtype=torch.uint8, device="cuda")
    call("pf_pack_weights", p(dev(W)), N, K, qtype, p(packed), None)
    Cd = torch.zeros((M, N), device="cuda")
    call("pf_gemm_packed", p(dev(A)), p(dev(a_s)), p(packed), p(dev(ws)), qtype, p(Cd), M, N, K, None)
    want = np.zeros(M * N, np.float32)
    olib.po_matmul_quantized(Af.ravel(), W.ravel(), want, M, N, K, ws, None)
    np.testing.assert_array_equal(Cd.cpu().numpy().ravel().view(np.uint32), want.view(np.uint32))


def test_pack_rejects_out_of_range():
    W = np.full((8, 128), 9, np.int8)  # 9 does not fit Q4
    packed = torch.zeros(_lib.lib().pf_packed_weight_bytes(8, 128, 1), dtype=torch.uint8, device="cuda")
    L = _lib.lib()
    flags = C.c_uint32()
    _lib.check(L.pf_read_device_error(C.byref(flags), 1), "clear")
    _lib.check(L.pf_pack_weights(p(dev(W)), 8, 128, 1, p(packed), None), "pack")
    torch.cuda.synchronize()
    # the range error is latched on the device (the engine loaders report it)
    _lib.check(L.pf_read_device_error(C.byref(flags), 1), "read")
    assert flags.value & 2


@pytest.mark.parametrize("M,n", [(1, 4), (7, 2048), (320, 2048)])
def test_rmsnorm_rows(olib, M, n):
    rng = np.random.default_rng(n)
    x = (rng.standard_normal((M, n)) * 30).astype(np.float32)
    w = rng.uniform(0.5, 1.5, n).astype(np.float32)
    out = torch.zeros((M, n), device="cuda")
    call("pf_rmsnorm_rows", p(out), p(dev(x)), p(dev(w)), M, n, None)
    got = out.cpu().numpy()
    for i in range(M):
        dev_order = np.zeros(n, np.float32)
        olib.po_rmsnorm(dev_order, np.ascontiguousarray(x[i]), w, n, 1e-6, 1)
        np.testing.assert_array_equal(got[i].view(np.uint32), dev_order.view(np.uint32))
        ref_order = np.zeros(n, np.float32)
        olib.po_rmsnorm(ref_order, np.ascontiguousarray(x[i]), w, n, 1e-6, 0)
        np.testing.assert_allclose(got[i], ref_order, rtol=1e-5, atol=1e-6)  # reference order: tolerance


@pytest.mark.parametrize("M,n", [(1, 5), (9, 1029), (4, 16384)])
def test_softmax_rows(olib, M, n):
    rng = np.random.default_rng(n)
    v = (rng.standard_normal((M, n)) * 4).astype(np.float32)
    d = dev(v)
    call("pf_softmax_rows", p(d), M, n, None)
    got = d.cpu().numpy()
    for i in range(M):
        want = np.ascontiguousarray(v[i]).copy()
        olib.po_softmax(want, n)
        # expf vs std::exp and the reference's sequential float sum (error ~sqrt(n) ulp)
        np.testing.assert_allclose(got[i], want, rtol=1e-4, atol=1e-9)


def test_argmax_first_max(olib):
    rng = np.random.default_rng(0)
    M, n = 64, 16384
    v = rng.standard_normal((M, n)).astype(np.float32)
    v[3, [10, 500, 9000]] = 100.0  # ties: first index wins
    v[4] = 0.0
    v[5, -1] = 50.0
    out = torch.zeros(M, dtype=torch.int32, device="cuda")
    call("pf_argmax_rows", p(dev(v)), M, n, p(out), None)
    got = out.cpu().numpy()
    for i in range(M):
        assert got[i] == olib.po_argmax(np.ascontiguousarray(v[i]), n)
    assert got[3] == 10 and got[4] == 0 and got[5] == n - 1


@pytest.mark.parametrize("shape", ["full", "ties", "ragged", "outlier", "flat"])
@pytest.mark.parametrize("mode", ["top_p", "top_k", "temp"])
def test_sampling_matches_oracle(olib, mode, shape):
    """Same logits and uniform draws: the sampled token must agree.  The sums
    are the reference's float sums in its order; the exponentials are double
    exp rounded to float, which can differ from the C library's float exp in
    rare halfway cases, so the bar is >= 99% agreement.  "ties" rows hold few
    distinct values (sort order on equal logits: ascending index; the value
    buckets overflow, so the radix sort runs); "ragged" rows have a vocabulary
    that is not a multiple of the sort's 1024-entry rounds and ten masked
    (-inf) entries; "outlier" rows carry one logit 45 deviations above the rest
    (a tied embedding's own-token logit: it lands in an end bucket); "full",
    "ragged" and "outlier" rows take the bucket sort, "flat" rows (half the
    entries one value) overflow a bucket and take the radix sort."""
    import oracle
    rng = np.random.default_rng(7)
    M, n = {"full": (256, 16384), "ties": (128, 16384), "ragged": (128, 5000), "outlier": (128, 16384),
            "flat": (64, 16384)}[shape]
    lg = (rng.standard_normal((M, n)) * rng.choice([0.5, 2.0, 8.0], (M, 1))).astype(np.float32)
    if shape == "ties":
        lg = np.round(lg * 2.0).astype(np.float32) * np.float32(0.5)
        lg[::4] = np.where(lg[::4] == 0.0, np.float32(-0.0), lg[::4])  # -0 and +0 compare equal
    if shape == "ragged":
        lg[:, rng.choice(n, 10, replace=False)] = -np.inf  # masked entries: zero terms
    if shape == "outlier":
        lg[np.arange(M), rng.integers(0, n, M)] = 45.0 * lg.std(axis=1)
    if shape == "flat":
        lg[:, rng.choice(n, n // 2, replace=False)] = np.float32(-1.0)
    u = rng.uniform(0, 1, M).astype(np.float32)
    cfg = {"top_p": (0.8, 0.95, 40, 0), "top_k": (0.8, 1.0, 40, 0), "temp": (0.8, 1.0, 0, 0)}[mode]
    sc = _lib.SamplingConfigC(*cfg)
    out = torch.zeros(M, dtype=torch.int32, device="cuda")
    call("pf_sample_rows", p(dev(lg)), M, n, C.byref(sc), p(dev(u)), p(out), None)
    got = out.cpu().numpy()
    oc = oracle.PfSamplingConfig(*cfg)
    want = np.array([olib.po_sample(np.ascontiguousarray(lg[i]), n, C.byref(oc), float(u[i])) for i in range(M)])
    assert ((got >= 0) & (got < n)).all()
    if shape in ("ties", "flat") and mode != "temp":
        # The reference's std::sort compares values only, so which of several
        # equal logits sits at a sorted position is its implementation's
        # choice; equal logits give equal terms and partial sums, so the draw
        # lands on the same position and the same value.
        rows = np.arange(M)
        assert (lg[rows, got] == lg[rows, want]).mean() >= 0.99, (lg[rows, got] != lg[rows, want]).sum()
    else:
        assert (got == want).mean() >= 0.99, (got != want).sum()


def test_empty_batches_are_noops():
    """Zero rows (or zero bytes) do nothing and return PF_OK, as the reference's
    row loops do; a bad shape is refused on the host (PF_ERR_INVALID) before
    any launch."""
    L = _lib.lib()
    f = torch.zeros(256, device="cuda")
    i8 = torch.zeros(256 * 128, dtype=torch.int8, device="cuda")
    i32 = torch.zeros(256, dtype=torch.int32, device="cuda")
    packed = torch.zeros(L.pf_packed_weight_bytes(64, 128, 1), dtype=torch.uint8, device="cuda")
    sc = _lib.SamplingConfigC(0.8, 0.95, 40, 0)
    calls = {
        "pf_quantize_activation_rows": (p(f), p(i8), p(f), 0, 128, None),
        "pf_dequant_q4_to_int8": (p(i8), p(i8), C.c_float(1.0), 0, None),
        "pf_dequant_ternary_to_int8": (p(i8), p(i8), 0, None),
        "pf_matmul_int8": (p(i8), p(i8), p(i32), 0, 64, 128, None),
        "pf_matmul_quantized": (p(f), p(i8), p(f), 0, 64, 128, p(f), None, None),
        "pf_gemm_packed": (p(i8), p(f), p(packed), p(f), 1, p(f), 0, 64, 128, None),
        "pf_pack_weights": (p(i8), 0, 128, 1, p(packed), None),
        "pf_rmsnorm_rows": (p(f), p(f), p(f), 0, 128, None),
        "pf_softmax_rows": (p(f), 0, 128, None),
        "pf_argmax_rows": (p(f), 0, 128, p(i32), None),
        "pf_sample_rows": (p(f), 0, 128, C.byref(sc), p(f), p(i32), None),
    }
    for name, args in calls.items():
        assert getattr(L, name)(*args) == 0, (name, L.pf_last_error())
    torch.cuda.synchronize()
    assert L.pf_matmul_int8(p(i8), p(i8), p(i32), 4, 0, 128, None) == 1  # N = 0: PF_ERR_INVALID
    assert L.pf_gemm_packed(p(i8), p(f), p(packed), p(f), 1, p(f), 4, 64, 100, None) == 1  # K % 128 != 0


def _scan_rows(rng, n):
    """Rows of terms for the sampler's sums: exponentials of flat and steep
    rows, values on a coarse grid (exact halfway cases everywhere), dyadic
    values, zeros and tiny terms, terms of half an ulp of the running sum,
    normalised quotients, plain uniforms."""
    rows = []
    for mode in range(8):
        for _ in range(6):
            U = rng.uniform(size=n)
            spread = 10.0 ** rng.uniform(-1, 2)
            if mode == 0:
                z = np.exp(-spread * U)
            elif mode == 1:
                z = rng.integers(0, 64, n) * 0.125
            elif mode == 2:
                z = np.ldexp(rng.integers(0, 4096, n).astype(np.float64), -rng.integers(0, 30, n))
            elif mode == 3:
                z = np.where(U < 0.1, 0.0, np.exp(-30.0 * rng.uniform(size=n)))
            elif mode == 4:
                z = np.exp(-5.0 * spread * U) * 1e-6
            elif mode == 5:
                z = np.ldexp(1.0, -24 - rng.integers(0, 3, n)) * (1 + rng.integers(0, 3, n))
                z[0] = 1.0
            elif mode == 6:
                z = np.exp(-spread * U)
                z = z / z.sum()
            else:
                z = U
            rows.append(z.astype(np.float32))
    return np.stack(rows)


def _scan_stops(rng, rows):
    tot = rows.astype(np.float64).sum(axis=1)
    us = (rng.uniform(size=len(rows)) * tot).astype(np.float32)
    ps = ((0.5 + 0.5 * rng.uniform(size=len(rows))) * tot).astype(np.float32)
    us[::7] = 0.0  # a draw of 0 stops at the first term
    return us, ps


@pytest.mark.parametrize("n", [16384, 5000, 37])
def test_exact_warp_scan_matches_serial_float_sums(n):
    """The sampler's normalising sum and cumulative scan are the reference's
    one-at-a-time float additions (src/engine.cpp:895-1003); the kernel
    computes them with one warp, exactly, from the rounding of each addition
    within a binade of the running sum (scan.cuh).  The device compares that
    with the plain float loop on every row: the full sum, the stop index and
    the stopping sum must agree in every bit, in index order (unsorted rows:
    temperature sampling) and on non-increasing rows (top-p / top-k, with the
    early exit once terms fall below a quarter ulp of the sum)."""
    rng = np.random.default_rng(n)
    rows = _scan_rows(rng, n)
    special = np.zeros((6, n), np.float32)
    special[0] = 1.0
    special[0, n // 3] = np.nan
    special[1] = 0.5
    special[1, n // 2] = np.inf
    special[2] = np.float32(1e-40)  # subnormal terms: the float path
    special[3] = np.float32(3e37)  # the sum overflows to inf
    special[4, n // 2] = 1.0  # zeros, one term
    special[5] = np.float32(2.0 ** -101)  # a sum that starts below 2^-100 and grows past it
    unsorted = np.concatenate([rows, special])
    us, ps = _scan_stops(rng, unsorted)
    us[len(rows):] = [0.3, 0.9, 1e-38, 1e38, 0.5, 1e-30]
    ps[len(rows):] = [0.9, 0.9, 1e-37, np.inf, 0.9, 1e-29]
    for terms, sorted_, uu, pp in ((unsorted, 0, us, ps), (-np.sort(-rows, axis=1), 1) + _scan_stops(rng, rows)):
        bad = C.c_uint32(0)
        _lib.check(_lib.lib().pf_check_ordered_scan(p(dev(terms)), len(terms), n, sorted_, p(dev(uu)), p(dev(pp)),
                                                    C.byref(bad)), "pf_check_ordered_scan")
        assert bad.value == 0, f"{bad.value} of {len(terms)} rows differ (sorted={sorted_})"


def test_branch_free_reciprocal_is_correctly_rounded():
    """The SwiGLU epilogues take 1 / (1 + exp(-g)) from a branch-free double
    Newton iteration (numerics.cuh) so that many of them interleave; it must
    equal the correctly rounded reciprocal (CUDA's __frcp_rn) for every float
    in [1, +inf], which the device checks exhaustively."""
    bad, first = C.c_uint64(0), C.c_uint32(0)
    _lib.check(_lib.lib().pf_check_reciprocal(C.byref(bad), C.byref(first)), "pf_check_reciprocal")
    assert bad.value == 0, f"{bad.value} mismatches, first at bits {first.value:#010x}"
