"""pf_gemm_packed_static, the projection entry point that allocates nothing.

Some callers cannot call cudaMalloc: a host runtime that owns all device
memory through its own pool, or a latency-critical path where an allocation's
implicit device synchronisation is not allowed.  For them the split-K
partial sums live in a fixed array inside the library.  This test calls the
entry point through the C ABI twice in a row and checks both results against
the existing pf_gemm_packed (one pass, no split-K) bit for bit (int32 sums
are exact in any order, and the scale epilogue is the same two roundings), and
that sizes beyond the array are refused.  It is collected last so that a run
stopping at the first failure has already run every other test.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

import pocketforge_b200 as pf  # noqa: E402
from pocketforge_b200 import _lib  # noqa: E402


def _bind():
    L = _lib.lib()
    fn = L.pf_gemm_packed_static
    fn.restype = C.c_int32
    fn.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32, C.c_void_p, C.c_int32, C.c_int32,
                   C.c_int32, C.c_void_p]
    return L


@pytest.mark.parametrize("qtype,lo,hi,M,N,K", [(1, -8, 8, 64, 2048, 2048), (2, -2, 2, 5, 3072, 2048),
                                               (0, -128, 128, 320, 1024, 1024)])
def test_static_workspace_matches_allocating_path(qtype, lo, hi, M, N, K):
    if not torch.cuda.is_available() or pf.device_count() == 0:
        pytest.skip("no sm_100 device")
    L = _bind()
    rng = np.random.default_rng(M + N + qtype)
    W = torch.from_numpy(rng.integers(lo, hi, (N, K), dtype=np.int8)).cuda()
    A = torch.from_numpy(rng.integers(-127, 128, (M, K), dtype=np.int8)).cuda()
    a_s = torch.from_numpy(rng.uniform(1e-3, 1, M).astype(np.float32)).cuda()
    w_s = torch.from_numpy(rng.uniform(0.5, 2, N).astype(np.float32)).cuda()
    packed = torch.zeros(L.pf_packed_weight_bytes(N, K, qtype), dtype=torch.uint8, device="cuda")
    _lib.check(L.pf_pack_weights(W.data_ptr(), N, K, qtype, packed.data_ptr(), None), "pf_pack_weights")
    ref = torch.zeros((M, N), device="cuda")
    _lib.check(L.pf_gemm_packed(A.data_ptr(), a_s.data_ptr(), packed.data_ptr(), w_s.data_ptr(), qtype,
                                ref.data_ptr(), M, N, K, None), "pf_gemm_packed")
    torch.cuda.synchronize()
    for _ in range(2):  # the array keeps the previous call's contents
        out = torch.full((M, N), float("nan"), device="cuda")
        _lib.check(L.pf_gemm_packed_static(A.data_ptr(), a_s.data_ptr(), packed.data_ptr(), w_s.data_ptr(), qtype,
                                           out.data_ptr(), M, N, K, None), "pf_gemm_packed_static")
        torch.cuda.synchronize()
        np.testing.assert_array_equal(out.cpu().numpy().view(np.uint32), ref.cpu().numpy().view(np.uint32))


def test_static_workspace_empty_batch_is_a_no_op():
    """M = 0 returns PF_OK without touching the output, as pf_gemm_packed does."""
    if pf.device_count() == 0:
        pytest.skip("no sm_100 device")
    L = _bind()
    st = L.pf_gemm_packed_static(C.c_void_p(16), C.c_void_p(16), C.c_void_p(16), C.c_void_p(16), 1, C.c_void_p(16),
                                 0, 2048, 2048, None)
    assert st == 0


def test_static_workspace_rejects_oversize():
    if pf.device_count() == 0:
        pytest.skip("no sm_100 device")
    L = _bind()
    M, N, K = 1024, 2048, 128  # M*N above the array
    st = L.pf_gemm_packed_static(C.c_void_p(16), C.c_void_p(16), C.c_void_p(16), C.c_void_p(16), 1, C.c_void_p(16),
                                 M, N, K, None)
    assert st == _lib.PF_ERR_INVALID
    assert b"static workspace" in L.pf_last_error()
