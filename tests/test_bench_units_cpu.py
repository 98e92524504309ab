"""The per-unit figures behind bench.py's roofline numerator, pinned against
their derivation for the 1B model (no GPU): bytes per attended KV entry,
packed projection weights, the Q4 tied embedding and the MTP heads."""
import os
import sys

import pytest

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import bench  # noqa: E402
import pocketforge_b200 as pf  # noqa: E402

M1B = pf.BASE_1B


def test_kv_entry_bytes():
    # 8 kv heads x (64 K + 64 V int8 + two fp32 scales) per layer, 22 layers
    assert bench.kv_entry_bytes(M1B) == 22 * 8 * (64 + 64 + 8) == 23936


def test_packed_weight_bytes():
    d, f, q, kv = 2048, 5632, 32 * 64, 8 * 64
    params = (q + 2 * kv) * d + d * q + 2 * f * d + d * f  # QKV, O, gate + up, down
    rows = (q + 2 * kv) + d + 2 * f + d
    assert params == 45_088_768
    assert M1B.weight_bytes() == 22 * (params // 2 + 4 * rows)  # Q4: half a byte per weight, fp32 row scales
    q2 = pf.ModelConfig(qtype=[pf.QT_Q4] * 4 + [pf.QT_Q2, pf.QT_Q2, pf.QT_Q15])
    ffn = 3 * f * d
    assert M1B.weight_bytes() - q2.weight_bytes() == 22 * (ffn // 2 - ffn // 4)  # 2-bit FFN codes


def test_step_bytes_compose():
    n, ctx, committed, K = 64, 519, 64 * 3, 4
    got = bench.algorithmic_bytes_per_step(M1B, n, ctx, committed, K)
    emb = 16384 * 2048 // 2  # Q4 tied embedding read by the unembed GEMM
    mtp = K * 3 * 2048 * 2048 // 2 + K * 3 * 2048 * 4
    want = M1B.weight_bytes() + emb + mtp + (n * ctx + committed) * 23936
    assert got == want
    assert got == pytest.approx(1.34e9, rel=0.01)  # the figure quoted for config2 at context 519
