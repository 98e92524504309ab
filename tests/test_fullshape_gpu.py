"""GPU parity at the benchmarked shapes: the synthetic ~1B model of the
benchmark configurations (22 layers, d 2048, 32 query / 8 kv heads, FFN 5632,
tied vocabulary 16,384, 4 MTP heads) run by the GPU engine and by the oracle's
Level-B engine on the same seeded weights (both generate them from seed 0 /
MTP seed 3 through the reference's Quantizer and MTPHeads::quantize_q4) and
the same prompts.

The bars are those of test_engine_gpu.py: token streams and pending tokens
identical, logits and hidden states within 1e-3 of the row's largest
magnitude (1e-2 for a sequence whose int8 KV flipped at a rounding near-tie),
committed int8 KV >= 99.9% identical bytes, layer-skip counts exact when no
decision lies within rounding of its threshold.

MTP heads on this model: the chained heads grow the hidden state
quadratically (h += down(silu(gate h) * up h) with the reference's Q4 head
weights), and the oracle's third and fourth heads overflow float range at
d = 2048, as the reference's own float arithmetic does.  Drafts are compared
where the oracle's head logits are finite; the finite fraction is printed.

The oracle runs its sequences on all host threads (about 0.8 s per token
and thread at the full shape)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

from helpers import Cfg, make_weights, prompts  # noqa: E402
from test_engine_gpu import compare_kv, run_pair  # noqa: E402

import pocketforge_b200 as pf  # noqa: E402


@pytest.fixture(scope="module", autouse=True)
def need_device():
    if pf.device_count() == 0:
        pytest.skip("no sm_100 device")


def full_model(**over) -> Cfg:
    """The benchmark model's dimensions (pocketforge_b200.BASE_1B)."""
    base = dict(n_layers=22, n_embd=2048, n_heads=32, n_kv_heads=8, head_dim=64, n_ff=5632, n_vocab=16384,
                n_mtp_heads=4, sink_size=4, window_size=8192, pool_block=64, max_context=8192)
    base.update(over)
    return Cfg(**base)


def mtp_finite(o):
    """Fraction of (sequence, head) MTP logit rows that are finite, per head."""
    return np.isfinite(o.mtp_logits()).all(axis=-1).mean(axis=0)


def test_full_model_greedy_config2_shape():
    """config2's model and verify shape (K = 4, greedy), 4 sequences of
    14-26-token prompts, 2 verify steps."""
    cfg = full_model()
    prm = prompts(4, [14, 26, 20, 17], cfg.n_vocab, seed=1)
    g, o = run_pair(cfg, None, prm, 2)
    compare_kv(g, o, cfg, len(prm))
    fin = mtp_finite(o)
    print("config2 shape: MTP rows finite per head", fin.tolist())
    assert fin[0] == 1.0  # the first head never overflows on this model
    g.close()


def test_full_model_config1_shape():
    """config1's shape: one sequence (5 verify rows), a 2048-entry window.
    Every projection, the MTP chain and the 3-plane unembedding take the
    few-row path (gemv.cu); 3 verify steps.  With a single sequence, one int8
    rounding near-tie early in the context moves a larger share of the
    committed KV (a measured run: 733 of 675,840 bytes), so the byte bar is
    99.8% here."""
    cfg = full_model(window_size=2048)
    prm = prompts(1, [24], cfg.n_vocab, seed=13)
    g, o = run_pair(cfg, None, prm, 3)
    compare_kv(g, o, cfg, len(prm), min_same=0.998)
    g.close()


def test_full_width_long_context():
    """Full width (d 2048, 32/8 heads, FFN 5632, vocab 16,384) with two
    layers, so the prompts can reach 550-650 entries: attention with 4 query
    heads per kv head over many 32-entry blocks, the 5632-wide K-split down
    projection, the 3-digit-plane unembedding over 16,384 x 2048 and the MTP
    digit-plane chain at d = 2048."""
    cfg = full_model(n_layers=2)
    prm = prompts(3, [600, 555, 646], cfg.n_vocab, seed=11)
    g, o = run_pair(cfg, None, prm, 2)
    compare_kv(g, o, cfg, len(prm), scale_frac=0.995)
    print("full width, 2 layers: MTP rows finite per head", mtp_finite(o).tolist())
    g.close()


# Layer-skip threshold for the config4-shaped case.  Measured on the oracle
# (8 prompts of 12 tokens): the skipped fraction is 38% at 0.01, 60% at 0.02,
# 65% at 0.04 and saturates at 75% from 0.1 (layers 0, 1, 20 and 21 never
# skip); below 0.1 decisions crowd the threshold (smallest margins ~1e-3),
# at 0.15 the smallest margin is 0.22, so exact skip counts are a fair test.
CONFIG4_SKIP = 0.15


def test_full_model_config4_mix():
    """config4's mix at full size: Q2 gate/up, Q1.5 down, Q4 attention,
    layer skipping at a calibrated threshold, stochastic acceptance with
    temperature 0.8, top-k 40 (ignored by the top-p branch), top-p 0.95 and
    per-sequence seeds."""
    cfg = full_model(qtype=[1, 1, 1, 1, 2, 2, 3], skip_enabled=1, skip_threshold=CONFIG4_SKIP)
    prm = prompts(4, [12, 19, 15, 10], cfg.n_vocab, seed=2)
    g, o = run_pair(cfg, None, prm, 2, sampling=(0.8, 0.95, 40, 0), seeds=[2, 3, 4, 5],
                    skip_threshold=CONFIG4_SKIP)
    compare_kv(g, o, cfg, len(prm))
    comp, skip = o.skip_counts()
    print(f"config4 mix: FFNs computed {comp}, skipped {skip} ({skip / (comp + skip):.2f}), "
          f"smallest decision margin {o.skip_margin():.3g}")
    assert o.skip_margin() > 1e-3
    assert g.read_skip_counts() == o.skip_counts()
    assert 0.3 < skip / (comp + skip) < 0.8
    g.close()


def test_pooled_tier_window_4096():
    """config3's tier structure (4 sinks, a 4096-entry window, pool blocks of
    64) with contexts past the window, so every attention also reads pooled
    history entries and the verify rows evict into the fp64 pooling
    accumulators.  Two layers, d 512 with 8 query / 2 kv heads (4 query heads
    per kv head, as at config3)."""
    cfg = Cfg(n_layers=2, n_embd=512, n_heads=8, n_kv_heads=2, n_ff=1024, n_vocab=1024, window_size=4096,
              pool_block=64, max_context=8192, n_mtp_heads=4)
    w = make_weights(cfg, seed=7)
    prm = prompts(3, [4400, 5020, 4731], cfg.n_vocab, seed=12)
    g, o = run_pair(cfg, w, prm, 2)
    compare_kv(g, o, cfg, len(prm), scale_frac=0.995)
    g.close()
