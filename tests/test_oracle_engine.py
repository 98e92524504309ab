"""The oracle's Level-B step: properties the batched K+1 verification must have
(test infrastructure checks, CPU only)."""
import numpy as np
import pytest

from helpers import Cfg, OracleEngine, make_weights, prompts


@pytest.fixture(scope="module")
def tiny():
    cfg = Cfg()
    return cfg, make_weights(cfg)


def greedy_stream(cfg, w, prm, n_tokens, order=1):
    eng = OracleEngine(cfg, w, order=order)
    eng.prefill(prm)
    out = [[int(t)] for t in eng.pending()]
    while min(len(o) for o in out) < n_tokens:
        n, em = eng.step()
        for b in range(len(prm)):
            out[b] += [int(t) for t in em[b, : n[b]]]
    return [o[:n_tokens] for o in out], eng


def test_stream_independent_of_drafts(tiny):
    """With greedy verification and commit of the accepted prefix only (D7)
    the emitted stream is plain greedy decoding, whatever the drafts are."""
    cfg, w = tiny
    prm = prompts(2, [9, 14], cfg.n_vocab)
    ref, _ = greedy_stream(cfg, w, prm, 24)
    K = cfg.n_mtp_heads
    for wrong_at in range(K + 1):  # drafts correct up to `wrong_at`, then wrong
        eng = OracleEngine(cfg, w)
        eng.prefill(prm)
        out = [[int(t)] for t in eng.pending()]
        accepted = []
        while min(len(o) for o in out) < 24:
            d = np.zeros((2, K), np.int32)
            for b in range(2):
                nxt = ref[b][len(out[b]):len(out[b]) + K]
                nxt = nxt + [0] * (K - len(nxt))
                d[b] = nxt
                if wrong_at < K:
                    d[b, wrong_at] = (d[b, wrong_at] + 1) % cfg.n_vocab
            eng.set_drafts(d)
            n, em = eng.step()
            accepted.append(n.copy())
            for b in range(2):
                out[b] += [int(t) for t in em[b, : n[b]]]
        assert [o[:24] for o in out] == ref
        full = [a for a in accepted[:-1]]  # the last step may run past the reference
        assert all((a == wrong_at + 1).all() for a in full)


def test_positions_and_cache_sizes(tiny):
    cfg, w = tiny
    prm = prompts(3, [5, 11, 30], cfg.n_vocab, seed=4)
    eng = OracleEngine(cfg, w)
    eng.prefill(prm)
    assert list(eng.positions()) == [5, 11, 30]
    tot = np.array([5, 11, 30])
    for _ in range(4):
        n, _ = eng.step()
        tot += n
        assert list(eng.positions()) == list(tot)
    for b in range(3):
        k, ks, v, vs = eng.kv(b, 0, 0)
        assert len(k) == tot[b]


def test_device_order_close_to_reference_order(tiny):
    """The device's RMSNorm summation order changes logits only at float
    rounding level on the tiny model (both orders are restated in the oracle)."""
    cfg, w = tiny
    prm = prompts(2, [12, 7], cfg.n_vocab, seed=2)
    s1, e1 = greedy_stream(cfg, w, prm, 8, order=0)
    s2, e2 = greedy_stream(cfg, w, prm, 8, order=1)
    l1, l2 = e1.logits(), e2.logits()
    rel = np.abs(l1 - l2).max() / np.abs(l1).max()
    assert rel < 1e-3, rel


def test_eviction_and_pooling_semantics():
    """Small window: positions beyond it evict into the pool; the committed
    cache holds sink + pool + window entries in the reference's order."""
    cfg = Cfg(window_size=16, pool_block=4, max_context=512)
    w = make_weights(cfg)
    prm = prompts(1, [40], cfg.n_vocab, seed=5)
    eng = OracleEngine(cfg, w)
    eng.prefill(prm)
    L0 = 40
    k, ks, v, vs = eng.kv(0, 1, 0)
    n_pool = (L0 - 4 - 16) // 4
    assert len(k) == 4 + n_pool + 16
    for _ in range(3):
        eng.step()
    L1 = int(eng.positions()[0])
    k, ks, v, vs = eng.kv(0, 1, 0)
    assert len(k) == 4 + (L1 - 4 - 16) // 4 + 16


def test_layer_skip_counts():
    cfg = Cfg(n_layers=6, skip_enabled=1, skip_threshold=5.0)
    w = make_weights(cfg)
    prm = prompts(2, [10, 10], cfg.n_vocab, seed=6)
    eng = OracleEngine(cfg, w, skip_threshold=5.0)
    eng.prefill(prm)
    for _ in range(3):
        eng.step()
    comp, skipped = eng.skip_counts()
    assert skipped > 0 and comp > 0
