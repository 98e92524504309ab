"""Test helpers: tiny model configs, weights from the oracle's generator, and
a small wrapper over the oracle's Level-B engine (test infrastructure)."""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass, field, replace
from typing import Optional

import numpy as np

import oracle


@dataclass
class Cfg:
    n_layers: int = 2
    n_embd: int = 128
    n_heads: int = 2
    n_kv_heads: int = 1
    head_dim: int = 64
    n_ff: int = 256
    n_vocab: int = 256
    n_mtp_heads: int = 4
    sink_size: int = 4
    window_size: int = 2048
    pool_block: int = 64
    max_context: int = 4096
    rope_theta: float = 10000.0
    norm_eps: float = 1e-6
    skip_enabled: int = 0
    skip_threshold: float = 0.01
    qtype: list = field(default_factory=lambda: [1] * 7)
    emb_qtype: int = 1

    def oracle_c(self) -> oracle.PfModelConfig:
        c = oracle.PfModelConfig()
        for name, _ in oracle.PfModelConfig._fields_:
            if name == "qtype":
                for i, q in enumerate(self.qtype):
                    c.qtype[i] = q
            else:
                setattr(c, name, type(getattr(c, name))(getattr(self, name)))
        return c

    def shape(self, m):
        nq, nk = self.n_heads * self.head_dim, self.n_kv_heads * self.head_dim
        return [(nq, self.n_embd), (nk, self.n_embd), (nk, self.n_embd), (self.n_embd, nq),
                (self.n_ff, self.n_embd), (self.n_ff, self.n_embd), (self.n_embd, self.n_ff)][m]

    def product(self):
        import pocketforge_b200 as pf
        return pf.ModelConfig(**{k: getattr(self, k) for k in self.__dataclass_fields__})


def make_weights(cfg: Cfg, seed: int = 0, mtp_seed: int = 3):
    L = oracle.lib()
    w = {}
    for l in range(cfg.n_layers):
        for m in range(7):
            r, c = cfg.shape(m)
            a = np.zeros(r * c, np.int8)
            rs = np.zeros(r, np.float32)
            gs = np.zeros(1, np.float32)
            L.po_synth_matrix(seed, l, m, r, c, cfg.qtype[m], a, rs, gs)
            w[(l, m)] = (a.reshape(r, c), rs)
    emb = np.zeros(cfg.n_vocab * cfg.n_embd, np.int8)
    ers = np.zeros(cfg.n_vocab, np.float32)
    egs = np.zeros(1, np.float32)
    L.po_synth_matrix(seed, 0, 10, cfg.n_vocab, cfg.n_embd, cfg.emb_qtype, emb, ers, egs)
    w["emb"] = (emb.reshape(cfg.n_vocab, cfg.n_embd), float(egs[0]))
    d = cfg.n_embd
    for h in range(cfg.n_mtp_heads):
        parts = []
        for j in range(3):
            q = np.zeros(d * d // 2, np.uint8)
            s = np.zeros(d, np.float32)
            L.po_synth_mtp_matrix(mtp_seed, h, j, d, q, s)
            parts += [q, s]
        w[("mtp", h)] = parts
    return w


def host_threads() -> int:
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except AttributeError:
        return max(1, os.cpu_count() or 1)


class OracleEngine:
    """weights: a make_weights() dict, or None for the synthetic model of the
    benchmark configurations (seed 0 / MTP seed 3, the generator both sides
    restate).  Sequences run on `threads` host threads (results do not
    depend on it)."""

    def __init__(self, cfg: Cfg, weights, order: int = 1, sampling=None, skip_threshold=None, threads=None,
                 seed: int = 0, mtp_seed: int = 3):
        self.cfg = cfg
        self.L = oracle.lib()
        self._c = cfg.oracle_c()
        self.h = self.L.po_engine_create(C.byref(self._c))
        self.L.po_engine_set_order(self.h, order)
        self.L.po_engine_set_threads(self.h, threads or host_threads())
        if sampling is not None:
            self._s = oracle.PfSamplingConfig(*sampling)
            self.L.po_engine_set_sampling(self.h, C.byref(self._s))
        if skip_threshold is not None:
            self.L.po_engine_set_skip_threshold(self.h, skip_threshold)
        self.n = 0
        if weights is None:
            self.L.po_engine_load_synthetic(self.h, seed, mtp_seed, threads or host_threads())
            return
        for l in range(cfg.n_layers):
            for m in range(7):
                a, rs = weights[(l, m)]
                self.L.po_engine_set_matrix(self.h, l, m, np.ascontiguousarray(a.ravel()), rs)
        emb, gs = weights["emb"]
        self.L.po_engine_set_embedding(self.h, np.ascontiguousarray(emb.ravel()), gs)
        for h in range(cfg.n_mtp_heads):
            self.L.po_engine_set_mtp_head(self.h, h, *weights[("mtp", h)])
        self.n = 0

    def __del__(self):
        try:
            self.L.po_engine_destroy(self.h)
        except Exception:
            pass

    def prefill(self, prompts, seeds=None):
        toks = np.ascontiguousarray(np.concatenate([np.asarray(p, np.int32) for p in prompts]))
        offs = np.zeros(len(prompts) + 1, np.int64)
        offs[1:] = np.cumsum([len(p) for p in prompts])
        sd = np.ascontiguousarray(seeds, np.uint32) if seeds is not None else None
        self.L.po_engine_prefill(self.h, len(prompts), toks, offs, sd.ctypes.data if sd is not None else None)
        self.n = len(prompts)

    def step(self):
        K = self.cfg.n_mtp_heads
        n = np.zeros(self.n, np.int32)
        em = np.zeros((self.n, K + 1), np.int32)
        self.L.po_engine_step(self.h, n.ctypes.data, em.ctypes.data)
        return n, em

    def logits(self):
        a = np.zeros(self.n * (self.cfg.n_mtp_heads + 1) * self.cfg.n_vocab, np.float32)
        self.L.po_engine_read_logits(self.h, a)
        return a.reshape(self.n, self.cfg.n_mtp_heads + 1, self.cfg.n_vocab)

    def drafts(self):
        a = np.zeros(self.n * self.cfg.n_mtp_heads, np.int32)
        self.L.po_engine_read_drafts(self.h, a)
        return a.reshape(self.n, -1)

    def set_drafts(self, d):
        self.L.po_engine_set_drafts(self.h, np.ascontiguousarray(d, np.int32).ravel())

    def pending(self):
        a = np.zeros(self.n, np.int32)
        self.L.po_engine_read_pending(self.h, a)
        return a

    def positions(self):
        a = np.zeros(self.n, np.int32)
        self.L.po_engine_read_positions(self.h, a)
        return a

    def hidden(self):
        a = np.zeros(self.n * self.cfg.n_embd, np.float32)
        self.L.po_engine_read_hidden(self.h, a)
        return a.reshape(self.n, -1)

    def mtp_logits(self):
        a = np.zeros(self.n * self.cfg.n_mtp_heads * self.cfg.n_vocab, np.float32)
        self.L.po_engine_read_mtp_logits(self.h, a)
        return a.reshape(self.n, self.cfg.n_mtp_heads, -1)

    def skip_margin(self) -> float:
        """Smallest |delta - threshold| / threshold of any layer-skip decision so far."""
        return float(self.L.po_engine_skip_margin(self.h))

    def skip_counts(self):
        a, b = C.c_int64(), C.c_int64()
        self.L.po_engine_read_skip_counts(self.h, C.byref(a), C.byref(b))
        return a.value, b.value

    def kv(self, b, l, g, max_n=100000):
        hd = 64
        k = np.zeros(max_n * hd, np.int8)
        v = np.zeros(max_n * hd, np.int8)
        ks = np.zeros(max_n, np.float32)
        vs = np.zeros(max_n, np.float32)
        n = self.L.po_engine_read_kv(self.h, b, l, g, k, ks, v, vs, max_n)
        return k[: n * hd].reshape(n, hd), ks[:n], v[: n * hd].reshape(n, hd), vs[:n]

    def probe(self, b, token):
        lg = np.zeros(self.cfg.n_vocab, np.float32)
        hd = np.zeros(self.cfg.n_embd, np.float32)
        self.L.po_engine_probe_row(self.h, b, token, lg, hd)
        return lg, hd


def prompts(n, length, vocab, seed=1):
    rng = np.random.default_rng(seed)
    if np.isscalar(length):
        length = [length] * n
    return [rng.integers(0, vocab, int(L)).astype(np.int32) for L in length]
