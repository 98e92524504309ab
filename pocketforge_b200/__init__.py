"""pocketforge_b200 — B200 (sm_100a) implementation of PocketForge's MTP
speculative-decode step, behind the C ABI of include/pf_b200.h.

Python host side: configuration presets and a thin `BatchEngine` over the
C ABI (device memory, kernels and CUDA graphs live in libpf_b200.so).
The C++ host side for the reference's own interfaces is include/forge/.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field, replace
from typing import List, Optional, Sequence

import numpy as np

from . import _lib
from ._lib import PfError, check, lib, ptr

QT_Q8, QT_Q4, QT_Q2, QT_Q15 = 0, 1, 2, 3
MAT_Q, MAT_K, MAT_V, MAT_O, MAT_GATE, MAT_UP, MAT_DOWN = range(7)


@dataclass
class ModelConfig:
    """pf_model_config (ModelConfig + KVCacheConfig + MTPConfig of the reference)."""

    n_layers: int = 22
    n_embd: int = 2048
    n_heads: int = 32
    n_kv_heads: int = 8
    head_dim: int = 64
    n_ff: int = 5632
    n_vocab: int = 16384
    n_mtp_heads: int = 4
    sink_size: int = 4
    window_size: int = 8192
    pool_block: int = 64
    max_context: int = 131072
    rope_theta: float = 10000.0
    norm_eps: float = 1e-6          # rmsnorm's constant (src/matmul_neon.cpp:234)
    skip_enabled: bool = False
    skip_threshold: float = 0.01    # ModelConfig::skip_threshold default
    qtype: Sequence[int] = field(default_factory=lambda: [QT_Q4] * 7)
    emb_qtype: int = QT_Q4

    def to_c(self) -> _lib.ModelConfigC:
        c = _lib.ModelConfigC()
        for name, _ in _lib.ModelConfigC._fields_:
            if name == "qtype":
                for i, q in enumerate(self.qtype):
                    c.qtype[i] = int(q)
            else:
                setattr(c, name, type(getattr(c, name))(getattr(self, name)))
        return c

    def matrix_shape(self, m: int):
        nq, nk = self.n_heads * self.head_dim, self.n_kv_heads * self.head_dim
        return [(nq, self.n_embd), (nk, self.n_embd), (nk, self.n_embd), (self.n_embd, nq),
                (self.n_ff, self.n_embd), (self.n_ff, self.n_embd), (self.n_embd, self.n_ff)][m]

    def weight_bytes(self) -> int:
        """Packed bytes of the transformer projections (HBM traffic per full pass)."""
        bits = {QT_Q4: 4, QT_Q2: 2, QT_Q15: 2, QT_Q8: 8}
        tot = 0
        for m in range(7):
            r, c = self.matrix_shape(m)
            tot += r * c * bits[self.qtype[m]] // 8 + 4 * r
        return tot * self.n_layers


# The synthetic ~1B model of the benchmark configurations.
BASE_1B = ModelConfig()

PRESETS = {
    # configs of the reference's benchmark description (model dims shared)
    "config1": dict(model=replace(BASE_1B, window_size=2048), seqs=1, prompt=128, gen=256),
    "config2": dict(model=replace(BASE_1B, window_size=8192, max_context=8192), seqs=64, prompt=512, gen=512),
    # positions >= max_context are not stored: room for the 512 generated
    # tokens and the verify rows after the 131072-token prompt
    "config3": dict(model=replace(BASE_1B, window_size=4096, max_context=131072 + 4096), seqs=16, prompt=131072,
                    gen=512),
    "config4": dict(model=replace(BASE_1B, qtype=[QT_Q4, QT_Q4, QT_Q4, QT_Q4, QT_Q2, QT_Q2, QT_Q15],
                                  skip_enabled=True), seqs=128, prompt=256, gen=256,
                    sampling=dict(temperature=0.8, top_k=40, top_p=0.95, seed=2)),
    "config5": dict(model=BASE_1B, seqs=256, prompt=2048, gen=128),
}


def device_count() -> int:
    return int(lib().pf_device_count())


class BatchEngine:
    """Batched MTP speculative decoding on one GPU (pf_engine_*)."""

    def __init__(self, cfg: ModelConfig, max_seqs: int, max_positions: int, device: int = 0):
        self.cfg = cfg
        self.max_seqs = max_seqs
        self.max_positions = max_positions
        self.K = cfg.n_mtp_heads
        self._c = cfg.to_c()
        h = C.c_void_p()
        check(lib().pf_engine_create(C.byref(self._c), max_seqs, max_positions, device, C.byref(h)),
              "pf_engine_create")
        self._h = h
        self.n_seqs = 0

    def close(self):
        if getattr(self, "_h", None) is not None and self._h.value:
            lib().pf_engine_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- weights ----
    def load_synthetic(self, seed: int = 0, mtp_seed: int = 3, threads: int = 7):
        check(lib().pf_engine_load_synthetic(self._h, C.byref(self._c), seed, mtp_seed, threads),
              "pf_engine_load_synthetic")

    def set_matrix(self, layer: int, m: int, w: np.ndarray, rs: np.ndarray):
        w = np.ascontiguousarray(w, np.int8)
        rs = np.ascontiguousarray(rs, np.float32)
        check(lib().pf_engine_set_matrix(self._h, layer, m, ptr(w), ptr(rs)), "pf_engine_set_matrix")

    def set_embedding(self, emb: np.ndarray, gscale: float = 1.0):
        emb = np.ascontiguousarray(emb, np.int8)
        check(lib().pf_engine_set_embedding(self._h, ptr(emb), float(gscale)), "pf_engine_set_embedding")

    def set_mtp_head(self, h: int, gq, gs, uq, us, dq, ds):
        a = [np.ascontiguousarray(x, t) for x, t in ((gq, np.uint8), (gs, np.float32), (uq, np.uint8),
                                                     (us, np.float32), (dq, np.uint8), (ds, np.float32))]
        check(lib().pf_engine_set_mtp_head(self._h, h, *[ptr(x) for x in a]), "pf_engine_set_mtp_head")

    def set_sampling(self, temperature=0.8, top_p=0.95, top_k=40, greedy=False):
        s = _lib.SamplingConfigC(temperature, top_p, top_k, 1 if greedy else 0)
        check(lib().pf_engine_set_sampling(self._h, C.byref(s)), "pf_engine_set_sampling")

    def set_skip_threshold(self, t: float):
        check(lib().pf_engine_set_skip_threshold(self._h, float(t)), "pf_engine_set_skip_threshold")

    # ---- decoding ----
    def prefill(self, prompts: Sequence[Sequence[int]], seeds: Optional[Sequence[int]] = None):
        toks = np.ascontiguousarray(np.concatenate([np.asarray(p, np.int32) for p in prompts]), np.int32)
        offs = np.zeros(len(prompts) + 1, np.int64)
        offs[1:] = np.cumsum([len(p) for p in prompts])
        sp = 0
        if seeds is not None:
            sd = np.ascontiguousarray(seeds, np.uint32)
            sp = ptr(sd)
        check(lib().pf_engine_prefill(self._h, len(prompts), ptr(toks), ptr(offs), sp or None), "pf_engine_prefill")
        self.n_seqs = len(prompts)

    def step(self):
        n = np.zeros(self.n_seqs, np.int32)
        em = np.zeros((self.n_seqs, self.K + 1), np.int32)
        check(lib().pf_engine_step(self._h, ptr(n), ptr(em)), "pf_engine_step")
        return n, em

    def set_drafts(self, drafts):
        d = np.ascontiguousarray(drafts, np.int32)
        check(lib().pf_engine_set_drafts(self._h, ptr(d)), "pf_engine_set_drafts")

    def run_steps(self, steps: int) -> float:
        check(lib().pf_engine_run_steps(self._h, steps), "pf_engine_run_steps")
        return self.last_ms()

    def launches_per_step(self) -> int:
        v = C.c_int32()
        check(lib().pf_engine_launches_per_step(self._h, C.byref(v)), "pf_engine_launches_per_step")
        return int(v.value)

    def last_ms(self) -> float:
        v = C.c_float()
        check(lib().pf_engine_last_ms(self._h, C.byref(v)), "pf_engine_last_ms")
        return float(v.value)

    def set_attention_splits(self, n: int) -> None:
        """CTAs per (sequence, kv head) in the verify attention; 0 = automatic."""
        check(lib().pf_engine_set_attention_splits(self._h, int(n)), "pf_engine_set_attention_splits")

    def set_kernel_timing(self, on: bool) -> None:
        check(lib().pf_engine_set_kernel_timing(self._h, 1 if on else 0), "pf_engine_set_kernel_timing")

    def kernel_times(self):
        """Device ms and launch counts of the last step: ((attention_ms, n),
        (projection_ms, n)); needs set_kernel_timing(True) before the step."""
        ms = (C.c_float * 2)()
        n = (C.c_int32 * 2)()
        check(lib().pf_engine_kernel_times(self._h, ms, n), "pf_engine_kernel_times")
        return (float(ms[0]), int(n[0])), (float(ms[1]), int(n[1]))

    def generate(self, prompts, max_new_tokens: int, seeds=None) -> List[List[int]]:
        """Prefill, then speculative steps until every sequence has max_new_tokens."""
        self.prefill(prompts, seeds)
        out = [[] for _ in prompts]
        pend = self.read_pending()
        for b in range(len(prompts)):
            out[b].append(int(pend[b]))
        while min(len(o) for o in out) < max_new_tokens:
            n, em = self.step()
            for b in range(len(prompts)):
                out[b].extend(int(t) for t in em[b, : n[b]])
        return [o[:max_new_tokens] for o in out]

    # ---- reads ----
    def _read(self, fn, shape, dtype):
        a = np.zeros(shape, dtype)
        check(getattr(lib(), fn)(self._h, ptr(a)), fn)
        return a

    def read_logits(self):
        return self._read("pf_engine_read_logits", (self.n_seqs, self.K + 1, self.cfg.n_vocab), np.float32)

    def read_drafts(self):
        return self._read("pf_engine_read_drafts", (self.n_seqs, self.K), np.int32)

    def read_pending(self):
        return self._read("pf_engine_read_pending", (self.n_seqs,), np.int32)

    def read_positions(self):
        return self._read("pf_engine_read_positions", (self.n_seqs,), np.int32)

    def read_hidden(self):
        return self._read("pf_engine_read_hidden", (self.n_seqs, self.cfg.n_embd), np.float32)

    def read_mtp_logits(self):
        return self._read("pf_engine_read_mtp_logits", (self.n_seqs, self.K, self.cfg.n_vocab), np.float32)

    def read_skip_counts(self):
        a, b = C.c_int64(), C.c_int64()
        check(lib().pf_engine_read_skip_counts(self._h, C.byref(a), C.byref(b)), "pf_engine_read_skip_counts")
        return a.value, b.value

    def read_log(self, cap: int):
        counts = np.zeros(self.n_seqs, np.int32)
        toks = np.zeros((self.n_seqs, cap), np.int32)
        check(lib().pf_engine_read_log(self._h, ptr(counts), ptr(toks), cap), "pf_engine_read_log")
        return counts, toks

    def read_kv(self, seq: int, layer: int, g: int, max_entries: int):
        k = np.zeros((max_entries, 64), np.int8)
        v = np.zeros((max_entries, 64), np.int8)
        ks = np.zeros(max_entries, np.float32)
        vs = np.zeros(max_entries, np.float32)
        n = C.c_int32()
        check(lib().pf_engine_read_kv(self._h, seq, layer, g, ptr(k), ptr(ks), ptr(v), ptr(vs), max_entries,
                                      C.byref(n)), "pf_engine_read_kv")
        return k[: n.value], ks[: n.value], v[: n.value], vs[: n.value]


def synth_matrix(seed: int, layer: int, m: int, rows: int, cols: int, qtype: int):
    w = np.zeros((rows, cols), np.int8)
    rs = np.zeros(rows, np.float32)
    gs = np.zeros(1, np.float32)
    check(lib().pf_synth_matrix(seed, layer, m, rows, cols, qtype, ptr(w), ptr(rs), ptr(gs)), "pf_synth_matrix")
    return w, rs, float(gs[0])


def synth_mtp_matrix(seed: int, head: int, which: int, d: int):
    q = np.zeros((d, d // 2), np.uint8)
    s = np.zeros(d, np.float32)
    check(lib().pf_synth_mtp_matrix(seed, head, which, d, ptr(q), ptr(s)), "pf_synth_mtp_matrix")
    return q, s


__all__ = ["ModelConfig", "BatchEngine", "PRESETS", "BASE_1B", "PfError", "device_count", "synth_matrix",
           "synth_mtp_matrix"]
