"""`bench.py --impl reference`: the reference's own CPU implementation of the
path, compiled from its sources into oracle/_ref/libpfref.so, timed on the
host cores.

TEST/BASELINE INFRASTRUCTURE ONLY (see oracle/__init__.py).

The reference runs its literal Engine::generate (src/engine.cpp:276-396):
one sequence per process (the engine is single-threaded and keeps a
file-static sampler, so processes, not threads, use the cores), as many
processes as there are host cores.  Its model file carries the 1B shape and
the tied embedding; the engine reads nothing else.
"""
from __future__ import annotations

import ctypes as C
import multiprocessing as mp
import os
import tempfile
import time

import numpy as np

PROMPT = 8
NEW_TOKENS = 8


def _quiet():
    # the reference engine prints progress on stdout; keep bench.py's stdout one JSON line
    fd = os.open(os.devnull, os.O_WRONLY)
    os.dup2(fd, 1)


def _worker(args):
    path, seed = args
    import oracle
    L = oracle.ref()
    L.pfref_literal_generate.restype = C.c_int
    L.pfref_literal_generate.argtypes = [C.c_char_p, C.c_void_p, C.c_uint32, C.c_uint32, C.c_void_p,
                                         C.POINTER(C.c_float)]
    rng = np.random.default_rng(seed)
    prompt = rng.integers(0, 16384, PROMPT).astype(np.int32)
    out = np.zeros(NEW_TOKENS + 8, np.int32)
    tps = C.c_float()
    t0 = time.perf_counter()
    n = L.pfref_literal_generate(path.encode(), prompt.ctypes.data, PROMPT, NEW_TOKENS, out.ctypes.data,
                                 C.byref(tps))
    return n, time.perf_counter() - t0, float(tps.value)


def run(args, cores: int, model) -> dict:
    import oracle
    L = oracle.ref()
    L.pfref_write_model.restype = C.c_int
    L.pfref_write_model.argtypes = [C.c_char_p] + [C.c_uint32] * 8 + [C.c_void_p, C.c_int]
    emb = np.zeros(model.n_vocab * model.n_embd, np.float32)
    oracle.lib().po_synth_normals(0, 0, 10, emb.size, emb)
    procs = max(1, min(cores, 64))
    with tempfile.TemporaryDirectory() as td:
        path = os.path.join(td, "model.squeeze")
        rc = L.pfref_write_model(path.encode(), model.n_layers, model.n_embd, model.n_heads, model.n_kv_heads,
                                 model.n_ff, model.n_vocab, 131072, model.n_mtp_heads, emb.ctypes.data, 1)
        if rc != 0:
            return {"impl": "reference", "unavailable": "could not write the reference model file"}
        ctx = mp.get_context("spawn")
        with ctx.Pool(procs, initializer=_quiet) as pool:
            pool.map(_worker, [(path, 999)] * min(procs, 2))  # warm-up: page the library in
            t0 = time.perf_counter()
            res = pool.map(_worker, [(path, 1 + i) for i in range(procs)])
            wall = time.perf_counter() - t0
    gen = sum(r[0] for r in res)
    value = gen / wall
    sample = (f"reference Engine::generate (oracle/_ref, built from the reference sources with -O2 "
              f"-ffp-contract=off): {procs} processes x 1 sequence, {PROMPT}-token prompt, {NEW_TOKENS} new tokens "
              f"each ({gen} generated in {wall:.1f} s wall); its own metric incl. prompt tokens averaged "
              f"{np.mean([r[2] for r in res]):.2f} tok/s per process")
    return {"impl": "reference", "metric": "accepted tok/s", "value": value, "unit": "tok/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "data": "synthetic", "dtype": "fp32 (CPU reference)",
            "config": {"workload": f"{args.config} on the host CPU: 1B model shape, bounded sample"},
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": procs, "kind": "reference", "sample": sample},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
