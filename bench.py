#!/usr/bin/env python
"""Benchmark of the batched MTP speculative-decode step (one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config config2] [--impl ours|reference]

A step is one speculative-decode step of every sequence on a GPU: K+1 verify
rows per sequence through the 22-layer Q4 model over the 3-tier int8 KV cache,
greedy acceptance, KV commit, and K new MTP drafts.  Default workload is the
batch-64, K=4 configuration (config2 of BASELINE.json) with a synthetic
random-init model (weights N(0,0.02) seed 0 through the reference's Quantizer
and loader; MTP heads seed 3) and uniform-random 512-token prompts.

Multi-GPU (torchrun, one rank per GPU): every rank holds a full replica and
its own 64 sequences (weak scaling, no collective in the step); the timed
region is bracketed by barriers and device synchronisation and the slowest
rank's device time is used.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "accepted tok/s"
UNIT = "tok/s"
MTP_PROBE_STEPS = 4  # untimed steps after the timed region that record per-head acceptance


def measure_int8_peak():
    """int8 tensor-core peak of this GPU, measured: the best of 10 cuBLASLt
    int8 GEMMs (torch._int_mm) of 8192^3, 2*8192^3 operations each."""
    import torch
    n = 8192
    a = torch.randint(-127, 128, (n, n), dtype=torch.int8, device="cuda")
    b = torch.randint(-127, 128, (n, n), dtype=torch.int8, device="cuda").t()
    best = float("inf")
    for i in range(13):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        torch._int_mm(a, b)
        e1.record()
        e1.synchronize()
        if i >= 3:
            best = min(best, e0.elapsed_time(e1))
    del a, b
    torch.cuda.empty_cache()
    return 2 * n ** 3 / (best * 1e-3) / 1e12


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.out = ""

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                self.out = ""

    def summary(self):
        rows = [r.split(", ") for r in self.out.strip().splitlines() if r.count(",") >= 8]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for name, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(rows)}


def make_prompts(ids, length, vocab, seed=1):
    """Uniform-random prompts, one seeded stream per global sequence id, so
    any split of the ids over ranks gives the same global workload."""
    return [np.random.default_rng((seed, int(i))).integers(0, vocab, length).astype(np.int32) for i in ids]


def kv_entry_bytes(model):
    return model.n_layers * model.n_kv_heads * (2 * model.head_dim + 8)


def attended_entries(model, ctx):
    """KV entries a query at context length ctx attends: the sinks, the
    window, and one pooled entry per pool_block positions beyond them (the
    3-tier cache, src/kv_cache.cpp:129-198)."""
    S, W, pb = model.sink_size, model.window_size, model.pool_block
    sink = min(ctx, S)
    win = min(max(ctx - S, 0), W)
    pool = max(ctx - S - W, 0) // pb
    return sink + win + pool


def algorithmic_bytes_per_step(model, n_seqs, ctx_avg, committed_per_step, K):
    """Bytes a verify step must move (weights, LM head, MTP heads, attended
    int8 KV, committed KV writes); activations stay on chip / in L2."""
    W = model.weight_bytes()
    E = model.n_vocab * model.n_embd // 2 if model.emb_qtype == 1 else model.n_vocab * model.n_embd
    H = K * 3 * model.n_embd * model.n_embd // 2 + K * 3 * model.n_embd * 4
    kv_read = n_seqs * attended_entries(model, ctx_avg) * kv_entry_bytes(model)
    kv_write = committed_per_step * kv_entry_bytes(model)
    return W + E + H + kv_read + kv_write


def profiled_traffic():
    """DRAM traffic figures measured by ncu, from the committed summaries in
    profiles/ (lines "bench-traffic: <what> <bytes>")."""
    out = {}
    d = os.path.join(os.path.dirname(os.path.abspath(__file__)), "profiles")
    if os.path.isdir(d):
        for f in sorted(os.listdir(d)):
            if f.endswith((".md", ".txt")):
                for ln in open(os.path.join(d, f)):
                    if ln.startswith("bench-traffic:"):
                        parts = ln.split()
                        if len(parts) >= 3:
                            out[parts[1]] = float(parts[2])
    return out


def projection_ops_per_step(model, M, B, K):
    """int8 MACs x2 of the layer projections (M rows), the tied unembed of
    the M rows and the MTP chain (B rows, K heads, 3 planes each)."""
    d, f, nq, nkv = model.n_embd, model.n_ff, model.n_heads * model.head_dim, model.n_kv_heads * model.head_dim
    per_layer = d * (nq + 2 * nkv) + nq * d + d * 2 * f + f * d
    layers = 2 * M * per_layer * model.n_layers
    unembed = 2 * 3 * M * model.n_vocab * d
    mtp = 2 * 3 * B * K * (3 * d * d + model.n_vocab * d)
    return layers + unembed + mtp


def cpu_baseline(model, prompt_len, seconds_budget=20.0):
    """The oracle port (CPU restatement of the Level-B step) timed on one core
    on a bounded sample of the workload: 1 sequence at the config's context —
    its prompt prefilled first, untimed, on all host cores — then decode
    steps on one thread until ~budget."""
    import ctypes as C

    import oracle
    from oracle import PfModelConfig
    L = oracle.lib()
    c = PfModelConfig()
    for name, _ in PfModelConfig._fields_:
        if name == "qtype":
            for i, q in enumerate(model.qtype):
                c.qtype[i] = q
        else:
            setattr(c, name, type(getattr(c, name))(getattr(model, name)))
    host = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    e = L.po_engine_create(C.byref(c))
    try:
        L.po_engine_load_synthetic(e, 0, 3, host)
        toks = make_prompts([0], prompt_len, model.n_vocab)[0]
        t_pre = time.perf_counter()
        L.po_engine_set_prefill_threads(e, host)
        L.po_engine_prefill(e, 1, toks, np.array([0, prompt_len], np.int64), None)
        L.po_engine_set_prefill_threads(e, 1)
        t_pre = time.perf_counter() - t_pre
        n = np.zeros(1, np.int32)
        em = np.zeros(model.n_mtp_heads + 1, np.int32)
        gen, steps, t0 = 0, 0, time.perf_counter()
        while True:
            L.po_engine_step(e, n.ctypes.data, em.ctypes.data)
            gen += int(n[0])
            steps += 1
            el = time.perf_counter() - t0
            if el > seconds_budget or steps >= 8:
                break
        return {"value": gen / el, "unit": UNIT, "cores": 1, "kind": "port",
                "sample": f"oracle port (oracle/pf_oracle.cpp, -O2, 1 thread): 1 sequence of the config at context "
                          f"{prompt_len} (its {prompt_len}-token prompt prefilled untimed on {host} host threads in "
                          f"{t_pre:.0f} s), {steps} decode steps, {gen} tokens in {el:.1f} s on the full 1B model"}
    finally:
        L.po_engine_destroy(e)


def reference_arm(args):
    """The reference's own CPU implementation (oracle/_ref, compiled from its
    sources) on the host cores."""
    import multiprocessing as mp
    import oracle
    if not oracle.ref_available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libpfref.so not built"}))
        return
    from oracle import refbench
    import pocketforge_b200 as pf
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    out = refbench.run(args, cores, pf.PRESETS[args.config]["model"])
    print(json.dumps(out))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--config", default="config2")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--seqs", type=int, default=0, help="override sequences per GPU (global with --strong)")
    ap.add_argument("--strong", action="store_true",
                    help="strong scaling: the config's sequences are the global batch, split over the GPUs")
    ap.add_argument("--prompt", type=int, default=0, help="override prompt length")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank == 0:
            reference_arm(args)
        return

    import torch
    import torch.distributed as dist

    import pocketforge_b200 as pf
    from pocketforge_b200 import replicas

    if world > 1:
        torch.cuda.set_device(local)
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    preset = pf.PRESETS[args.config]
    model = preset["model"]
    global_seqs = (args.seqs or preset["seqs"]) * (1 if args.strong else world)
    # Weak scaling: every rank owns the config's sequences of a global batch of
    # seqs * world; strong scaling: the config's batch is split over the ranks.
    # Rank r holds the contiguous block [g0, g1) of global ids.
    g0, g1 = replicas.sequence_slice(global_seqs, world, rank)
    seqs = g1 - g0
    plen = args.prompt or preset["prompt"]
    K = model.n_mtp_heads
    R = K + 1
    # room for: warm-up, timed steps, 2 kernel-timing steps, MTP_PROBE_STEPS
    max_pos = plen + (args.warmup + args.steps + 2 + MTP_PROBE_STEPS) * R + 8
    if model.max_context < max_pos:
        max_pos = model.max_context
    eng = pf.BatchEngine(model, seqs, max_pos, device=local)
    eng.load_synthetic(seed=0, mtp_seed=3, threads=7)
    sampling = preset.get("sampling")
    if sampling:
        eng.set_sampling(sampling["temperature"], sampling["top_p"], sampling["top_k"], False)
    prompts = make_prompts(range(g0, g1), plen, model.n_vocab)
    seeds = [sampling["seed"] + i for i in range(g0, g1)] if sampling else None

    # ---- end to end through the public API: pinned host prompts -> prefill
    # -> steps with every step's tokens read back to the host.
    e2e = None
    if not args.no_e2e:
        pinned = torch.from_numpy(np.concatenate(prompts)).pin_memory()
        host_prompts = np.split(pinned.numpy(), seqs)
        # Warm the engine through the same calls (first launch of each kernel,
        # step-graph capture), untimed; the timed prefill starts the sequences over.
        eng.prefill(host_prompts, seeds)
        for _ in range(args.warmup):
            eng.step()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        torch.cuda.nvtx.range_push("prefill")  # (a range for profilers; free otherwise)
        eng.prefill(host_prompts, seeds)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()  # (the first step needs the prefill's result anyway)
        t_pre = time.perf_counter() - t0
        got = seqs  # the first token comes out of prefill
        for _ in range(args.steps):
            n, em = eng.step()
            got += int(n.sum())
        torch.cuda.synchronize()
        el = time.perf_counter() - t0
        el, got = replicas.step_totals(el, got)
        e2e = {"value": got / el, "unit": UNIT, "prefill_ms": round(t_pre * 1e3, 2),
               "h2d_bytes_per_step": int(seqs * plen * 4 / max(1, args.steps)),
               "d2h_bytes_per_step": int(seqs * (R + 1) * 4),
               "includes": f"prefill of {seqs}x{plen} prompt tokens from pinned host memory + {args.steps} "
                           f"pf_engine_step calls, each reading the step's tokens back to the host, on an engine "
                           f"warmed by one untimed prefill + {args.warmup} steps"}

    # ---- device-resident timing
    eng.prefill(prompts, seeds)
    eng.run_steps(args.warmup)
    pos0 = eng.read_positions().astype(np.int64)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        torch.cuda.nvtx.range_push("pf_timed")  # ncu --nvtx-include pf_timed/ selects these launches
        ms = eng.run_steps(args.steps)
        torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    pos1 = eng.read_positions().astype(np.int64)
    tokens = int((pos1 - pos0).sum())
    launches = eng.launches_per_step() * args.steps * world  # every rank launches the same step graph
    # ---- per-kernel device time: a second, shorter timed region whose
    # captured step carries CUDA event pairs around every attention and
    # projection launch (they serialise the graph, so the step time above is
    # taken without them).
    eng.set_kernel_timing(True)
    eng.run_steps(2)
    (attn_ms, attn_n), (proj_ms, proj_n) = eng.kernel_times()
    eng.set_kernel_timing(False)
    # ---- MTP drafts on this synthetic model (untimed): the fraction of each
    # head's logit rows that are finite (the chained heads can overflow float
    # range, in the reference's arithmetic as well) and how often each draft
    # position is accepted.
    mtp_rows = eng.read_mtp_logits()
    mtp_finite = np.isfinite(mtp_rows).all(axis=-1).mean(axis=0)
    del mtp_rows
    accepted_at = np.zeros(K)
    for _ in range(MTP_PROBE_STEPS):
        n_em, _ = eng.step()
        accepted_at += [(n_em - 1 > h).mean() for h in range(K)]
    accepted_at /= MTP_PROBE_STEPS
    # ---- strong scaling beside weak (N > 1): the config's own batch split
    # over the ranks, on the same engines, same steps.
    strong = None
    if world > 1 and not args.strong:
        s0, s1 = replicas.sequence_slice(args.seqs or preset["seqs"], world, rank)
        sprompts = make_prompts(range(s0, s1), plen, model.n_vocab)
        sseeds = [sampling["seed"] + i for i in range(s0, s1)] if sampling else None
        eng.prefill(sprompts, sseeds)
        eng.run_steps(args.warmup)
        spos0 = eng.read_positions().astype(np.int64)
        dist.barrier()
        torch.cuda.synchronize()
        sms = eng.run_steps(args.steps)
        torch.cuda.synchronize()
        stok = int((eng.read_positions().astype(np.int64) - spos0).sum())
        sms_max, stok_all = replicas.step_totals(sms, stok)
        strong = {"value": stok_all / (sms_max * 1e-3), "unit": UNIT, "global_seqs": args.seqs or preset["seqs"],
                  "seqs_per_gpu": s1 - s0, "ms_per_step": sms_max / args.steps, "scaling": "strong"}
    int8_peak = measure_int8_peak() if rank == 0 else None
    ms_max, tokens_all = replicas.step_totals(ms, tokens)
    per_rank = replicas.gather_to_root({"rank": rank, "device_ms": ms, "tokens": tokens})
    step_ms = ms / args.steps
    ctx_avg = float(((pos0 + pos1) / 2).mean())
    committed = (pos1 - pos0).sum() / args.steps
    bytes_step = algorithmic_bytes_per_step(model, seqs, ctx_avg, committed, K)
    peak, peak_kind = load_peaks()
    achieved = bytes_step / (step_ms * 1e-3) / 1e9
    # Dominant kernel: attention over the int8 KV cache, one launch per layer,
    # all sequences; algorithmic bytes = attended entries x 8 kv heads x
    # (64 K + 64 V + 2 fp32 scales) for one layer.
    ctx_mid = float(((pos0 + pos1) / 2 + 2 * R).mean())  # the timing steps ran after the timed region
    attn_bytes = seqs * attended_entries(model, ctx_mid) * model.n_kv_heads * (2 * model.head_dim + 8)
    attn_us = attn_ms * 1e3 / max(1, attn_n)
    attn_gbs = attn_bytes / (attn_us * 1e-6) / 1e9
    proj_bytes = bytes_step - seqs * attended_entries(model, ctx_avg) * kv_entry_bytes(model) - \
        committed * kv_entry_bytes(model)
    proj_ops = projection_ops_per_step(model, seqs * R, seqs, K)
    traffic = profiled_traffic()
    clocks = clk.summary()
    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        cpu = cpu_baseline(model, min(plen, 512))  # (longer prompts: the first 512 tokens of the context)
    if rank == 0:
        line = {
            "metric": METRIC, "value": tokens_all / (ms_max * 1e-3), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
            "higher_is_better": True, "scaling": "strong" if args.strong else "weak", "vs_baseline": None,
            "dtype": "int8",
            "data": "synthetic",
            "config": {"workload": f"{args.config}: {seqs} sequences/GPU x {plen}-token uniform-random prompts, "
                                   f"MTP K={K} {'stochastic' if sampling else 'greedy'} verify of M={seqs * R} "
                                   f"rows/step, 1B Q4 model (22L, d2048, 32/8 heads, ffn 5632, vocab 16384)",
                       "seqs_per_gpu": seqs, "global_seqs": global_seqs, "prompt": plen,
                       "context_avg": ctx_avg, "window": model.window_size,
                       "l2": "no flush: weights (0.52 GB) + KV read per step exceed the 126 MB L2",
                       "parallelism": f"replicas x{world}"},
            "verify_step_us": step_ms * 1e3,
            "roofline": {"bound": "hbm", "achieved": attn_gbs, "peak": peak, "unit": "GB/s",
                         "frac": attn_gbs / peak, "peak_kind": peak_kind,
                         "traffic": traffic.get("attn_decode_per_seq_entry", 0.0) * seqs * attended_entries(model, ctx_mid) or None,
                         "kernel": "attn_decode_kernel: one layer's attention, all sequences x 8 kv heads",
                         "algorithmic_bytes_per_launch": attn_bytes, "launch_us": attn_us,
                         "launches_timed": attn_n,
                         "step": {"achieved": achieved, "frac": achieved / peak,
                                  "algorithmic_bytes_per_step": bytes_step,
                                  "traffic": traffic.get("step_per_seq_entry", 0.0) * seqs * attended_entries(model, ctx_avg)
                                  + traffic.get("step_fixed", 0.0) or None,
                                  "unit_of_work": "one verify step (CUDA graph launch)"},
                         "projections": {"ms_per_step": proj_ms, "launches": proj_n,
                                         "algorithmic_bytes": proj_bytes,
                                         "achieved_gbs": proj_bytes / (proj_ms * 1e-3) / 1e9,
                                         "int8_tops": proj_ops / (proj_ms * 1e-3) / 1e12,
                                         "int8_peak_tops": int8_peak,
                                         "int8_frac": proj_ops / (proj_ms * 1e-3) / 1e12 / int8_peak,
                                         "int8_peak_kind": "measured: best of 10 torch._int_mm 8192^3 on this GPU"}},
            "mtp": {"finite_frac_per_head": [round(float(x), 4) for x in mtp_finite],
                    "mtp_finite_frac": float(mtp_finite.mean()),
                    "accepted_frac_per_draft": [round(float(x), 4) for x in accepted_at],
                    "note": "synthetic heads (reference MTPHeads::quantize_q4 of seeded uniform weights) chained "
                            "h += down(silu(gate h) * up h); rows whose logits overflow float range give "
                            "arbitrary drafts, in the reference's arithmetic as well"},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "clocks": clocks,
            "gpu_launches": launches,
        }
        if world > 1:
            line["per_rank"] = per_rank
        if strong is not None:
            line["extra"] = {"strong": strong}
        if model.skip_enabled:
            comp, skp = eng.read_skip_counts()
            line["layer_skip"] = {"threshold": model.skip_threshold, "ffn_computed": comp, "ffn_skipped": skp,
                                  "skipped_frac": skp / max(1, comp + skp)}
        print(json.dumps(line))
    eng.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
