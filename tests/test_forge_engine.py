""".squeeze loading and the C++ engines of the forge:: API (forge::Engine,
forge::BatchEngine) against the oracle's Level-B engine.

A small model (head_dim 64) is written as a .squeeze file with int8 (Q8)
blocks in the reference's block layout (per 32 values a float scale, then
the 32 int8 values; zstd frames), read back by the C++ loader
(pocketforge_b200/forge/squeeze.cpp), and driven by tests/cpp/
forge_engine_driver.cpp.  The oracle gets the same int8 values, row scales
(the mean of a row's block scales) and embedding scale (the mean row scale),
as the reference's WeightLoader::load_block_with_scales decodes them
(src/quant_format.cpp:345-388).  Greedy token streams must match.
"""
import os
import struct
import subprocess
import tempfile

import numpy as np
import pytest

from helpers import Cfg, OracleEngine

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def q8_block_stream(q, d):
    """q: int8 [n] (n a multiple of 32), d: float [n/32] -> the block stream."""
    out = bytearray()
    for b in range(len(d)):
        out += struct.pack("<f", float(d[b]))
        out += q[32 * b: 32 * b + 32].astype(np.int8).tobytes()
    return bytes(out)


def write_squeeze(path, cfg, mats):
    """mats: {(layer, matrix): (q int8 [rows][cols], d float32 [rows*cols/32])}."""
    import pyarrow as pa
    zstd = pa.Codec("zstd")
    blobs, index = [], []
    offset = 256
    for (l, m), (q, d) in mats.items():
        raw = q8_block_stream(q.ravel(), d)
        comp = zstd.compress(raw, asbytes=True)
        index.append(struct.pack("<6IB3xI", l, m, q.shape[0], q.shape[1], len(comp), len(raw), 0, offset))
        blobs.append(comp)
        offset += len(comp)
    header = bytearray(256)
    header[0:8] = b"FORGE\0\0\0"
    struct.pack_into("<10I2Q", header, 8, 1, len(mats), cfg.n_layers, cfg.n_embd, cfg.n_heads, cfg.n_kv_heads,
                     cfg.n_ff, cfg.n_vocab, 512, cfg.n_mtp_heads, offset, 32 * len(index))
    with open(path, "wb") as f:
        f.write(bytes(header))
        for b in blobs:
            f.write(b)
        for r in index:
            f.write(r)


def decoded(q, d, rows, cols):
    """int8 values, row scales and global scale as the reference loader returns them."""
    bpr = cols // 32
    rs = np.zeros(rows, np.float32)
    for b in range(len(d)):
        rs[b // bpr] = np.float32(rs[b // bpr] + d[b])
    rs = (rs / np.float32(bpr)).astype(np.float32)
    tot = np.float32(0)
    for r in range(rows):
        tot = np.float32(tot + rs[r])
    return q, rs, float(np.float32(tot / np.float32(rows)))


def test_squeeze_writer_layout(tmp_path):
    """The header and index records land where the reference's packed
    SqueezeHeader (256 bytes) and 32-byte WeightBlock records put them."""
    cfg = Cfg(n_layers=1)
    q = np.zeros((32, 64), np.int8)
    path = str(tmp_path / "m.squeeze")
    write_squeeze(path, cfg, {(0, 3): (q, np.ones(64, np.float32))})
    b = open(path, "rb").read()
    assert b[:5] == b"FORGE" and len(b) > 256 + 32
    version, nb, L, d = struct.unpack_from("<4I", b, 8)
    assert (version, nb, L, d) == (1, 1, 1, cfg.n_embd)
    index_off, index_size = struct.unpack_from("<2Q", b, 48)
    assert index_size == 32 and index_off + 32 == len(b)
    layer, m, rows, cols, cs, osz, qt = struct.unpack_from("<6IB", b, index_off)
    assert (layer, m, rows, cols, osz, qt) == (0, 3, 32, 64, 64 * 36, 0)


@pytest.mark.gpu
def test_cpp_engines_match_oracle():
    cfg = Cfg(n_mtp_heads=2, qtype=[0] * 7, emb_qtype=0, window_size=512, max_context=512)
    rng = np.random.default_rng(11)
    mats, weights = {}, {}
    for l in range(cfg.n_layers):
        for m in range(7):
            r, c = cfg.shape(m)
            q = rng.integers(-6, 7, (r, c), dtype=np.int8)
            d = rng.uniform(0.002, 0.02, r * c // 32).astype(np.float32)
            mats[(l, m)] = (q, d)
            a, rs, _ = decoded(q, d, r, c)
            weights[(l, m)] = (a, rs)
    qe = rng.integers(-127, 128, (cfg.n_vocab, cfg.n_embd), dtype=np.int8)
    de = rng.uniform(0.01, 0.03, cfg.n_vocab * cfg.n_embd // 32).astype(np.float32)
    mats[(0, 10)] = (qe, de)
    _, _, gs = decoded(qe, de, cfg.n_vocab, cfg.n_embd)
    weights["emb"] = (qe, gs)
    import oracle
    L = oracle.lib()
    d = cfg.n_embd
    for h in range(cfg.n_mtp_heads):  # the engines' MTP heads: seeded generator, seed 3
        parts = []
        for j in range(3):
            qq = np.zeros(d * d // 2, np.uint8)
            s = np.zeros(d, np.float32)
            L.po_synth_mtp_matrix(3, h, j, d, qq, s)
            parts += [qq, s]
        weights[("mtp", h)] = parts

    prompt = [5, 17, 200, 33, 9]
    max_new = 12
    with tempfile.TemporaryDirectory() as td:
        path = os.path.join(td, "m.squeeze")
        write_squeeze(path, cfg, mats)
        exe = os.path.join(td, "driver")
        lib_dir = os.path.join(ROOT, "pocketforge_b200")
        subprocess.run(["g++", "-O1", "-std=c++17", "-I" + os.path.join(ROOT, "include"),
                        os.path.join(ROOT, "tests", "cpp", "forge_engine_driver.cpp"), "-o", exe,
                        "-L" + lib_dir, "-l:libforge_b200.so", "-Wl,-rpath," + lib_dir], check=True)
        out = subprocess.run([exe, path, str(max_new), *map(str, prompt)], capture_output=True, text=True,
                             timeout=300)
    assert out.returncode == 0, out.stdout + out.stderr
    lines = {ln.split(":")[0]: ln.split(":", 1)[1].split() for ln in out.stdout.splitlines() if ":" in ln}

    o = OracleEngine(cfg, weights)
    o.prefill([prompt])
    want = [int(o.pending()[0])]
    while len(want) < max_new:
        n, em = o.step()
        want += [int(t) for t in em[0, : n[0]]]
    want = want[:max_new]
    assert [int(t) for t in lines["engine"]] == want
    assert [int(t) for t in lines["batch 0"]] == want
    assert [int(t) for t in lines["batch 2"]] == want
    assert int(lines["forward"][0]) == want[0] and int(lines["forward"][1]) == cfg.n_vocab


# (attention q, k, v, o, gate, up, down, embedding) quantization types:
# 0 Q8, 1 Q4, 2 Q2, 3 Q1.5 (the reference's per-matrix formats)
REF_FORMATS = {"q4": [1, 1, 1, 1, 1, 1, 1, 1], "q2_q15_mix": [1, 1, 1, 1, 2, 2, 3, 1],
               "q8": [0, 0, 0, 0, 0, 0, 0, 0]}


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", sorted(REF_FORMATS))
def test_reference_written_squeeze_matches_oracle(rlib, fmt):
    """A .squeeze file written by the reference's own Quantizer::quantize_matrix,
    compress_block and write_squeeze (oracle/_ref, compiled from its sources)
    from N(0, 0.02) weights, loaded by forge::Engine::load_model and
    forge::BatchEngine::load_squeeze.  The oracle gets exactly what the
    reference's WeightLoader::load_block_with_scales decodes from the same file
    (Q4 / Q2 streams decoded from their first byte, scales 1; Q8 row scales
    the mean of the block scales).  Greedy token streams must match."""
    qt = REF_FORMATS[fmt]
    cfg = Cfg(n_mtp_heads=2, qtype=qt[:7], emb_qtype=qt[7], window_size=512, max_context=512)
    rng = np.random.default_rng(21)
    shapes = [cfg.shape(m) for m in range(7)]
    mats = [rng.normal(0.0, 0.02, shapes[m]).astype(np.float32) for _ in range(cfg.n_layers) for m in range(7)]
    mats.append(rng.normal(0.0, 0.02, (cfg.n_vocab, cfg.n_embd)).astype(np.float32))
    flat = np.ascontiguousarray(np.concatenate([m.ravel() for m in mats]))
    prompt = [5, 17, 200, 33, 9, 120]
    max_new = 12
    import oracle
    L = oracle.lib()
    with tempfile.TemporaryDirectory() as td:
        path = os.path.join(td, "ref.squeeze")
        assert rlib.pfref_write_squeeze_model(path.encode(), cfg.n_layers, cfg.n_embd, cfg.n_heads, cfg.n_kv_heads,
                                              cfg.n_ff, cfg.n_vocab, 512, cfg.n_mtp_heads, flat,
                                              np.asarray(qt, np.int32)) == 0
        weights = {}

        def load(layer, m, rows, cols):
            out = np.zeros(rows * cols, np.int8)
            rs = np.zeros(rows, np.float32)
            gs = np.zeros(1, np.float32)
            assert rlib.pfref_load_block(path.encode(), layer, m, out, rs, gs, rows * cols) == rows * cols
            return out.reshape(rows, cols), rs, float(gs[0])

        for l in range(cfg.n_layers):
            for m in range(7):
                a, rs, _ = load(l, m, *shapes[m])
                weights[(l, m)] = (a, rs)
        qe, _, gs = load(0, 10, cfg.n_vocab, cfg.n_embd)
        weights["emb"] = (qe, gs)
        d = cfg.n_embd
        for h in range(cfg.n_mtp_heads):  # the engines' MTP heads: seeded generator, seed 3
            parts = []
            for j in range(3):
                qq = np.zeros(d * d // 2, np.uint8)
                s = np.zeros(d, np.float32)
                L.po_synth_mtp_matrix(3, h, j, d, qq, s)
                parts += [qq, s]
            weights[("mtp", h)] = parts
        exe = os.path.join(td, "driver")
        lib_dir = os.path.join(ROOT, "pocketforge_b200")
        subprocess.run(["g++", "-O1", "-std=c++17", "-I" + os.path.join(ROOT, "include"),
                        os.path.join(ROOT, "tests", "cpp", "forge_engine_driver.cpp"), "-o", exe,
                        "-L" + lib_dir, "-l:libforge_b200.so", "-Wl,-rpath," + lib_dir], check=True)
        out = subprocess.run([exe, path, str(max_new), "q=" + ",".join(map(str, qt)), *map(str, prompt)],
                             capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stdout + out.stderr
    lines = {ln.split(":")[0]: ln.split(":", 1)[1].split() for ln in out.stdout.splitlines() if ":" in ln}

    o = OracleEngine(cfg, weights)
    o.prefill([prompt])
    want = [int(o.pending()[0])]
    while len(want) < max_new:
        n, em = o.step()
        want += [int(t) for t in em[0, : n[0]]]
    want = want[:max_new]
    assert [int(t) for t in lines["engine"]] == want
    assert [int(t) for t in lines["batch 0"]] == want
    assert [int(t) for t in lines["batch 2"]] == want
