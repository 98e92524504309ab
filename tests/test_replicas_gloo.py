"""Host logic of the multi-GPU replicas (pocketforge_b200/replicas.py) with
two gloo ranks on the CPU: the sequence partition, the max-over-ranks device
time / summed tokens of a timed region, and the gather to rank 0."""
import json
import os
import socket
import tempfile

import pytest

from pocketforge_b200 import replicas


def test_sequence_slice_partitions_every_id_once():
    for g in (1, 7, 64, 65, 257):
        for world in (1, 2, 3, 8):
            blocks = [replicas.sequence_slice(g, world, r) for r in range(world)]
            assert blocks[0][0] == 0 and blocks[-1][1] == g
            for (a0, a1), (b0, _) in zip(blocks, blocks[1:]):
                assert a1 == b0
            sizes = [b - a for a, b in blocks]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        replicas.sequence_slice(8, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir):
    import datetime

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    try:
        w, r, lr = replicas.replica_env()
        g0, g1 = replicas.sequence_slice(10, w, r)
        ms, tok = replicas.step_totals(1.5 + r, 100 * (r + 1))
        got = replicas.gather_to_root({"rank": r, "seqs": [g0, g1]})
        with open(os.path.join(out_dir, f"r{rank}.json"), "w") as f:
            json.dump({"env": [w, r, lr], "slice": [g0, g1], "ms": ms, "tok": tok, "gathered": got}, f)
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks():
    import torch.multiprocessing as mp
    with tempfile.TemporaryDirectory() as td:
        mp.start_processes(_rank_main, args=(2, _free_port(), td), nprocs=2, join=True, start_method="spawn")
        r0 = json.load(open(os.path.join(td, "r0.json")))
        r1 = json.load(open(os.path.join(td, "r1.json")))
    assert r0["env"] == [2, 0, 0] and r1["env"] == [2, 1, 1]
    assert r0["slice"] == [0, 5] and r1["slice"] == [5, 10]
    for r in (r0, r1):  # every rank sees the slowest time and the total tokens
        assert r["ms"] == 2.5 and r["tok"] == 300
    assert r0["gathered"] == [{"rank": 0, "seqs": [0, 5]}, {"rank": 1, "seqs": [5, 10]}]
    assert r1["gathered"] is None
