"""Multi-rank host logic on CPU: cost-balanced sequence partition (the Python helper and the
library's esm_partition agree), the variable-size output gather, and the split of a mutational
scan's variants with the gather of their score rows, run as two gloo ranks (the same code runs
over NCCL on GPUs)."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp


def test_partition_is_contiguous_and_balanced():
    import sharding
    rng = np.random.default_rng(0)
    lengths = rng.integers(64, 513, size=32)
    for world in (1, 2, 4, 8):
        parts = sharding.partition(lengths, world, 480, 1920)
        assert len(parts) == world
        idx = [i for p in parts for i in p]
        assert idx == list(range(len(lengths)))
        costs = [sum(sharding.forward_cost(lengths[i], 480, 1920) for i in p) for p in parts]
        biggest = max(sharding.forward_cost(L, 480, 1920) for L in lengths)
        assert max(costs) - min(costs) <= 2 * biggest + 1e-6


def test_partition_more_ranks_than_sequences():
    import sharding
    parts = sharding.partition([100, 200], 4)
    assert sum(len(p) for p in parts) == 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, lengths, q):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(root / "codon-infer_b200"))
    import torch
    import torch.distributed as dist
    import sharding
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        parts = sharding.partition(lengths, world)
        mine = list(parts[rank])
        # Stand-in per-sequence output: the sequence index and length in each row of its block.
        rows = [torch.tensor([[i, j, lengths[i]] for j in range(lengths[i])], dtype=torch.float32) for i in mine]
        local = torch.cat(rows) if rows else torch.zeros((0, 3))
        full = sharding.gather_rows(local)
        if rank == 0:
            q.put(full.numpy())
    finally:
        dist.destroy_process_group()


def test_two_rank_gather_restores_sequence_order():
    lengths = [5, 17, 3, 9, 12]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, lengths, q)) for r in range(2)]
    for p in procs:
        p.start()
    full = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    expect = np.array([[i, j, L] for i, L in enumerate(lengths) for j in range(L)], dtype=np.float32)
    np.testing.assert_array_equal(full, expect)


def test_library_partition_matches_helper():
    import esm_b200
    import sharding
    rng = np.random.default_rng(1)
    for B in (0, 1, 7, 64, 300):
        lengths = rng.integers(1, 1025, size=B)
        for world in (1, 2, 3, 8):
            a = [list(r) for r in esm_b200.partition(lengths, world, 1280, 5120)]
            b = [list(r) for r in sharding.partition(lengths, world, 1280, 5120)]
            assert a == b


def _fake_scan_rows(positions):
    # Stand-in for the scan's per-position output (the 20 deltas and the entropy), a pure function
    # of the position, so any split must reassemble the same table.
    rows = [np.concatenate([np.full(20, p, np.float32) + np.arange(20, dtype=np.float32) / 32, [p * 0.5]])
            for p in positions]
    return np.stack(rows).astype(np.float32) if rows else np.zeros((0, 21), np.float32)


def _scan_worker(rank, world, port, n, q):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(root / "codon-infer_b200"))
    import torch
    import torch.distributed as dist
    import esm_b200
    import sharding
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        # The benchmark's split of the scan: equal-length variants, contiguous blocks.
        blocks = esm_b200.partition([302] * n, world, 640, 2560)
        mine = blocks[rank]
        full = sharding.gather_rows(torch.from_numpy(_fake_scan_rows(list(mine))))
        if rank == 0:
            q.put(([len(b) for b in blocks], full.numpy()))
    finally:
        dist.destroy_process_group()


def test_two_rank_scan_split_and_score_gather():
    n = 300
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_scan_worker, args=(r, 2, port, n, q)) for r in range(2)]
    for p in procs:
        p.start()
    sizes, full = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert sizes == [150, 150]
    np.testing.assert_array_equal(full, _fake_scan_rows(range(n)))
