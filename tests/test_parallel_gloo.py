"""N-sharded linear host logic on CPU: partition, shard cutting and the
all-gather along N over a world-size-2 gloo group.

The per-rank compute here is the oracle (the CPU checker standing in for
the GPU kernel, which the gpu tests run); what is under test is that the
shards and the gather reassemble the unsharded result bit for bit.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from leaf_b200.parallel import RowGather, RowShards, shard_host_weight

# (tokens, rows, cols, bits, group, bias): one token even split (direct
# gather), ragged rows, several tokens, INT4 grouped, a shard with no rows.
CASES = [
    (1, 64, 96, 8, 96, True),
    (1, 37, 64, 8, 64, False),
    (3, 50, 128, 8, 128, True),
    (2, 33, 64, 4, 32, True),
    (1, 1, 32, 8, 32, False),
]


def test_row_shards_cover_rows_once():
    for rows in (0, 1, 7, 32, 37, 5632):
        for world in (1, 2, 3, 8):
            part = RowShards(rows, world)
            seen = []
            for r in range(world):
                seen.extend(range(part.begin(r), part.end(r)))
                assert part.count(r) in (rows // world, rows // world + 1)
            assert seen == list(range(rows))
            assert part.widest == (rows + world - 1) // world


def test_shard_host_weight_int4_rows():
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((9, 64)) * 0.02).astype(np.float32)
    payload, scales = oracle.quantize_weight(w, 4, 32)
    bias = rng.standard_normal(9).astype(np.float32)
    d, s, b, lo, hi = shard_host_weight(payload, scales, bias, 9, 64, 4, 32, 1, 2)
    assert (lo, hi) == (4, 9)
    assert d.shape == (5, 32) and s.shape == (5, 2) and b.shape == (5,)
    assert np.array_equal(d, payload.reshape(9, 32)[4:])
    assert np.array_equal(s, scales.reshape(9, 2)[4:])


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, failures):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        for ci, (tokens, rows, cols, bits, group, with_bias) in enumerate(CASES):
            rng = np.random.default_rng(100 + ci)  # identical on every rank
            x = rng.standard_normal((tokens, cols)).astype(np.float32)
            w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
            payload, scales = oracle.quantize_weight(w, bits, group)
            bias = rng.standard_normal(rows).astype(np.float32) if with_bias else None
            full = oracle.linear_int(x, payload, scales, bits, group, bias)
            d, s, b, lo, hi = shard_host_weight(payload, scales, bias, rows, cols, bits, group,
                                                rank, world)
            local = (oracle.linear_int(x, d, s, bits, group, b) if hi > lo
                     else np.zeros((tokens, 0), np.float32))
            got = RowGather(rows)(torch.from_numpy(np.ascontiguousarray(local))).numpy()
            if not np.array_equal(got.view(np.uint32), full.view(np.uint32)):
                failures.put(f"rank {rank} case {ci}: gathered output differs")
    except Exception as exc:  # noqa: BLE001
        failures.put(f"rank {rank}: {exc!r}")
    finally:
        dist.destroy_process_group()


def test_sharded_gather_world2_gloo():
    ctx = mp.get_context("spawn")
    failures = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, failures)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a gloo rank did not finish"
    errors = []
    while not failures.empty():
        errors.append(failures.get())
    assert not errors, errors
    assert all(p.exitcode == 0 for p in procs)


def test_row_gather_rejects_wrong_slice():
    pytest.importorskip("torch.distributed")
    # Partition arithmetic alone (no group needed): a slice of the wrong width
    # is refused before any collective is issued.
    gather = RowGather.__new__(RowGather)
    gather.group, gather.world, gather.rank = None, 2, 0
    gather.part = RowShards(10, 2)
    from leaf_b200 import LeafError
    with pytest.raises(LeafError):
        gather(torch.zeros((1, 4)))
