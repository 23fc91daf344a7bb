"""N-sharded linear on 2 GPUs (one process per GPU): the NCCL all-gather
path and the peer-memory all-gather of the C ABI (fused into the decode
GEMV epilogue) against the unsharded leafq_linear on the same GPU, bit for
bit.  Skipped on machines with fewer than two GPUs."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

# (tokens, rows, cols, bits, group, bias): decode GEMV shapes (fused
# epilogue), ragged rows, the tcgen05 prefill path, INT4 grouped, W4A32.
CASES = [
    (1, 5632, 2048, 8, 2048, True, 8),
    (1, 2561, 2048, 8, 2048, False, 8),
    (5, 1000, 512, 8, 512, True, 8),
    (200, 2048, 2048, 8, 2048, True, 8),
    (3, 514, 256, 4, 32, True, 8),
    (1, 1030, 4096, 4, 32, False, 32),
]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, failures):
    import torch.distributed as dist

    import leaf_b200 as lq
    import oracle
    from leaf_b200.parallel import PeerAllGather, RowShards, ShardedLinear

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    peer = None
    try:
        peer = PeerAllGather(max_elements=max(t * r for t, r, *_ in CASES))
        for ci, (tokens, rows, cols, bits, group, with_bias, abits) in enumerate(CASES):
            rng = np.random.default_rng(500 + ci)  # identical on every rank
            x_host = rng.standard_normal((tokens, cols)).astype(np.float32)
            w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
            payload, scales = oracle.quantize_weight(w, bits, group)
            bias = rng.standard_normal(rows).astype(np.float32) if with_bias else None
            full = lq.QuantWeight.from_host(payload, scales, rows, cols, bits, group, bias)
            x = torch.from_numpy(x_host).cuda()
            expect = lq.linear(x, full, abits).cpu().numpy()
            nccl = ShardedLinear.from_host(payload, scales, rows, cols, bits, group, bias,
                                           activation_bits=abits)
            fused = ShardedLinear(nccl.shard, rows, abits, peer=peer)
            for rep in range(3):  # the peer path alternates buffer halves
                for name, op in (("nccl", nccl), ("peer", fused)):
                    got = op(x).cpu().numpy()
                    if not np.array_equal(got.view(np.uint32), expect.view(np.uint32)):
                        failures.put(f"rank {rank} case {ci} {name} rep {rep}: differs")
            # Standalone gather of ragged slices.
            part = RowShards(rows, world)
            local = torch.from_numpy(expect[:, part.begin(rank):part.end(rank)].copy()).cuda()
            got = peer.run(local, part.begin(rank), rows).cpu().numpy()
            if not np.array_equal(got.view(np.uint32), expect.view(np.uint32)):
                failures.put(f"rank {rank} case {ci} allgather_run differs")
        # The fused decode linear inside a CUDA graph, replayed with new x.
        rows, cols = 2048, 2048
        rng = np.random.default_rng(9)
        w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
        payload, scales = oracle.quantize_weight(w, 8, cols)
        full = lq.QuantWeight.from_host(payload, scales, rows, cols, 8, cols)
        op = ShardedLinear(ShardedLinear.from_host(payload, scales, rows, cols, 8, cols).shard,
                           rows, 8, peer=peer)
        x = torch.zeros((1, cols), device="cuda")
        out = torch.empty((1, rows), device="cuda")
        op(x, out=out)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            op(x, out=out)
        for rep in range(4):
            x.copy_(torch.from_numpy(rng.standard_normal((1, cols)).astype(np.float32)))
            graph.replay()
            expect = lq.linear(x, full).cpu().numpy()
            if not np.array_equal(out.cpu().numpy().view(np.uint32), expect.view(np.uint32)):
                failures.put(f"rank {rank} graph replay {rep} differs")
        del graph
        if lq.load().leafq_device_status() != 0:
            failures.put(f"rank {rank}: device status {lq.load().leafq_last_error()}")
    except Exception as exc:  # noqa: BLE001
        failures.put(f"rank {rank}: {exc!r}")
    finally:
        if peer is not None:
            peer.close()
        dist.destroy_process_group()


def test_sharded_linear_two_gpus():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = torch.multiprocessing.get_context("spawn")
    failures = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, failures)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank did not finish"
    errors = []
    while not failures.empty():
        errors.append(failures.get())
    assert not errors, errors
    assert all(p.exitcode == 0 for p in procs)


def _decoder_rank_main(rank, world, port, path, prompts, new_tokens, failures, results):
    import torch.distributed as dist

    from leaf_b200.decoder import Decoder

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        got = {}
        for gather in ("nccl", "peer"):
            dec = Decoder(path, sequences=len(prompts), group=dist.group.WORLD, gather=gather)
            got[gather] = dec.generate_batch(prompts, new_tokens)
            if dec.device_status() != 0:
                failures.put(f"rank {rank} {gather}: device status")
            dec.close()
        results.put((rank, got))
    except Exception as exc:  # noqa: BLE001
        failures.put(f"rank {rank}: {exc!r}")
    finally:
        dist.destroy_process_group()


def test_sharded_decoder_two_gpus(tmp_path):
    """The batched decoder with every linear's rows split over 2 GPUs (each
    output all-gathered by NCCL, or in the decode steps by the peer-memory
    gather inside the step's CUDA graph): every sequence's tokens equal the
    unsharded decoder's, and the first is the reference's recorded request."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import decoder_fixture as fx  # tests/golden
    from test_gpu_decoder import _artifact
    from leaf_b200.decoder import Decoder

    path, golden = _artifact(tmp_path, "tiny_w8", fx.TINY)
    generated = golden["generated"].tolist()
    rng = np.random.default_rng(21)
    prompt = golden["prompt"].tolist()
    prompts = [prompt] + [rng.integers(0, fx.TINY.vocab, size=len(prompt)).tolist() for _ in range(2)]
    expect = Decoder(path, sequences=3).generate_batch(prompts, len(generated))
    assert expect[0] == generated
    ctx = torch.multiprocessing.get_context("spawn")
    failures, results = ctx.Queue(), ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_decoder_rank_main,
                         args=(r, 2, port, str(path), prompts, len(generated), failures, results))
             for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(2):
        try:
            rank, tokens = results.get(timeout=300)
            got[rank] = tokens
        except Exception:  # noqa: BLE001
            break
    for p in procs:
        p.join(timeout=60)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    errors = []
    while not failures.empty():
        errors.append(failures.get())
    assert not errors, errors
    assert not alive, "a rank did not finish"
    for rank in (0, 1):
        assert got.get(rank) == {"nccl": expect, "peer": expect}, rank
