"""Persistent decode plans against op-by-op leafq_linear and the oracle."""
import numpy as np
import pytest
import torch

import leaf_b200 as lq
import oracle
from leaf_b200.decode import DecodeOp, DecodePlan
from leaf_b200.stack import LinearStack, StackShape

pytestmark = pytest.mark.gpu


def _weight(rng, n, k, bias):
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    payload, scales = oracle.quantize_weight(w, 8, k)
    b = (rng.standard_normal(n) * 0.01).astype(np.float32) if bias else None
    return payload, scales, b, lq.QuantWeight.from_host(payload, scales, n, k, 8, k, b)


def test_chain_matches_oracle_and_linear(cuda_device):
    rng = np.random.default_rng(77)
    x0 = rng.standard_normal((1, 2048)).astype(np.float32)
    x0[0, 3] = 25.0
    # (rows, cols, x_offset): op j reads cols outputs of op j-1 starting at
    # x_offset.  Covers chunked K (4800 > 2048), fewer rows than blocks (64,
    # 37), ragged rows, an offset slice, bias on every other op.
    chain = [(2560, 2048, 0), (4800, 2048, 512), (64, 4800, 0), (1000, 64, 0), (37, 992, 8)]
    ops, refs = [], []
    for j, (rows, cols, off) in enumerate(chain):
        payload, scales, b, w = _weight(rng, rows, cols, bias=(j % 2 == 0))
        y = torch.empty((1, rows), dtype=torch.float32, device="cuda")
        if j == 0:
            ops.append(DecodeOp(w, x=torch.from_numpy(x0).cuda(), y=y))
        else:
            ops.append(DecodeOp(w, wait=j - 1, x_offset=off, y=y))
        refs.append((payload, scales, b, cols, off))
    plan = DecodePlan(ops)
    for _ in range(3):  # repeated runs: each launch uses a fresh tag
        for op in ops:
            op.y.fill_(float("nan"))
        plan.run()
        torch.cuda.synchronize()
        xin = x0
        for (payload, scales, b, cols, off), op in zip(refs, ops):
            x_used = np.ascontiguousarray(xin[:, off:off + cols])
            expect = oracle.linear_int(x_used, payload, scales, 8, cols, b)
            got = op.y.cpu().numpy()
            assert np.array_equal(got.view(np.uint32), expect.view(np.uint32))
            again = lq.linear(torch.from_numpy(x_used).cuda(), op.weight)
            assert np.array_equal(again.cpu().numpy().view(np.uint32), expect.view(np.uint32))
            xin = expect
    assert lq.load().leafq_device_status() == 0
    plan.close()


def test_tinyllama_stack_persistent_equals_per_linear(cuda_device):
    shape = StackShape(layers=3)  # full widths, fewer layers
    stack = LinearStack(shape, seed=5)
    stack.run_eager(pdl=False)
    torch.cuda.synchronize()
    expect = stack.logits.cpu().numpy().copy()
    stack.capture_persistent()
    for _ in range(3):
        stack.logits.fill_(0.0)
        stack.graph.replay()
        torch.cuda.synchronize()
        assert np.array_equal(stack.logits.cpu().numpy().view(np.uint32), expect.view(np.uint32))
    # A new input changes every later output; the plan follows it.
    stack.x.copy_(torch.randn_like(stack.x))
    stack.run_eager(pdl=True)
    torch.cuda.synchronize()
    expect2 = stack.logits.cpu().numpy().copy()
    stack.graph.replay()
    torch.cuda.synchronize()
    assert np.array_equal(stack.logits.cpu().numpy().view(np.uint32), expect2.view(np.uint32))
    assert lq.load().leafq_device_status() == 0


def test_plan_rejects_bad_ops(cuda_device):
    rng = np.random.default_rng(1)
    _, _, _, w = _weight(rng, 16, 64, False)
    x = torch.zeros((1, 64), device="cuda")
    with pytest.raises(lq.LeafError):
        DecodePlan([DecodeOp(w, wait=0)])  # an op may not read its own output
    with pytest.raises(lq.LeafError):
        DecodePlan([DecodeOp(w, x=x), DecodeOp(w, wait=0, x_offset=2)])  # unaligned offset
    with pytest.raises(lq.LeafError):
        DecodePlan([DecodeOp(w, x=x)], tokens=2)
