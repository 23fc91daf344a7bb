"""Persistent decode plans against op-by-op leafq_linear and the oracle."""
import numpy as np
import pytest
import torch

import leaf_b200 as lq
import oracle
from leaf_b200.decode import DecodePlan
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
    # (rows, cols) of a chain whose op j reads the first cols_j outputs of op
    # j-1 (a prefix view is contiguous for one token): chunked K (4800 >
    # 2048), fewer rows than blocks (64, 37), ragged rows, bias on every
    # other op.
    chain = [(2560, 2048), (4800, 2048), (64, 4800), (1000, 64), (37, 1000 // 16 * 16)]
    ops = []
    refs = []
    x = torch.from_numpy(x0).cuda()
    wait = -1
    for j, (rows, cols) in enumerate(chain):
        payload, scales, b, w = _weight(rng, rows, cols, bias=(j % 2 == 0))
        y = torch.empty((1, rows), dtype=torch.float32, device="cuda")
        xin = x[:, :cols]
        ops.append((xin, w, y, wait))
        refs.append((payload, scales, b, cols))
        x, wait = y, j
    plan = DecodePlan(ops)
    for _ in range(2):  # two runs: counters are reset between runs
        for _, _, y, _ in ops:
            y.fill_(float("nan"))
        plan.run()
        torch.cuda.synchronize()
        xin = x0
        for (payload, scales, b, cols), (_, w, y, _) in zip(refs, ops):
            expect = oracle.linear_int(xin[:, :cols], payload, scales, 8, cols, b)
            got = y.cpu().numpy()
            assert np.array_equal(got.view(np.uint32), expect.view(np.uint32))
            # and op-by-op leafq_linear on the same device input gives the same bits
            again = lq.linear(torch.from_numpy(np.ascontiguousarray(xin[:, :cols])).cuda(), w)
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
    assert lq.load().leafq_device_status() == 0


def test_plan_rejects_bad_ops(cuda_device):
    rng = np.random.default_rng(1)
    _, _, _, w = _weight(rng, 16, 64, False)
    x = torch.zeros((1, 64), device="cuda")
    y = torch.zeros((1, 16), device="cuda")
    with pytest.raises(lq.LeafError):
        DecodePlan([(x, w, y, 0)])  # an op may not wait on itself
    with pytest.raises(lq.LeafError):
        DecodePlan([(x, w, y, -1)], tokens=2)
