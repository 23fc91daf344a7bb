"""leafq_linear_w8a8_static_scratch, the entry point that allocates nothing.

It exists for callers that cannot allocate device memory (a plugin whose
host runtime owns all of it, a serving loop that may not call the allocator
after start-up, a fixed-budget embedder) and so cannot pass leafq_linear a
workspace.  Its scratch is one library-owned device array shared by every
call; each call overwrites what it uses, so two calls in a row on one stream
must each give exactly leafq_linear's result.  This file is collected last
so that a run stopping at the first failure has run every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

import leaf_b200 as lq
import oracle
from leaf_b200 import _lib

pytestmark = pytest.mark.gpu


def _weight(rng, n, k, bias=True):
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    payload, scales = oracle.quantize_weight(w, 8, k)
    b = (rng.standard_normal(n) * 0.01).astype(np.float32) if bias else None
    return lq.QuantWeight.from_host(payload, scales, n, k, 8, k, b)


def _static_call(x, w):
    y = torch.empty((x.shape[0], w.rows), dtype=torch.float32, device=x.device)
    stream = torch.cuda.current_stream(x.device).cuda_stream
    status = _lib.load().leafq_linear_w8a8_static_scratch(
        stream, x.data_ptr(), x.shape[0], w.cols, w.data.data_ptr(), w.scales.data_ptr(), w.rows,
        None if w.bias is None else w.bias.data_ptr(), y.data_ptr(), 0)
    return status, y


def _check_twice(cases, seed):
    rng = np.random.default_rng(seed)
    for tokens, cols, rows, bias in cases:
        w = _weight(rng, rows, cols, bias)
        x = torch.from_numpy(rng.standard_normal((tokens, cols)).astype(np.float32)).cuda()
        expected = lq.linear(x, w)
        status, y = _static_call(x, w)
        assert status == _lib.LEAFQ_OK, _lib.load().leafq_last_error()
        torch.cuda.synchronize()
        got, want = y.cpu().numpy(), expected.cpu().numpy()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (tokens, cols, rows)
    assert _lib.load().leafq_device_status() == _lib.LEAFQ_OK


def test_static_scratch_matches_workspace_linear_twice(cuda_device):
    # Two calls in a row with different shapes: the second reuses (and must
    # fully overwrite) the scratch the first one filled.
    _check_twice(((300, 2048, 1000, True), (64, 1024, 512, False)), 4242)


def test_static_scratch_decode_sizes_match_linear(cuda_device):
    # 1-8 tokens take leafq_linear's decode GEMV (no scratch); a width the
    # GEMV does not take goes through the scratch and the generic kernel.
    # Each shape twice in a row, bit for bit against leafq_linear.
    _check_twice(((1, 2048, 5632, True), (1, 2048, 5632, True), (8, 1040, 300, True), (8, 1040, 300, False),
                  (5, 12288, 96, True), (5, 12288, 96, True)), 99)


def test_static_scratch_accepts_the_exact_limits(cuda_device):
    # tokens * cols exactly 8 MiB of codes, and exactly 16384 tokens.
    _check_twice(((2048, 4096, 48, True), (16384, 512, 40, False)), 5)


def test_static_scratch_rejects_oversized_calls(cuda_device):
    rng = np.random.default_rng(7)
    w = _weight(rng, 16, 4096, False)
    x = torch.zeros((2049, 4096), dtype=torch.float32, device="cuda")  # 8 MiB + 4 KiB of codes
    status, _ = _static_call(x, w)
    assert status == _lib.LEAFQ_ERR_INVALID
    assert b"code bytes" in _lib.load().leafq_last_error()


def test_static_scratch_rejects_too_many_tokens(cuda_device):
    rng = np.random.default_rng(8)
    w = _weight(rng, 16, 128, False)
    x = torch.zeros((16385, 128), dtype=torch.float32, device="cuda")  # 2 MiB of codes, one token too many
    status, _ = _static_call(x, w)
    assert status == _lib.LEAFQ_ERR_INVALID
    assert b"token scales" in _lib.load().leafq_last_error()
