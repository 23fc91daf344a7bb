"""The many-token prefill GEMM on CTA pairs (gemm_w8a8_tc2_kernel:
tcgen05.mma.cta_group::2 over 256 x 256 tiles, each CTA of a cluster of two
loading half of the codes and half of the weight rows) against the CPU
restatement of Decoder::Impl::linear (quant_vnni_tile / quant_tile_avx,
decoder.cpp:571-702, epilogue :1229), bit for bit.  The shapes reach the pair
path (at least 1024 tokens and a full round of 256 x 256 tiles); the oracle
checks a seeded sample of weight rows for every token, including the rows of
the last, partial tile, and ragged M, N and K tails."""
import numpy as np
import pytest
import torch

import leaf_b200 as lq
import oracle
from conftest import bits_equal

pytestmark = pytest.mark.gpu


def _weight(rng, n, k, bias=True):
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    payload, scales = oracle.quantize_weight(w, 8, k)
    b = (rng.standard_normal(n) * 0.01).astype(np.float32) if bias else None
    return payload, scales, b


def _x(rng, m, k):
    x = rng.standard_normal((m, k)).astype(np.float32)
    x[rng.random((m, k)) < 0.01] *= 20.0
    return x


@pytest.mark.parametrize("m,k,n", [(1024, 2048, 5632), (1300, 2000, 5000), (4096, 2048, 5632),
                                   (2048, 5632, 2560)])
def test_pair_gemm_matches_oracle(cuda_device, m, k, n):
    rng = np.random.default_rng(m + 3 * k + 7 * n)
    payload, scales, bias = _weight(rng, n, k)
    x = _x(rng, m, k)
    w = lq.QuantWeight.from_host(payload, scales, n, k, 8, k, bias)
    y = lq.linear(torch.from_numpy(x).cuda(), w).cpu().numpy()
    rows = np.unique(np.concatenate([rng.choice(n, 48, replace=False), np.arange(n - 8, n), np.arange(0, 4),
                                     np.arange(128, 132), np.arange(252, 260)]))
    expect = oracle.linear_int(x, payload[rows], scales[rows], 8, k, bias[rows])
    assert bits_equal(y[:, rows], expect)
    assert lq.load().leafq_device_status() == 0


def test_pair_gemm_accumulators_exact(cuda_device):
    # Unit scales and codes at +-127: y equals the int32 dot product itself
    # (exact in float below 2^24), so every (token, row) sum is checked.
    m, k, n = 1024, 1024, 5120
    rng = np.random.default_rng(77)
    q = rng.integers(-127, 128, (m, k)).astype(np.int8)
    wq = rng.integers(-127, 128, (n, k)).astype(np.int8)
    w = lq.QuantWeight.from_host(wq, np.ones((n, 1), dtype=np.float32), n, k, 8, k)
    y = lq.linear_int_q(torch.from_numpy(q).cuda(), torch.ones(m, device="cuda"), w).cpu().numpy()
    expect = q.astype(np.int64) @ wq.astype(np.int64).T
    assert np.array_equal(y.astype(np.int64), expect)
