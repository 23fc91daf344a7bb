"""Grouped INT8 prefill on the tensor cores (gemm_w8a8_grouped_tc_kernel:
tcgen05.mma kind::i8 per weight group into a ring of TMEM slots, the
groups' scaled sums accumulated in order by the epilogue) against the CPU
restatement of Decoder::Impl::linear's integer branch (quant_tile_avx /
quant_vnni_tile, decoder.cpp:571-617, 661-702; bias :1229), bit for bit, in
both of the reference's group-accumulation forms: one FMA per group (AVX2 +
FMA builds) and two roundings (the AVX-VNNI tile, LEAFQ_FLAG_VNNI_ROUNDING).
Group sizes 32 .. 512, ragged M / N / K (K a multiple of 32 but not of 128),
with and without bias; a seeded sample of rows plus the last tile's rows is
checked for every token."""
import numpy as np
import pytest
import torch

import leaf_b200 as lq
import oracle
from conftest import bits_equal

pytestmark = pytest.mark.gpu


def _case(rng, m, k, n, group, with_bias):
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    w[:, rng.random(k) < 0.02] *= 8.0  # columns that dominate their group's scale
    payload, scales = oracle.quantize_weight(w, 8, group)
    x = rng.standard_normal((m, k)).astype(np.float32)
    x[rng.random((m, k)) < 0.01] *= 20.0
    bias = (rng.standard_normal(n) * 0.01).astype(np.float32) if with_bias else None
    return payload, scales, x, bias


@pytest.mark.parametrize("m,k,n,group", [(512, 2048, 5632, 128), (300, 2048, 1000, 64), (9, 1024, 258, 32),
                                         (1100, 2080, 520, 160), (64, 5632, 2048, 128), (200, 4096, 384, 512),
                                         (130, 256, 4100, 32)])
@pytest.mark.parametrize("fused", [True, False])
def test_grouped_tc_matches_oracle(cuda_device, m, k, n, group, fused):
    rng = np.random.default_rng(m * 7 + k + n + group + int(fused))
    payload, scales, x, bias = _case(rng, m, k, n, group, with_bias=(m % 2 == 0))
    w = lq.QuantWeight.from_host(payload, scales, n, k, 8, group, bias)
    flags = 0 if fused else lq.LEAFQ_FLAG_VNNI_ROUNDING
    y = lq.linear(torch.from_numpy(x).cuda(), w, flags=flags).cpu().numpy()
    rows = np.unique(np.concatenate([rng.choice(n, min(n, 64), replace=False), np.arange(max(0, n - 70), n),
                                     np.arange(0, min(n, 4))]))
    expect = oracle.linear_int(x, payload[rows], scales[rows], 8, group,
                               None if bias is None else bias[rows], fused=fused)
    assert bits_equal(y[:, rows], expect)
    assert lq.load().leafq_device_status() == 0


def test_grouped_tc_from_codes_every_row(cuda_device):
    # leafq_linear_int_q from given codes, all rows and tokens compared.
    rng = np.random.default_rng(21)
    m, k, n, group = 257, 1024, 640, 64
    payload, scales, x, bias = _case(rng, m, k, n, group, with_bias=True)
    q, sx = oracle.quantize_act(x)
    w = lq.QuantWeight.from_host(payload, scales, n, k, 8, group, bias)
    y = lq.linear_int_q(torch.from_numpy(q).cuda(), torch.from_numpy(sx).cuda(), w).cpu().numpy()
    assert bits_equal(y, oracle.linear_int_q(q, sx, payload, scales, 8, group, bias))


def test_grouped_tc_agrees_with_cuda_core_path(cuda_device):
    # The int32 group sums are only written by the CUDA-core kernel; asking
    # for them routes there.  Both paths give the same outputs.
    rng = np.random.default_rng(5)
    m, k, n, group = 96, 2048, 512, 128
    payload, scales, x, _ = _case(rng, m, k, n, group, with_bias=False)
    q, sx = oracle.quantize_act(x)
    w = lq.QuantWeight.from_host(payload, scales, n, k, 8, group)
    qd, sxd = torch.from_numpy(q).cuda(), torch.from_numpy(sx).cuda()
    y_tc = lq.linear_int_q(qd, sxd, w).cpu().numpy()
    y_cc, acc = lq.linear_int_q(qd, sxd, w, want_acc=True)
    assert bits_equal(y_tc, y_cc.cpu().numpy())
    expect_acc = np.einsum("mgk,ngk->mng", q.reshape(m, k // group, group).astype(np.int64),
                           payload.reshape(n, k // group, group).astype(np.int64))
    assert np.array_equal(acc.cpu().numpy().astype(np.int64), expect_acc)
