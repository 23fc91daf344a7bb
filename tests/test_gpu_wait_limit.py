"""A bounded device wait that runs out, on one GPU, without hanging or
faulting anything.

Every spin in the library (pipeline barriers, tagged hand-off words, the
peer all-gather's collect) gives up after the device's wait limit, records
the site in the device error word and lets its kernel return; the reference
bounds its worker spin the same way
(engine/include/leaf/runtime/host_support.h:185-197).  Here the limit is cut
to 1 ms and the peer all-gather of a one-rank group is asked to collect rows
that no rank ever stores (row_begin + local_rows < rows): the collect kernel
must return on its own, write NaN for the missing words, and
leafq_device_status() must report LEAFQ_ERR_TIMEOUT once; the next gather
then succeeds with the default limit restored.
"""
import ctypes
import time

import numpy as np
import pytest
import torch

from leaf_b200 import _lib

pytestmark = pytest.mark.gpu


def _gather(lib, ag, local, row_begin, rows, out):
    stream = torch.cuda.current_stream().cuda_stream
    return lib.leafq_allgather_run(stream, ag, local.data_ptr(), local.shape[0], local.shape[1], row_begin, rows,
                                   out.data_ptr())


def test_wait_limit_rejects_out_of_range_values(cuda_device):
    lib = _lib.load()
    assert lib.leafq_set_wait_limit_ns(10) == _lib.LEAFQ_ERR_INVALID
    assert lib.leafq_set_wait_limit_ns(61 * 10**9) == _lib.LEAFQ_ERR_INVALID
    assert lib.leafq_set_wait_limit_ns(0) == _lib.LEAFQ_OK


def test_collect_wait_runs_out_and_the_next_call_succeeds(cuda_device):
    lib = _lib.load()
    assert lib.leafq_device_status() == _lib.LEAFQ_OK
    tokens, rows, mine = 4, 256, 160
    handle = (ctypes.c_uint8 * _lib.LEAFQ_IPC_HANDLE_BYTES)()
    ag = ctypes.c_void_p()
    assert lib.leafq_allgather_init(0, 1, tokens * rows, ctypes.byref(ag), handle) == _lib.LEAFQ_OK
    try:
        assert lib.leafq_allgather_connect(ag, handle) == _lib.LEAFQ_OK
        rng = np.random.default_rng(3)
        values = torch.from_numpy(rng.standard_normal((tokens, rows)).astype(np.float32)).cuda()
        out = torch.zeros((tokens, rows), dtype=torch.float32, device="cuda")

        # 1. Rows [mine, rows) are never stored: their words wait 1 ms, give up.
        assert lib.leafq_set_wait_limit_ns(1_000_000) == _lib.LEAFQ_OK
        t0 = time.perf_counter()
        assert _gather(lib, ag, values[:, :mine].contiguous(), 0, rows, out) == _lib.LEAFQ_OK
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
        assert lib.leafq_device_status() == _lib.LEAFQ_ERR_TIMEOUT
        text = lib.leafq_last_error()
        assert b"timed out" in text and b"site 13" in text, text
        assert lib.leafq_device_status() == _lib.LEAFQ_OK  # read and cleared
        assert elapsed < 1.0, f"the collect took {elapsed:.3f} s to give up"
        got = out.cpu().numpy()
        want = values.cpu().numpy()
        assert np.array_equal(got[:, :mine].view(np.uint32), want[:, :mine].view(np.uint32))
        assert np.all(got[:, mine:].view(np.uint32) == 0x7FC00000), "missing words must read as NaN"

        # 2. Default limit again; a complete gather on the same buffers
        # (the other half of the receive buffer, then the first one again).
        assert lib.leafq_set_wait_limit_ns(0) == _lib.LEAFQ_OK
        for rep in range(2):
            out.zero_()
            scaled = values * float(rep + 2)
            assert _gather(lib, ag, scaled, 0, rows, out) == _lib.LEAFQ_OK
            torch.cuda.synchronize()
            assert lib.leafq_device_status() == _lib.LEAFQ_OK
            assert np.array_equal(out.cpu().numpy().view(np.uint32), scaled.cpu().numpy().view(np.uint32))
    finally:
        lib.leafq_set_wait_limit_ns(0)
        lib.leafq_allgather_destroy(ag)
