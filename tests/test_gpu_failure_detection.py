"""Failure detection on the GPU without a GPU fault: a bounded device wait that can never
be satisfied gives up after a short limit, the host reads CAB_ERR_TIMEOUT from the device
status word, and the context keeps working (a real op runs and matches the oracle)."""

import ctypes

import numpy as np
import pytest
import torch

from oracle import cab_oracle as orc

pytestmark = pytest.mark.gpu

cab = pytest.importorskip("cab_attention")
from cab_attention import _lib  # noqa: E402
from cab_attention.kernels import coarsen_qk_max_l2  # noqa: E402


def test_bounded_wait_times_out_and_context_survives():
    assert _lib.device_status() == 0
    flag = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    rc = _lib.lib().cab_selftest_wait_timeout(50_000, flag.data_ptr(), stream)  # 50 ms
    _lib.check(rc, "cab_selftest_wait_timeout")
    status = ctypes.c_int(-1)
    _lib.check(_lib.lib().cab_device_status(stream, ctypes.byref(status)), "cab_device_status")
    assert status.value == _lib.CAB_ERR_TIMEOUT
    assert int(flag.item()) == 1
    # the status word was cleared by the read, and the context still runs real work
    assert _lib.device_status() == 0
    g = torch.Generator().manual_seed(5)
    q = torch.randn(1, 2, 256, 64, generator=g).to(torch.bfloat16)
    qc, kc = coarsen_qk_max_l2(q.cuda(), q.cuda(), 64)
    want, _ = orc.coarsen_maxl2(q.float().numpy(), 64)
    assert np.array_equal(qc.float().cpu().numpy(), want)
    assert _lib.device_status() == 0


def test_selftest_rejects_bad_limits():
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert _lib.lib().cab_selftest_wait_timeout(0, flag.data_ptr(), None) == 1
    assert _lib.lib().cab_selftest_wait_timeout(20_000_000, flag.data_ptr(), None) == 1
