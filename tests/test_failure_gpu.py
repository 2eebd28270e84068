"""Failure detection without a GPU fault: the bounded wait of the tensor-core
kernels gives up, reports through the device status word, and the context stays
usable (``dsalt_selftest_wait_timeout``: a barrier that nothing ever arrives on)."""

from __future__ import annotations

import ctypes
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_the_context_survives():
    from dsalt.kernels import _ext
    from dsalt.kernels.dsalt_cuda import check_device_status, device_status
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    check_device_status(dev)  # start from a clear status word
    st = device_status(dev)
    lib = _ext.load()
    stream = torch.cuda.current_stream(dev)
    t0 = time.perf_counter()
    rc = lib.dsalt_selftest_wait_timeout(ctypes.c_void_p(st.data_ptr()), ctypes.c_void_p(stream.cuda_stream))
    assert rc == _ext.OK
    torch.cuda.synchronize(dev)
    elapsed = time.perf_counter() - t0
    assert 0.5 < elapsed < 30.0  # the wait ran to its limit (about 2 s) and returned
    with pytest.raises(RuntimeError, match="timed out"):
        check_device_status(dev)
    # the status word was cleared and the context still runs work
    assert check_device_status(dev) == 0
    x = torch.arange(8, device=dev, dtype=torch.float32)
    assert torch.equal((x * 2).cpu(), torch.arange(8, dtype=torch.float32) * 2)
