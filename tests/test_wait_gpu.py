"""GPU: failure detection of device-side waits, made to run out without faulting anything.

acb_stream_wait_flag is the library's bounded device wait (the same poll as the persistent decode
step's grid barrier). A flag that nothing raises must end the wait after its limit with
ACB_DEVERR_TIMEOUT in the error word, leave the context usable and let the stream go on; a flag
raised by the host while the GPU waits (mapped pinned memory) must release it without an error;
arguments outside the contract are refused before anything is launched."""
import ctypes as C
import time

import numpy as np
import pytest

import acb

pytestmark = pytest.mark.gpu

ACB_DEVERR_TIMEOUT = 4


def _wait(flag_ptr, value, limit_ns, err_ptr, stream=None):
    return acb.lib().acb_stream_wait_flag(flag_ptr, value, limit_ns, err_ptr, acb._stream(stream))


def test_wait_runs_out_and_context_stays_usable(cuda):
    import torch
    flag = torch.zeros(1, dtype=torch.int32, device=cuda)  # nothing ever raises it
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    assert _wait(flag.data_ptr(), 1, 50_000_000, err.data_ptr()) == 0
    after = torch.arange(1000, device=cuda, dtype=torch.float32).sum()  # queued behind the wait
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    assert int(err.item()) == ACB_DEVERR_TIMEOUT
    assert 0.045 <= dt < 5.0, dt
    assert float(after.item()) == 499500.0
    # the same stream and context after the time-out: a raised flag passes at once
    flag.fill_(5)
    err.zero_()
    assert _wait(flag.data_ptr(), 3, 2_000_000_000, err.data_ptr()) == 0
    torch.cuda.synchronize()
    assert int(err.item()) == 0


def test_wait_released_by_the_host(cuda):
    import torch
    try:
        from cuda import cudart
    except ImportError:  # pragma: no cover
        pytest.skip("cuda-python not importable")
    host = torch.zeros(1, dtype=torch.int32).pin_memory()
    e, dptr = cudart.cudaHostGetDevicePointer(host.data_ptr(), 0)
    if int(e) != 0 or not dptr:
        pytest.skip("pinned memory is not mapped for the device")
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    assert _wait(int(dptr), 7, 5_000_000_000, err.data_ptr()) == 0
    done = torch.cuda.Event()
    done.record()
    time.sleep(0.05)
    assert not done.query()  # the GPU is still waiting for the host
    host.numpy()[0] = 7
    done.synchronize()
    dt = time.perf_counter() - t0
    assert int(err.item()) == 0
    assert dt < 4.0, dt


def test_wait_refuses_bad_arguments(cuda):
    import torch
    flag = torch.zeros(2, dtype=torch.int32, device=cuda)
    for args in ((None, 1, 1000), (flag.data_ptr(), 1, 0), (flag.data_ptr(), 1, 10_000_000_001),
                 (flag.data_ptr() + 1, 1, 1000)):
        assert _wait(*args, None) == 1  # ACB_ERR_INVALID_ARG, nothing launched
    torch.cuda.synchronize()
