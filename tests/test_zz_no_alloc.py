"""GPU: acb_argmax_noalloc, the sampling entry point that needs no device allocation.

Some hosts cannot let a library allocate when it samples: their own pool owns the whole device,
or the decode thread must never call cudaMalloc because it can synchronise the device. For
them acb_argmax_noalloc keeps its scratch in a fixed array inside the library's device memory.
These tests call it through the C ABI and check it against acb_argmax (caller-provided
scratch): the token ids and the top1 - top2 margins must be identical, on two calls in a row
(the second call reuses the array the first one left behind), over a sequence of shapes whose
partials would overlap a moving counter, and on a first call issued from a non-blocking stream.
The file sorts last so that a run stopping at its first failure has already run every other test.
"""
import ctypes as C

import numpy as np
import pytest

import acb

pytestmark = pytest.mark.gpu


def _entry():
    fn = acb.lib().acb_argmax_noalloc
    fn.restype = C.c_int
    fn.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                   C.c_void_p, C.c_int64, C.c_void_p, C.c_int, C.c_void_p]
    return fn


def test_noalloc_argmax_matches_argmax_on_two_calls(cuda):
    import torch
    fn = _entry()
    rng = np.random.default_rng(2026)
    for rows, V in ((3, 217472), (5, 151936)):  # two calls in a row, different shapes and data
        lg = torch.from_numpy(rng.standard_normal((rows, V)).astype(np.float32)).to(cuda)
        lg[1, 777] = 1e3
        lg[1, 5] = 1e3  # a tie: the lower index must win
        ids_ref = torch.empty(rows, dtype=torch.int32, device=cuda)
        mar_ref = torch.empty(rows, dtype=torch.float32, device=cuda)
        acb.argmax(lg, ids_ref, margin=mar_ref)
        ids = torch.full((rows,), -1, dtype=torch.int32, device=cuda)
        mar = torch.full((rows,), -1.0, dtype=torch.float32, device=cuda)
        st = fn(lg.data_ptr(), V, V, rows, ids.data_ptr(), mar.data_ptr(), None, None, None, 0, None, 0,
                acb._stream(None))
        assert st == 0, acb.lib().acb_last_error()
        torch.cuda.synchronize()
        assert torch.equal(ids, ids_ref)
        assert torch.equal(mar, mar_ref)
        assert int(ids[1].item()) == 5
        assert ids.cpu().numpy().tolist()[0] == int(np.argmax(lg[0].cpu().numpy()))


def test_noalloc_argmax_rejects_rows_beyond_its_array(cuda):
    import torch
    fn = _entry()
    rows, V = 33, 1024
    lg = torch.zeros((rows, V), dtype=torch.float32, device=cuda)
    ids = torch.empty(rows, dtype=torch.int32, device=cuda)
    st = fn(lg.data_ptr(), V, V, rows, ids.data_ptr(), None, None, None, None, 0, None, 0, acb._stream(None))
    assert st == 2  # ACB_ERR_UNSUPPORTED, nothing launched
    assert b"ACB_ARGMAX_NOALLOC_MAX_ROWS" in acb.lib().acb_last_error()


def test_noalloc_argmax_shape_sequence(cuda):
    """Calls of different shapes in a row share the array: the row counters live at a fixed
    offset, so a smaller call never lands its counters on a larger call's leftover partials."""
    import torch
    fn = _entry()
    rng = np.random.default_rng(77)
    for rows, V in ((3, 217472), (1, 151936), (32, 217472), (1, 8192), (5, 1001), (2, 217472)):
        lg = torch.from_numpy(rng.standard_normal((rows, V)).astype(np.float32)).to(cuda)
        ids = torch.full((rows,), -1, dtype=torch.int32, device=cuda)
        mar = torch.full((rows,), -1.0, dtype=torch.float32, device=cuda)
        st = fn(lg.data_ptr(), V, V, rows, ids.data_ptr(), mar.data_ptr(), None, None, None, 0, None, 0,
                acb._stream(None))
        assert st == 0, acb.lib().acb_last_error()
        torch.cuda.synchronize()
        host = lg.cpu().numpy()
        assert ids.cpu().numpy().tolist() == [int(np.argmax(r)) for r in host], (rows, V)
        srt = np.sort(host, axis=1)
        assert np.array_equal(mar.cpu().numpy(), srt[:, -1] - srt[:, -2]), (rows, V)


_FRESH = r"""
import sys, numpy as np, torch, ctypes as C
sys.path[:0] = [{pkg!r}]
import acb
fn = acb.lib().acb_argmax_noalloc
fn.restype = C.c_int
fn.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
               C.c_void_p, C.c_int64, C.c_void_p, C.c_int, C.c_void_p]
dev = torch.device("cuda:0")
s = torch.cuda.Stream(dev)  # created with cudaStreamNonBlocking: no implicit ordering with stream 0
rng = np.random.default_rng(5)
for rows, V in ((4, 217472), (1, 4096)):
    host = rng.standard_normal((rows, V)).astype(np.float32)
    with torch.cuda.stream(s):
        lg = torch.from_numpy(host).to(dev, non_blocking=False)
        ids = torch.full((rows,), -1, dtype=torch.int32, device=dev)
        st = fn(lg.data_ptr(), V, V, rows, ids.data_ptr(), None, None, None, None, 0, None, 0, s.cuda_stream)
        assert st == 0, acb.lib().acb_last_error()
    s.synchronize()
    assert ids.cpu().numpy().tolist() == [int(np.argmax(r)) for r in host], (rows, V)
print("ok")
"""


def test_noalloc_argmax_first_call_on_nonblocking_stream(cuda):
    """The first call on a device (which looks up the array and clears its counters) made from
    a non-blocking stream in a fresh process: the clear is ordered before the kernel."""
    import os
    import subprocess
    import sys
    pkg = os.path.dirname(acb.__file__)
    r = subprocess.run([sys.executable, "-c", _FRESH.format(pkg=pkg)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout + r.stderr
