"""CPU: the GGUF reader behind acb_qw3lm_load (the gf_load / gf_get_* replacement) reads
gguf-py-written files, fuses nothing itself, and rejects truncated / missing files with status
codes (the reference exits or returns false, src/gguf-weights.h:74-155)."""
import ctypes as C
import os

import numpy as np
import pytest

import acb
import oracle as O
from lm_fixtures import TINY, make_tensors, policy_all, policy_q4_k_m, write_gguf


def _open(path):
    h = C.c_void_p()
    st = acb.lib().acb_gguf_open(path.encode(), C.byref(h))
    return st, h


@pytest.mark.parametrize("policy", [policy_all(O.Q8_0), policy_q4_k_m])
def test_reader_matches_written_tensors(tmp_path, policy):
    p = str(tmp_path / "m.gguf")
    t = make_tensors(TINY, policy, seed=3)
    write_gguf(p, TINY, t)
    st, h = _open(p)
    assert st == 0
    L = acb.lib()
    try:
        assert L.acb_gguf_n_tensors(h) == len(t)
        info = L.acb_gguf_tensor_info
        info.restype = C.c_int
        info.argtypes = [C.c_void_p, C.c_int64, C.POINTER(C.c_char_p), C.POINTER(C.c_int), C.POINTER(C.c_int),
                         C.POINTER(C.c_int64), C.POINTER(C.c_void_p), C.POINTER(C.c_size_t)]
        for name, (qt, raw, K, N) in t.items():
            idx = L.acb_gguf_find_tensor(h, name.encode())
            assert idx >= 0, name
            nm, ty, nd, ne, data, nb = C.c_char_p(), C.c_int(), C.c_int(), (C.c_int64 * 4)(), C.c_void_p(), C.c_size_t()
            assert info(h, idx, C.byref(nm), C.byref(ty), C.byref(nd), ne, C.byref(data), C.byref(nb)) == 0
            assert nm.value.decode() == name and ty.value == qt and ne[0] == K
            got = np.ctypeslib.as_array((C.c_uint8 * nb.value).from_address(data.value))
            assert np.array_equal(got, raw.view(np.uint8).reshape(-1)), name
        cfg = L.acb_gguf_get_str(h, b"acestep.config_json").decode()
        assert '"hidden_size": 256' in cfg
        assert L.acb_gguf_find_tensor(h, b"nope") == -1
    finally:
        L.acb_gguf_close(h)


def test_truncated_and_missing_files(tmp_path):
    p = str(tmp_path / "m.gguf")
    write_gguf(p, TINY, make_tensors(TINY, policy_all(O.Q8_0), seed=1))
    data = open(p, "rb").read()
    q = str(tmp_path / "cut.gguf")
    open(q, "wb").write(data[: len(data) - 1000])
    st, _ = _open(q)
    assert st == 7  # ACB_ERR_FORMAT
    assert b"truncated" in acb.lib().acb_last_error()
    st, _ = _open(str(tmp_path / "absent.gguf"))
    assert st == 6  # ACB_ERR_IO
    r = str(tmp_path / "junk.gguf")
    open(r, "wb").write(b"NOPE" + bytes(100))
    st, _ = _open(r)
    assert st == 7
