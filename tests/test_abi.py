"""CPU: the C-ABI library loads, exports every function include/*.h declares, and rejects bad
arguments with a status code before touching a device (no compute calls here)."""
import ctypes as C

import numpy as np
import pytest

import acb
import oracle as O


def test_library_exports_every_header_symbol():
    L = acb.lib()
    names = acb.header_functions()
    assert len(names) >= 11
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing


def test_version_and_status_strings():
    L = acb.lib()
    assert L.acb_version() >= (0 << 16) | (1 << 8)
    for s in range(0, 9):
        assert L.acb_status_string(s)
    assert L.acb_status_string(0) == b"ok"


@pytest.mark.parametrize("t,n,rb", [(acb.Q8_0, 2048, 2176), (acb.Q4_K, 2560, 1440), (acb.Q6_K, 2048, 1680),
                                    (acb.F32, 7, 28), (acb.BF16, 7, 14), (acb.Q8_0, 33, -1), (99, 32, -1)])
def test_row_bytes(t, n, rb):
    assert acb.lib().acb_row_bytes(t, n) == rb


def test_invalid_arguments_are_status_codes():
    L = acb.lib()
    # null pointers: rejected before any CUDA call
    assert L.acb_rms_norm(None, acb.F32, 8, None, None, acb.F32, 8, 4, 8, 1e-6, None) == 1
    assert L.acb_swiglu(None, acb.F32, 16, 8, None, acb.F32, 8, 4, 8, None) == 1
    assert L.acb_get_rows(None, acb.Q8_0, 10, 32, None, 4, None, acb.F32, 32, None, None) == 1
    assert L.acb_gated_residual(None, None, acb.F32, None, 0, None, 1, 1, 8, None) == 1
    assert L.acb_adaln_modulate(None, acb.F32, None, 1e-6, None, None, 0, None, acb.F32, 1, 1, 8, None) == 1
    # unsupported head_dim (checked before launch)
    buf = (C.c_float * 64)()
    assert L.acb_qk_norm_rope(C.addressof(buf), acb.F32, 96, C.addressof(buf), acb.F32, 96, 96, 0, 1, 1, 96, None,
                              1e-6, None, None, 0, None, None) == 2
    # get_rows: cols not a block multiple
    assert L.acb_get_rows(C.addressof(buf), acb.Q8_0, 1, 33, C.addressof(buf), 1, C.addressof(buf), acb.F32, 33,
                          None, None) == 1


def test_rope_table_matches_oracle_bitexact():
    """The library's host RoPE table (shared by every rotation kernel) equals the oracle's."""
    for D, base, n in ((128, 1e6, 8192), (64, 1e4, 300)):
        t = acb.rope_table(n, D, base).numpy()
        ref = O.rope_cache(np.arange(n, dtype=np.int32), D, base)
        assert np.array_equal(t.view(np.uint32), ref.view(np.uint32))


class _DecodeStep(C.Structure):
    """acb_decode_step (acb.h), for argument checks only."""
    _fields_ = [("layers", C.c_void_p), ("n_layers", C.c_int), ("hidden", C.c_int), ("ffn", C.c_int),
                ("n_heads", C.c_int), ("n_kv_heads", C.c_int), ("head_dim", C.c_int), ("eps", C.c_float),
                ("attn_scale", C.c_float), ("max_seq", C.c_int), ("max_pos", C.c_int), ("kv_set", C.c_int),
                ("embed", C.c_void_p), ("embed_rows", C.c_int64), ("head", C.c_void_p), ("vocab", C.c_int64),
                ("final_norm", C.c_void_p), ("rope", C.c_void_p), ("ids", C.c_void_p), ("pos", C.c_void_p),
                ("logits", C.c_void_p), ("greedy", C.c_int), ("n_steps", C.c_int), ("margin", C.c_void_p), ("hist", C.c_void_p),
                ("mhist", C.c_void_p), ("hist_base", C.c_void_p), ("scratch", C.c_void_p), ("err", C.c_void_p)]


def test_persistent_decode_shape_checks():
    L = acb.lib()
    L.acb_lm_decode_scratch_bytes.restype = C.c_size_t
    assert L.acb_lm_decode_step(None, None) == 1
    assert L.acb_lm_decode_scratch_bytes(None) == 0
    s = _DecodeStep(n_layers=28, hidden=2048, ffn=6144, n_heads=16, n_kv_heads=8, head_dim=128, eps=1e-6,
                    attn_scale=0.088, max_seq=8192, max_pos=8192, vocab=217472, embed_rows=217472)
    n = L.acb_lm_decode_scratch_bytes(C.byref(s))
    # scores [16][8192] f32 dominate; every region is present
    assert 16 * 8192 * 4 < n < 16 * 8192 * 4 + 4 * 1024 * 1024
    for field, bad in [("head_dim", 64), ("n_kv_heads", 2), ("ffn", 6000), ("vocab", 217473), ("hidden", 16384)]:
        t = _DecodeStep.from_buffer_copy(s)
        setattr(t, field, bad)
        assert L.acb_lm_decode_scratch_bytes(C.byref(t)) == 0, field
        assert "acb_lm_decode" in L.acb_last_error().decode()
    # every pointer null: invalid before any shape or device check
    assert L.acb_lm_decode_step(C.byref(s), None) == 1
