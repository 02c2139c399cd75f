"""ctypes binding of libacb (the C ABI in include/acb.h) for Python callers.

Device tensors are passed as torch CUDA tensors (only their data pointers cross the ABI) and
kernels are enqueued on torch's current stream. The library is loaded from lib/libacb.so next
to this file; there is no fallback of any kind: a missing or unloadable library raises.
"""
from __future__ import annotations

import ctypes as C
import os
import re
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB_PATH = os.path.join(HERE, "lib", "libacb.so")
HEADER_DIR = os.path.join(ROOT, "include")

F32, F16, Q8_0, Q4_K, Q6_K, Q8_K, I32, BF16 = 0, 1, 8, 12, 14, 15, 26, 30

STATUS = {0: "ok", 1: "invalid argument", 2: "unsupported", 3: "cuda error", 4: "out of range", 5: "oom",
          6: "io", 7: "format", 8: "device error flag"}


class AcbError(RuntimeError):
    def __init__(self, fn: str, status: int):
        super().__init__(f"{fn} failed: {status} ({STATUS.get(status, '?')})")
        self.status = status


_lib = None


def build() -> str:
    subprocess.run(["make", "-s", "-j8", "-C", HERE], check=True)
    return LIB_PATH


def header_functions() -> list[str]:
    """Names of every ACB_API function declared in include/*.h."""
    names = []
    for f in sorted(os.listdir(HEADER_DIR)):
        if f.endswith(".h"):
            txt = open(os.path.join(HEADER_DIR, f)).read()
            names += re.findall(r"^ACB_API\s+[\w\s\*]+?\b(acb_\w+|qwen3_\w+|qw3lm_\w+|dit_\w+)\s*\(", txt, re.M)
    return names


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"libacb not built: {LIB_PATH} missing (run `make -C {HERE}`)")
        L = C.CDLL(LIB_PATH)
        P, I64, I, F = C.c_void_p, C.c_int64, C.c_int, C.c_float
        sig = {
            "acb_version": (I, []),
            "acb_status_string": (C.c_char_p, [I]),
            "acb_last_cuda_error": (I, []),
            "acb_row_bytes": (I64, [I, I64]),
            "acb_rope_table_host": (I, [P, I, I, F]),
            "acb_rms_norm": (I, [P, I, I64, P, P, I, I64, I64, I, F, P]),
            "acb_qk_norm_rope": (I, [P, I, I64, P, I, I64, I64, I64, I64, I, I, P, F, P, P, I, P, P]),
            "acb_swiglu": (I, [P, I, I64, I64, P, I, I64, I64, I64, P]),
            "acb_adaln_modulate": (I, [P, I, P, F, P, P, I64, P, I, I64, I64, I, P]),
            "acb_gated_residual": (I, [P, P, I, P, I64, P, I64, I64, I, P]),
            "acb_get_rows": (I, [P, I, I64, I64, P, I64, P, I, I64, P, P]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


# ---- helpers ---------------------------------------------------------------------------------

def _ptr(t):
    if t is None:
        return None
    if isinstance(t, int):
        return t
    return t.data_ptr()


def _stream(stream=None):
    if stream is not None:
        return stream if isinstance(stream, int) else stream.cuda_stream
    import torch
    return torch.cuda.current_stream().cuda_stream


def _check(fn: str, st: int):
    if st != 0:
        raise AcbError(fn, st)


def dtype_id(t) -> int:
    import torch
    return {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16, torch.int32: I32}[t.dtype]


def rope_table(max_pos: int, head_dim: int, base: float):
    """Host RoPE table [max_pos, head_dim] (cos/sin interleaved) as a torch CPU tensor."""
    import torch
    t = torch.empty((max_pos, head_dim), dtype=torch.float32)
    _check("acb_rope_table_host", lib().acb_rope_table_host(t.data_ptr(), max_pos, head_dim, base))
    return t


# ---- ops -------------------------------------------------------------------------------------

def rms_norm(x, w, eps, out=None, out_dtype=None, stream=None):
    import torch
    rows = x.numel() // x.shape[-1]
    cols = x.shape[-1]
    if out is None:
        out = torch.empty(x.shape, dtype=out_dtype or x.dtype, device=x.device)
    _check("acb_rms_norm", lib().acb_rms_norm(_ptr(x), dtype_id(x), cols, _ptr(w), _ptr(out), dtype_id(out), cols,
                                               rows, cols, eps, _stream(stream)))
    return out


def qk_norm_rope(src, n_heads, head_dim, w, eps, pos, rope, out=None, out_dtype=None, src_tok_stride=None,
                 dst_tok_stride=None, dst_head_stride=None, dst_pos_stride=0, n_tok=None, err=None, stream=None):
    """src rows [T, >= n_heads*head_dim] (token stride src_tok_stride). Default destination is a
    dense [T, n_heads, head_dim] tensor."""
    import torch
    T = n_tok if n_tok is not None else src.shape[0]
    sts = src_tok_stride if src_tok_stride is not None else src.stride(0)
    if out is None:
        out = torch.empty((T, n_heads, head_dim), dtype=out_dtype or src.dtype, device=src.device)
        dst_tok_stride, dst_head_stride = n_heads * head_dim, head_dim
    max_pos = rope.shape[0] if rope is not None else (2 ** 31 - 1)
    _check("acb_qk_norm_rope", lib().acb_qk_norm_rope(
        _ptr(src), dtype_id(src), sts, _ptr(out), dtype_id(out), dst_tok_stride, dst_head_stride, dst_pos_stride,
        T, n_heads, head_dim, _ptr(w), eps, _ptr(pos), _ptr(rope), max_pos, _ptr(err), _stream(stream)))
    return out


def swiglu(gu, F, out=None, out_dtype=None, up_offset=None, stream=None):
    """gu rows [R, 2F] fused (gate | up)."""
    import torch
    rows = gu.numel() // gu.shape[-1]
    if out is None:
        out = torch.empty((*gu.shape[:-1], F), dtype=out_dtype or gu.dtype, device=gu.device)
    _check("acb_swiglu", lib().acb_swiglu(_ptr(gu), dtype_id(gu), gu.shape[-1], F if up_offset is None else up_offset,
                                           _ptr(out), dtype_id(out), F, rows, F, _stream(stream)))
    return out


def adaln_modulate(x, norm_w, eps, scale, shift, out=None, out_dtype=None, stream=None):
    """x [S, T, H]; scale/shift [H] or [S, H] float32."""
    import torch
    S, T, H = x.shape
    vs = 0 if scale.dim() == 1 else H
    if out is None:
        out = torch.empty(x.shape, dtype=out_dtype or x.dtype, device=x.device)
    _check("acb_adaln_modulate", lib().acb_adaln_modulate(_ptr(x), dtype_id(x), _ptr(norm_w), eps, _ptr(scale),
                                                           _ptr(shift), vs, _ptr(out), dtype_id(out), S, T, H,
                                                           _stream(stream)))
    return out


def gated_residual(r, o, gate, out=None, stream=None):
    import torch
    S, T, H = r.shape
    vs = 0 if gate.dim() == 1 else H
    if out is None:
        out = torch.empty_like(r)
    _check("acb_gated_residual", lib().acb_gated_residual(_ptr(r), _ptr(o), dtype_id(r), _ptr(gate), vs, _ptr(out),
                                                           S, T, H, _stream(stream)))
    return out


def get_rows(table, table_type, n_rows, cols, ids, out=None, out_dtype=None, err=None, stream=None):
    """table: uint8 device tensor of raw GGUF rows; ids int32 device tensor."""
    import torch
    n = ids.numel()
    if out is None:
        out = torch.empty((n, cols), dtype=out_dtype or torch.float32, device=ids.device)
    _check("acb_get_rows", lib().acb_get_rows(_ptr(table), table_type, n_rows, cols, _ptr(ids), n, _ptr(out),
                                               dtype_id(out), out.stride(0), _ptr(err), _stream(stream)))
    return out
