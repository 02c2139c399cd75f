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
          6: "io", 7: "format", 8: "device error flag", 9: "cancelled", 10: "timeout"}


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
            "acb_quantize": (I, [P, I64, I64, I, P, P]),
            "acb_gemm_bf16": (I, [P, I64, P, I64, I64, I64, I64, P, I, I64, P, P, I64, P, I64, I64, I, P, P]),
            "acb_attn_prefill": (I, [P, I64, I64, P, I64, I64, P, I64, I64, P, I, I64, I64, I, I, I, I, I, I, I, I,
                                     I, F, I, P]),
            "acb_gemv": (I, [P, I, I64, I64, I, I, P, I64, P, F, I, P, I64, I, P, I64, I, P, P]),
            "acb_q8_0_to_tiles": (I, [P, P, I64, I64, P]),
            "acb_qkv_post": (I, [P, I64, I64, I, I, I, P, P, F, P, P, I, P, I64, P, P, I, I, I, I, P, P]),
            "acb_attn_decode_splits": (I, [I, I]),
            "acb_attn_decode": (I, [P, I64, I, I, I, I, P, P, P, I, I, I, F, I, P, P, P, P, I64, P, I, P]),
            "acb_argmax_scratch_bytes": (C.c_size_t, [I, I64]),
            "acb_argmax": (I, [P, I64, I64, I, P, P, P, P, P, I64, P, P, I, P]),
            # model level (acb_models.h)
            "acb_last_error": (C.c_char_p, []),
            "acb_gguf_open": (I, [C.c_char_p, C.POINTER(C.c_void_p)]),
            "acb_gguf_close": (None, [P]),
            "acb_gguf_n_tensors": (I64, [P]),
            "acb_gguf_find_tensor": (I64, [P, C.c_char_p]),
            "acb_gguf_get_u32": (C.c_uint32, [P, C.c_char_p]),
            "acb_gguf_get_str": (C.c_char_p, [P, C.c_char_p]),
            "acb_qw3lm_load": (I, [C.c_char_p, I, I, I, C.POINTER(C.c_void_p)]),
            "acb_qw3lm_forward": (I, [P, P, I, I, P]),
            "acb_qw3lm_forward_batch": (I, [P, P, P, I, P, I, I]),
            "acb_qw3lm_reset_kv": (None, [P, I]),
            "acb_qw3lm_copy_kv": (I, [P, I, I]),
            "acb_qw3lm_build_partial_head": (I, [P, I]),
            "acb_qw3lm_kv_pos": (I, [P, I]),
            "acb_qw3lm_weight_bytes": (C.c_size_t, [P]),
            "acb_qw3lm_persistent_decode": (I, [P]),
            "acb_qw3lm_generate_greedy": (I, [P, P, I, I, I, P, P, P]),
            "acb_qw3lm_free": (None, [P]),
            "acb_qwen3_load_text_encoder": (I, [C.c_char_p, I, C.POINTER(C.c_void_p)]),
            "acb_qwen3_weight_bytes": (C.c_size_t, [P]),
            "acb_qwen3_forward": (I, [P, P, I, P]),
            "acb_qwen3_forward_device": (I, [P, P, I, P, P]),
            "acb_qwen3_embed_lookup": (I, [P, P, I, P]),
            "acb_qwen3_forward_hidden": (I, [P, P, I, I, I, I, P, P]),
            "acb_qwen3_set_exact": (I, [P, I]),
            "acb_dit_load": (I, [C.c_char_p, I, C.POINTER(C.c_void_p)]),
            "acb_dit_weight_bytes": (C.c_size_t, [P]),
            "acb_dit_set_exact": (I, [P, I]),
            "acb_dit_sinusoid": (I, [P, I, I, P, P]),
            "acb_dit_sde_philox": (I, [P, P, P, P, I, I64, P]),
            "acb_philox_randn": (I, [I64, P, I64, I, P]),
            "acb_philox_bits": (I, [I64, I64, I64, P, P]),
            "acb_dit_forward": (I, [P, P, P, I, I, I, F, F, P, I, P]),
            "acb_dit_generate": (I, [P, P, P, P, I, I, I, I, P, P, F, P]),
            "acb_dit_generate_solver": (I, [P, P, P, P, I, I, I, I, P, P, F, I, P]),
            "acb_dit_generate_ex": (I, [P, P, P, P, I, I, I, I, P, P, F, P, I, P, P, P, P, P, P, P, I, F, F,
                                        C.c_char_p, C.c_char_p, I, P, P, P]),
            "acb_dit_set_lengths": (I, [P, P, P, P]),
            "acb_comm_unique_id": (I, [P]),
            "acb_comm_init": (I, [P, I, I, I, I, C.POINTER(C.c_void_p)]),
            "acb_comm_rank": (I, [P]),
            "acb_comm_world": (I, [P]),
            "acb_comm_free": (None, [P]),
            "acb_dit_shard_plan": (I, [I, I, I, I, C.POINTER(I), C.POINTER(I), C.POINTER(I), C.POINTER(I)]),
            "acb_dit_generate_sharded": (I, [P, P, P, P, P, I, I, I, I, P, P, F, P, I, P, P, P, P, P, P, P,
                                             C.c_char_p, P, P, P]),
            "acb_dit_job_begin": (I, [P, P, P, P, P, I, I, I, F, P, I, P, P, P, P, P, P, P, C.c_char_p, P, P]),
            "acb_dit_job_step": (I, [P, I, F, F, I, P]),
            "acb_dit_job_end": (I, [P, P, P]),
            "acb_dit_stream": (P, [P]),
            "acb_dit_free": (None, [P]),
            "acb_dit_set_condition": (I, [P, P, I, I, I, P]),
            "acb_attn_tc": (I, [P, I64, P, I64, P, I64, P, I, I64, I, I, I, I, I, I, I, I, I, F, I, I64, I64, I64, P,
                                P]),
            "acb_attn_vt": (I, [P, I, I64, I64, I, I, I, I, P, I64, I64, P]),
            "acb_dit_eval_kernels": (I, [P]),
            "acb_dit_step_kernels": (I, [P]),
            "acb_qwen3_forward_kernels": (I, [P]),
            "acb_dit_eval": (I, [P, P, P, P, P]),
            "acb_dit_apg": (I, [P, P, P, I, F, F, F, I, I, I, P, P]),
            "acb_dit_euler": (I, [P, P, P, I, P, I64, P]),
            "acb_dit_dpm3m": (I, [P, P, P, P, I, P, I64, P]),
            "acb_dit_sde": (I, [P, P, P, P, I64, P]),
            "acb_act_quant_ex": (I, [P, I64, I64, I64, I64, I, I, P, I, I64, I64, P]),
            "acb_norm_quant": (I, [P, I64, I64, I64, P, F, P, P, I64, I64, I, I, P, I, I64, I64, P]),
            "acb_qk_norm_rope_planes": (I, [P, I, I64, P, I64, I64, I64, I, P, I, P, I, F, P, P, I, P, P]),
            "acb_attn_prefill_split": (I, [P, I64, I64, P, I64, I64, P, I64, I64, P, I, I64, I64, I, I, I, I, I, I, I,
                                           I, I, F, I, I64, I64, I64, P]),
            "acb_qwen3_free": (None, [P]),
            "acb_act_quant": (I, [P, I64, I64, I64, I, P, I, I64, P]),
            "acb_act_quant_swiglu": (I, [P, I64, I64, I64, I64, I, P, I, I64, P]),
            "acb_vec_dot_type": (I, [I]),
            "acb_gemm_workspace_bytes": (C.c_size_t, [I64, I64, I64]),
            "acb_conv1d_tc": (I, [P, I64, I64, I, P, I64, I, I, I, P, I, I64, P, P, I64, I, P, C.c_size_t, P, P]),
            "acb_vae_snake_f16": (I, [P, I64, I64, I, P, P, P, I64, P]),
            "acb_stream_wait_flag": (I, [P, C.c_uint32, C.c_uint64, P, P]),
            "acb_vae_out_conv": (I, [P, I64, I, P, P, P, P, P]),
            "acb_gemm_swiglu_quant": (I, [P, I64, P, I64, I64, I64, I64, P, I, I, P, I, I64, I, P, P]),
            "acb_gemm_qkv_planes": (I, [P, I64, P, I64, I64, I64, I, I, P, P, F, P, P, I, I64, P, I64, I64, P, I64, I64,
                                        I, P, P]),
            "acb_gemm_pair_clusters": (I, [I]),
            "acb_sample_work_bytes": (C.c_size_t, [I, I]),
            "acb_lora_delta_add": (I, [P, I64, I64, P, P, I, F, P]),
            "acb_requant": (I, [P, I64, I64, I, P, P]),
            "acb_sample_top_k_p": (I, [P, I64, P, I64, F, I, I64, I, I, F, F, I, P, P, P, P]),
            "acb_fsq_project_out": (I, [P, I, P, I, I, P, P, I64, P, P]),
            "acb_fsq_quantize": (I, [P, I64, P, I, P, P]),
            "acb_rows_repeat_add": (I, [P, I64, P, I64, I, I, I, P, I64, P]),
            "acb_rows_prepend": (I, [P, P, I64, I, I, I, P, I64, P]),
            "acb_fsq_decode_index": (None, [I, P]),
            "acb_fsq_encode_index": (I, [P]),
            "acb_cond_load": (I, [C.c_char_p, I, C.POINTER(C.c_void_p)]),
            "acb_cond_set_exact": (I, [P, I]),
            "acb_cond_forward": (I, [P, P, I, P, I, P, I, P, P]),
            "acb_cond_forward_device": (I, [P, P, I, P, I, P, I, P, P, P]),
            "acb_cond_null_embedding": (I, [P, P]),
            "acb_cond_free": (None, [P]),
            "acb_detok_load": (I, [C.c_char_p, I, C.POINTER(C.c_void_p)]),
            "acb_detok_set_exact": (I, [P, I]),
            "acb_detok_decode": (I, [P, P, I, P]),
            "acb_detok_decode_device": (I, [P, P, I, P, P]),
            "acb_detok_free": (None, [P]),
            "acb_tok_load": (I, [C.c_char_p, I, C.POINTER(C.c_void_p)]),
            "acb_tok_set_exact": (I, [P, I]),
            "acb_tok_encode": (I, [P, P, I, P, P, P]),
            "acb_tok_encode_device": (I, [P, P, I, P, P]),
            "acb_tok_free": (None, [P]),
            "acb_gemm_tc": (I, [P, I64, P, I64, I64, I64, I64, P, I, I64, P, P, I64, P, I64, I64, I, P, C.c_size_t, P,
                                P]),
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


# ---- decode path -------------------------------------------------------------------------------

PRO_X, PRO_RMSNORM, PRO_SUM_SPLITS, PRO_SWIGLU = 0, 1, 2, 3
EPI_STORE, EPI_ADD = 0, 1
FLAG_PDL = 1
FLAG_F16 = 2  # tensor-core operands are f16 (acb_gemm_bf16, acb_attn_prefill)
FLAG_GEMM_A = 4  # acb_attn_tc: quantised output in the exact [hi | hi | lo] operand layout


Q8_0_TILES = 1008


def q8_0_to_tiles(W, N, K, stream=None):
    """GGUF Q8_0 rows (uint8 tensor) -> the tensor-core GEMV's tiled copy (w_type Q8_0_TILES)."""
    import torch
    out = torch.empty_like(W)
    _check("acb_q8_0_to_tiles", lib().acb_q8_0_to_tiles(_ptr(W), _ptr(out), N, K, _stream(stream)))
    return out


def gemv(W, w_type, N, K, x, M=None, prologue=PRO_X, x_stride=None, norm_w=None, eps=1e-6, n_split=1, y=None,
         y_stride=None, epilogue=EPI_STORE, res=None, res_stride=None, flags=0, err=None, stream=None):
    """y[m][n] = W[n] . act(x)[m]; W raw GGUF rows (uint8 device tensor or pointer)."""
    import torch
    if M is None:
        M = x.shape[0] if x.dim() > 1 else 1
    xs = x_stride if x_stride is not None else (x.stride(0) if x.dim() > 1 else K)
    if y is None:
        y = torch.empty((M, N), dtype=torch.float32, device=x.device)
    ys = y_stride if y_stride is not None else (y.stride(0) if y.dim() > 1 else N)
    rs = res_stride if res_stride is not None else (res.stride(0) if res is not None and res.dim() > 1 else N)
    _check("acb_gemv", lib().acb_gemv(_ptr(W), w_type, N, K, M, prologue, _ptr(x), xs, _ptr(norm_w), eps, n_split,
                                       _ptr(y), ys, epilogue, _ptr(res), rs, flags, _ptr(err), _stream(stream)))
    return y


def qkv_post(qkv, n_tok, Nh, Nkv, D, q_norm, k_norm, eps, pos, rope, q_out, k_cache, v_cache, max_seq, set0,
             set_per_tok, flags=0, err=None, stream=None):
    _check("acb_qkv_post", lib().acb_qkv_post(
        _ptr(qkv), qkv.stride(0), n_tok, Nh, Nkv, D, _ptr(q_norm), _ptr(k_norm), eps, _ptr(pos), _ptr(rope),
        rope.shape[0], _ptr(q_out), q_out.stride(0), _ptr(k_cache), _ptr(v_cache), max_seq, set0, set_per_tok,
        flags, _ptr(err), _stream(stream)))


def attn_decode_splits(n_tok, Nkv):
    return lib().acb_attn_decode_splits(n_tok, Nkv)


def attn_decode(q, n_tok, Nh, Nkv, D, pos, k_cache, v_cache, max_seq, set0, set_per_tok, scale, n_split, scores,
                smax, part, out=None, tickets=None, flags=0, stream=None):
    _check("acb_attn_decode", lib().acb_attn_decode(
        _ptr(q), q.stride(0), n_tok, Nh, Nkv, D, _ptr(pos), _ptr(k_cache), _ptr(v_cache), max_seq, set0, set_per_tok,
        scale, n_split, _ptr(scores), _ptr(smax), _ptr(part), _ptr(out), out.stride(0) if out is not None else 0,
        _ptr(tickets), flags, _stream(stream)))


def argmax(logits, ids, margin=None, pos_advance=None, scratch=None, flags=0, stream=None):
    import torch
    rows, V = logits.shape
    if scratch is None:
        scratch = torch.zeros(lib().acb_argmax_scratch_bytes(rows, V), dtype=torch.uint8, device=logits.device)
    _check("acb_argmax", lib().acb_argmax(_ptr(logits), logits.stride(0), V, rows, _ptr(ids), _ptr(margin),
                                           _ptr(pos_advance), None, None, 0, None, _ptr(scratch), flags,
                                           _stream(stream)))
    return scratch


# ---- model level ----------------------------------------------------------------------------------

class QW3LM:
    """Qwen3 causal LM (acb_models.h): the qw3lm_* entry points of src/qwen3-lm.h."""

    def __init__(self, gguf_path: str, max_seq_len: int = 0, n_kv_sets: int = 1, device: int = 0):
        import numpy as np
        self.np = np
        h = C.c_void_p()
        st = lib().acb_qw3lm_load(gguf_path.encode(), max_seq_len, n_kv_sets, device, C.byref(h))
        if st != 0:
            raise AcbError(f"acb_qw3lm_load ({lib().acb_last_error().decode()})", st)
        self.h = h
        self.cfg = self._config()

    def _config(self):
        fields = ["vocab_size", "hidden_size", "intermediate_size", "n_heads", "n_kv_heads", "head_dim",
                  "n_layers", "rope_theta", "rms_norm_eps", "tie_embeddings", "max_seq_len"]

        class Cfg(C.Structure):
            _fields_ = [(f, C.c_float if f in ("rope_theta", "rms_norm_eps") else C.c_int) for f in fields]
        c = Cfg()
        fn = lib().acb_qw3lm_get_config
        fn.restype, fn.argtypes = C.c_int, [C.c_void_p, C.POINTER(Cfg)]
        _check("acb_qw3lm_get_config", fn(self.h, C.byref(c)))
        return {f: getattr(c, f) for f in fields}

    def close(self):
        if getattr(self, "h", None):
            lib().acb_qw3lm_free(self.h)
            self.h = None

    __del__ = close

    def weight_bytes(self) -> int:
        return lib().acb_qw3lm_weight_bytes(self.h)

    def kv_pos(self, s=0) -> int:
        return lib().acb_qw3lm_kv_pos(self.h, s)

    def persistent_decode(self) -> bool:
        """True when single-sequence decode runs as one persistent launch per token."""
        return bool(lib().acb_qw3lm_persistent_decode(self.h))

    def reset_kv(self, s=0):
        lib().acb_qw3lm_reset_kv(self.h, s)

    def copy_kv(self, src, dst):
        _check("acb_qw3lm_copy_kv", lib().acb_qw3lm_copy_kv(self.h, src, dst))

    def build_partial_head(self, lm_offset):
        _check("acb_qw3lm_build_partial_head", lib().acb_qw3lm_build_partial_head(self.h, lm_offset))

    def forward(self, ids, kv_set=0):
        np = self.np
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.empty(self.cfg["vocab_size"], dtype=np.float32)
        _check("acb_qw3lm_forward", lib().acb_qw3lm_forward(self.h, ids.ctypes.data, ids.size, kv_set,
                                                             out.ctypes.data))
        return out

    def forward_batch(self, ids, kv_sets, lm_offset=0, lm_count=0, out_v=None):
        np = self.np
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        sets = np.ascontiguousarray(kv_sets, dtype=np.int32)
        V = out_v or (lm_count if lm_count > 0 else self.cfg["vocab_size"])
        out = np.empty((ids.size, V), dtype=np.float32)
        _check("acb_qw3lm_forward_batch", lib().acb_qw3lm_forward_batch(
            self.h, ids.ctypes.data, sets.ctypes.data, ids.size, out.ctypes.data, lm_offset, lm_count))
        return out

    def forward_batch_sample(self, ids, kv_sets, n_active, use_cfg, cfg_scale, eos_idx, code_offset, n_codes,
                             temperature, top_p, top_k, u=None, lm_offset=0, lm_count=0):
        """Device-sampled phase-2 step: compact indices [n_active] (0 = EOS, 1 + c = code c)."""
        np = self.np
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        sets = np.ascontiguousarray(kv_sets, dtype=np.int32)
        uu = None if u is None else np.ascontiguousarray(u, dtype=np.float32)
        out = np.empty(n_active, dtype=np.int32)
        fn = lib().acb_qw3lm_forward_batch_sample
        fn.restype = C.c_int
        fn.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_float, C.c_int, C.c_int, C.c_int,
                       C.c_int, C.c_int, C.c_float, C.c_float, C.c_int, C.c_void_p, C.c_void_p]
        _check("acb_qw3lm_forward_batch_sample", fn(
            self.h, ids.ctypes.data, sets.ctypes.data, n_active, int(bool(use_cfg)), cfg_scale, lm_offset, lm_count,
            eos_idx, code_offset, n_codes, temperature, top_p, top_k, None if uu is None else uu.ctypes.data,
            out.ctypes.data))
        return out

    def generate_greedy(self, last_ids, set0, n_steps, want_margins=False):
        np = self.np
        last = np.ascontiguousarray(last_ids, dtype=np.int32)
        N = last.size
        toks = np.empty((N, n_steps), dtype=np.int32)
        marg = np.empty((N, n_steps), dtype=np.float32) if want_margins else None
        ms = C.c_float(0.0)
        _check("acb_qw3lm_generate_greedy", lib().acb_qw3lm_generate_greedy(
            self.h, last.ctypes.data, set0, N, n_steps, toks.ctypes.data,
            None if marg is None else marg.ctypes.data, C.byref(ms)))
        return toks, marg, ms.value


# ---- dense path ------------------------------------------------------------------------------------

def gemm_bf16(A, B, out=None, out_dtype=None, bias=None, res=None, gate=None, rows_per_sample=None, flags=0,
              err=None, stream=None, workspace=None):
    """C = A @ B.T (+ bias) (res + C or res + C * gate) on tcgen05. A [M,K], B [N,K] bf16 (or f16,
    which sets FLAG_F16) CUDA tensors. With `workspace` (a CUDA tensor of at least
    gemm_workspace_bytes(M, N, K) bytes) small-M shapes split K (acb_gemm_tc)."""
    import torch
    if A.dtype == torch.float16:
        flags |= FLAG_F16
    M, K = A.shape
    N = B.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype or torch.float32, device=A.device)
    gs = 0 if gate is None else (gate.stride(0) if gate.dim() > 1 else 0)
    wsb = 0 if workspace is None else workspace.numel() * workspace.element_size()
    _check("acb_gemm_tc", lib().acb_gemm_tc(
        _ptr(A), A.stride(0), _ptr(B), B.stride(0), M, N, K, _ptr(out), dtype_id(out), out.stride(0), _ptr(bias),
        _ptr(res), res.stride(0) if res is not None else 0, _ptr(gate), gs, rows_per_sample or M, flags,
        _ptr(workspace), wsb, _ptr(err), _stream(stream)))
    return out


def gemm_swiglu_quant(A, B, F, vec_type, layout, bias=None, err=None, stream=None):
    """acb_gemm_swiglu_quant: A [M, K] and B [2F, K] (gate rows then up rows) 16-bit -> the down
    projection's operand [M, F] (PLAIN) or [M, 3F] (GEMM_A), f16 (bf16 for vec_type BF16)."""
    import torch
    M, K = A.shape
    width = 3 * F if layout == LAYOUT_GEMM_A else F
    dt = torch.bfloat16 if vec_type == BF16 else torch.float16
    out = torch.empty((M, width), dtype=dt, device=A.device)
    flags = FLAG_F16 if A.dtype == torch.float16 else 0
    _check("acb_gemm_swiglu_quant", lib().acb_gemm_swiglu_quant(
        _ptr(A), A.stride(0), _ptr(B), B.stride(0), M, F, K, _ptr(bias), vec_type, layout, _ptr(out), dtype_id(out),
        width, flags, _ptr(err), _stream(stream)))
    return out


def gemm_qkv_planes(A, B, nq, nk, q_w, k_w, eps, seq, pos=None, rope=None, lo=True, err=None, stream=None):
    """acb_gemm_qkv_planes: A [M, K], B [(nq + 2 nk)*128, K] 16-bit -> (qk planes [2M or M, (nq+nk)*128] f16,
    vt planes from the V heads as acb_attn_vt lays them out, vt_ld, vt lo offset)."""
    import torch
    M, K = A.shape
    W = (nq + nk) * 128
    qk = torch.empty((2 * M if lo else M, W), dtype=torch.float16, device=A.device)
    B_ = M // seq
    vt_ld = (seq + 7) // 8 * 8
    vt_plane = B_ * nk * 128 * vt_ld
    vt = torch.zeros((2 * vt_plane if lo else vt_plane,), dtype=torch.float16, device=A.device)
    max_pos = rope.shape[0] if rope is not None else 0
    flags = FLAG_F16 if A.dtype == torch.float16 else 0
    _check("acb_gemm_qkv_planes", lib().acb_gemm_qkv_planes(
        _ptr(A), A.stride(0), _ptr(B), B.stride(0), M, K, nq, nk, _ptr(q_w), _ptr(k_w), eps, _ptr(pos), _ptr(rope),
        max_pos, seq, _ptr(qk), W, M * W if lo else 0, _ptr(vt), vt_ld, vt_plane if lo else 0, flags, _ptr(err),
        _stream(stream)))
    return qk, vt, vt_ld, (vt_plane if lo else 0)


def gemm_workspace_bytes(M, N, K) -> int:
    return lib().acb_gemm_workspace_bytes(M, N, K)


MASK_NONE, MASK_CAUSAL, MASK_WINDOW = 0, 1, 2



def gemm_pair_clusters(f16=False):
    """CTA pairs the GEMM runs on at once (0: the pair kernel is off)."""
    return int(lib().acb_gemm_pair_clusters(1 if f16 else 0))

def attn_prefill(q, k, v, Nh, Nkv, mask=MASK_NONE, window=0, causal_off=0, out=None, out_dtype=None, scale=None,
                 flags=0, stream=None):
    """q [B, Sq, >=Nh*128] bf16 (or f16, which sets FLAG_F16), k/v [B, Skv, >=Nkv*128] of the same
    type (views allowed: last dim contiguous)."""
    import math

    import torch
    if q.dtype == torch.float16:
        flags |= FLAG_F16
    B, Sq = q.shape[0], q.shape[1]
    Skv = k.shape[1]
    if out is None:
        out = torch.empty((B, Sq, Nh * 128), dtype=out_dtype or torch.bfloat16, device=q.device)
    _check("acb_attn_prefill", lib().acb_attn_prefill(
        _ptr(q), q.stride(0), q.stride(1), _ptr(k), k.stride(0), k.stride(1), _ptr(v), v.stride(0), v.stride(1),
        _ptr(out), dtype_id(out), out.stride(0), out.stride(1), B, Sq, Skv, Nh, Nkv, 128, mask, window, causal_off,
        scale if scale is not None else 1.0 / math.sqrt(128), flags, _stream(stream)))
    return out


def vec_dot_type(weight_type: int) -> int:
    return lib().acb_vec_dot_type(weight_type)


def act_quant(x, vec_type, out=None, stream=None):
    """x [M, K] f32 CUDA -> [M, K] f16 (bf16 for vec_type BF16) dequantised ggml activation."""
    import torch
    M, K = x.shape
    dt = torch.bfloat16 if vec_type == BF16 else torch.float16
    if out is None:
        out = torch.empty((M, K), dtype=dt, device=x.device)
    _check("acb_act_quant", lib().acb_act_quant(_ptr(x), x.stride(0), M, K, vec_type, _ptr(out), dtype_id(out),
                                                out.stride(0), _stream(stream)))
    return out


def act_quant_swiglu(gu, F, vec_type, out=None, stream=None):
    """gu [M, 2F] f32 fused gate|up rows -> act_quant(silu(g) * u) [M, F]."""
    import torch
    M = gu.shape[0]
    dt = torch.bfloat16 if vec_type == BF16 else torch.float16
    if out is None:
        out = torch.empty((M, F), dtype=dt, device=gu.device)
    _check("acb_act_quant_swiglu", lib().acb_act_quant_swiglu(
        _ptr(gu), gu.stride(0), F, M, F, vec_type, _ptr(out), dtype_id(out), out.stride(0), _stream(stream)))
    return out


class Qwen3Encoder:
    """Qwen3 encoder stack (acb_models.h): qwen3_load_text_encoder / qwen3_forward /
    qwen3_embed_lookup of src/qwen3-enc.h."""

    def __init__(self, gguf_path: str, device: int = 0):
        import numpy as np
        self.np = np
        h = C.c_void_p()
        st = lib().acb_qwen3_load_text_encoder(gguf_path.encode(), device, C.byref(h))
        if st != 0:
            raise AcbError(f"acb_qwen3_load_text_encoder ({lib().acb_last_error().decode()})", st)
        self.h = h
        fields = ["hidden_size", "intermediate_size", "n_heads", "n_kv_heads", "head_dim", "n_layers",
                  "rope_theta", "rms_norm_eps", "is_causal", "vocab_size"]

        class Cfg(C.Structure):
            _fields_ = [(f, C.c_float if f in ("rope_theta", "rms_norm_eps") else C.c_int) for f in fields]
        c = Cfg()
        fn = lib().acb_qwen3_get_config
        fn.restype, fn.argtypes = C.c_int, [C.c_void_p, C.POINTER(Cfg)]
        _check("acb_qwen3_get_config", fn(self.h, C.byref(c)))
        self.cfg = {f: getattr(c, f) for f in fields}

    def close(self):
        if getattr(self, "h", None):
            lib().acb_qwen3_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except (TypeError, AttributeError):  # module globals already torn down at interpreter exit
            pass

    def weight_bytes(self) -> int:
        return lib().acb_qwen3_weight_bytes(self.h)

    def set_exact(self, exact: bool):
        """exact (default): hi/lo split products tracking the reference to fp32 order; fast: f16."""
        _check("acb_qwen3_set_exact", lib().acb_qwen3_set_exact(self.h, int(bool(exact))))

    def forward(self, ids):
        """Host ids [S] -> host hidden states [S][H] f32 (final RMSNorm applied)."""
        ids = self.np.ascontiguousarray(ids, dtype=self.np.int32)
        out = self.np.empty((ids.size, self.cfg["hidden_size"]), dtype=self.np.float32)
        _check("acb_qwen3_forward", lib().acb_qwen3_forward(self.h, ids.ctypes.data, ids.size, out.ctypes.data))
        return out

    def forward_device(self, ids, out, stream=None):
        """Device int32 ids [S] -> device f32 out [S][H], enqueued on the stream."""
        _check("acb_qwen3_forward_device", lib().acb_qwen3_forward_device(
            self.h, _ptr(ids), ids.numel(), _ptr(out), _stream(stream)))
        return out

    def forward_hidden(self, hidden, layer_begin, layer_end, final_norm=False, out=None, stream=None):
        """Layers [layer_begin, layer_end) from device f32 hidden [S][H] -> device f32 [S][H]."""
        import torch
        if out is None:
            out = torch.empty_like(hidden)
        _check("acb_qwen3_forward_hidden", lib().acb_qwen3_forward_hidden(
            self.h, _ptr(hidden), hidden.shape[0], layer_begin, layer_end, int(final_norm), _ptr(out),
            _stream(stream)))
        return out

    def forward_kernels(self) -> int:
        """This library's kernel launches in the last forward (the captured graph's nodes)."""
        return lib().acb_qwen3_forward_kernels(self.h)

    def embed_lookup(self, ids):
        ids = self.np.ascontiguousarray(ids, dtype=self.np.int32)
        out = self.np.empty((ids.size, self.cfg["hidden_size"]), dtype=self.np.float32)
        _check("acb_qwen3_embed_lookup", lib().acb_qwen3_embed_lookup(self.h, ids.ctypes.data, ids.size,
                                                                      out.ctypes.data))
        return out


def sample_top_k_p(logits, temperature, top_p, top_k, u=None, uncond=None, cfg_scale=1.0, col0=-1, span_off=0,
                   span_len=None, stream=None):
    """Device sample_top_k_p over the rows of logits [rows][ld] (see acb.h): returns int32 [rows]
    indices into the compacted row [col0?] + [span_off, span_off + span_len)."""
    import torch
    rows, ld = logits.shape
    if span_len is None:
        span_len = ld - span_off
    Vc = (1 if col0 >= 0 else 0) + span_len
    work = torch.empty(max(1, lib().acb_sample_work_bytes(rows, Vc)) // 4, dtype=torch.float32, device=logits.device)
    idx = torch.empty(rows, dtype=torch.int32, device=logits.device)
    _check("acb_sample_top_k_p", lib().acb_sample_top_k_p(
        _ptr(logits), ld, None if uncond is None else _ptr(uncond), 0 if uncond is None else uncond.shape[1],
        float(cfg_scale), int(col0), int(span_off), int(span_len), rows, float(temperature), float(top_p),
        int(top_k), None if u is None else _ptr(u), _ptr(work), _ptr(idx), _stream(stream)))
    return idx


class Stork4Tables:
    """acb_stork4_tables over numpy copies of {ms, fpa, fpb, recf} (kept alive by this object)."""

    class _C(C.Structure):
        _fields_ = [("ms", C.c_void_p), ("ms_len", C.c_int), ("fpa", C.c_void_p), ("fpb", C.c_void_p),
                    ("recf", C.c_void_p), ("recf_len", C.c_int)]

    def __init__(self, tables):
        import numpy as np
        self.ms = np.ascontiguousarray(tables["ms"], dtype=np.int32)
        self.fpa = np.ascontiguousarray(tables["fpa"], dtype=np.float64)
        self.fpb = np.ascontiguousarray(tables["fpb"], dtype=np.float64)
        self.recf = np.ascontiguousarray(tables["recf"], dtype=np.float64)
        self.c = Stork4Tables._C(self.ms.ctypes.data, self.ms.size, self.fpa.ctypes.data, self.fpb.ctypes.data,
                                 self.recf.ctypes.data, self.recf.size)


class Stork4:
    """STORK4 solver state on device latents (acb_stork4_*, src/solvers/solver-stork.h)."""

    def __init__(self, tables, n, substeps=10):
        self.tables = Stork4Tables(tables)
        h = C.c_void_p()
        fn = lib().acb_stork4_create
        fn.restype, fn.argtypes = C.c_int, [C.c_void_p, C.c_int64, C.c_int, C.POINTER(C.c_void_p)]
        st = fn(C.byref(self.tables.c), int(n), int(substeps), C.byref(h))
        if st != 0:
            raise AcbError(f"acb_stork4_create ({lib().acb_last_error().decode()})", st)
        self.h = h

    def step(self, xt, vt, t_curr, t_prev, stream=None):
        """xt (device f32, in place) <- one STORK4 step with velocity vt (device f32)."""
        fn = lib().acb_stork4_step
        fn.restype, fn.argtypes = C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_float, C.c_float, C.c_void_p]
        _check("acb_stork4_step", fn(self.h, _ptr(xt), _ptr(vt), float(t_curr), float(t_prev), _stream(stream)))

    def close(self):
        if getattr(self, "h", None):
            fn = lib().acb_stork4_free
            fn.restype, fn.argtypes = None, [C.c_void_p]
            fn(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except (TypeError, AttributeError):  # module globals already torn down at interpreter exit
            pass


class VAE:
    """AutoencoderOobleck decoder (acb_models.h): vae_ggml_load / vae_ggml_decode(_tiled) of src/vae.h."""

    def __init__(self, gguf_path: str, device: int = 0):
        h = C.c_void_p()
        fn = lib().acb_vae_load
        fn.restype, fn.argtypes = C.c_int, [C.c_char_p, C.c_int, C.POINTER(C.c_void_p)]
        st = fn(gguf_path.encode(), device, C.byref(h))
        if st != 0:
            raise AcbError(f"acb_vae_load ({lib().acb_last_error().decode()})", st)
        self.h = h
        up = lib().acb_vae_upsample
        up.restype, up.argtypes = C.c_int, [C.c_void_p]
        self.up = up(self.h)

    def close(self):
        if getattr(self, "h", None):
            fn = lib().acb_vae_free
            fn.restype, fn.argtypes = None, [C.c_void_p]
            fn(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except (TypeError, AttributeError):  # module globals already torn down at interpreter exit
            pass

    def decode(self, latent):
        """Host latent [T][64] -> host audio [2][T * upsample]."""
        import numpy as np
        x = np.ascontiguousarray(latent, dtype=np.float32)
        T = x.shape[0]
        out = np.empty(2 * T * self.up, dtype=np.float32)
        n = C.c_int(0)
        fn = lib().acb_vae_decode
        fn.restype, fn.argtypes = C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.POINTER(C.c_int)]
        _check("acb_vae_decode", fn(self.h, x.ctypes.data, T, out.ctypes.data, T * self.up, C.byref(n)))
        return out.reshape(2, n.value)

    def decode_tiled(self, latent, chunk_size=256, overlap=64, cancel=None):
        """vae_ggml_decode_tiled: cancel() is asked before each tile; True stops with ACB_ERR_CANCELLED."""
        import numpy as np
        x = np.ascontiguousarray(latent, dtype=np.float32)
        T = x.shape[0]
        mx = T * self.up
        out = np.empty(2 * mx, dtype=np.float32)
        n = C.c_int(0)
        CANCEL = C.CFUNCTYPE(C.c_int, C.c_void_p)
        cb = CANCEL(lambda _d: 1 if cancel() else 0) if cancel is not None else CANCEL()  # CANCEL(): null
        fn = lib().acb_vae_decode_tiled
        fn.restype = C.c_int
        fn.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_int, CANCEL,
                       C.c_void_p, C.POINTER(C.c_int)]
        _check("acb_vae_decode_tiled", fn(self.h, x.ctypes.data, T, out.ctypes.data, mx, chunk_size, overlap, cb,
                                          None, C.byref(n)))
        return out[:2 * n.value].reshape(2, n.value)

    def decode_device(self, latent, audio, stream=None):
        fn = lib().acb_vae_decode_device
        fn.restype, fn.argtypes = C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]
        _check("acb_vae_decode_device", fn(self.h, _ptr(latent), latent.shape[0], _ptr(audio), _stream(stream)))
        return audio


def fsq_decode_index(index: int):
    """fsq_decode_index (src/fsq-detok.h:18-29): flat code -> 6 floats in [-1, 1]."""
    import numpy as np
    out = np.empty(6, dtype=np.float32)
    lib().acb_fsq_decode_index(int(index), out.ctypes.data)
    return out


def fsq_encode_index(raw6) -> int:
    """fsq_encode_index (src/fsq-tok.h:42-60): 6 project_in outputs -> flat code."""
    import numpy as np
    r = np.ascontiguousarray(raw6, dtype=np.float32)
    return int(lib().acb_fsq_encode_index(r.ctypes.data))


def _load_handle(fn: str, path: str, device: int):
    h = C.c_void_p()
    st = getattr(lib(), fn)(path.encode(), device, C.byref(h))
    if st != 0:
        raise AcbError(f"{fn} ({lib().acb_last_error().decode()})", st)
    return h


class CondEncoder:
    """Condition encoder (acb_models.h): cond_ggml_load / cond_ggml_forward of src/cond-enc.h."""

    FIELDS = ["hidden_size", "text_dim", "lyric_dim", "timbre_dim", "lyric_layers", "timbre_layers", "window",
              "timbre_cls"]

    def __init__(self, gguf_path: str, device: int = 0):
        self.h = _load_handle("acb_cond_load", gguf_path, device)

        class Cfg(C.Structure):
            _fields_ = [(f, C.c_int) for f in CondEncoder.FIELDS]
        c = Cfg()
        fn = lib().acb_cond_get_config
        fn.restype, fn.argtypes = C.c_int, [C.c_void_p, C.POINTER(Cfg)]
        _check("acb_cond_get_config", fn(self.h, C.byref(c)))
        self.cfg = {f: getattr(c, f) for f in CondEncoder.FIELDS}

    def close(self):
        if getattr(self, "h", None):
            lib().acb_cond_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except (TypeError, AttributeError):  # module globals already torn down at interpreter exit
            pass

    def set_exact(self, exact: bool):
        _check("acb_cond_set_exact", lib().acb_cond_set_exact(self.h, int(bool(exact))))

    def forward(self, text_hidden, lyric_embed, timbre_feats=None):
        """Host f32 [S_text][text_dim], [S_lyric][lyric_dim], [S_ref][timbre_dim] or None ->
        packed encoder states [S_lyric + (1) + S_text][hidden_size]."""
        import numpy as np
        t = np.ascontiguousarray(text_hidden, dtype=np.float32)
        ly = np.ascontiguousarray(lyric_embed, dtype=np.float32)
        tb = None if timbre_feats is None else np.ascontiguousarray(timbre_feats, dtype=np.float32)
        S_ref = 0 if tb is None else tb.shape[0]
        S = ly.shape[0] + (1 if S_ref > 0 else 0) + t.shape[0]
        out = np.empty((S, self.cfg["hidden_size"]), dtype=np.float32)
        n = C.c_int(0)
        _check("acb_cond_forward", lib().acb_cond_forward(
            self.h, t.ctypes.data, t.shape[0], ly.ctypes.data, ly.shape[0], None if tb is None else tb.ctypes.data,
            S_ref, out.ctypes.data, C.byref(n)))
        assert n.value == S
        return out

    def forward_device(self, text_hidden, lyric_embed, timbre_feats, out, stream=None):
        """Device tensors in, packed states into device `out`; returns the row count."""
        n = C.c_int(0)
        S_ref = 0 if timbre_feats is None else timbre_feats.shape[0]
        _check("acb_cond_forward_device", lib().acb_cond_forward_device(
            self.h, _ptr(text_hidden), text_hidden.shape[0], _ptr(lyric_embed), lyric_embed.shape[0],
            None if timbre_feats is None else _ptr(timbre_feats), S_ref, _ptr(out), C.byref(n), _stream(stream)))
        return n.value

    def null_embedding(self):
        import numpy as np
        out = np.empty(self.cfg["hidden_size"], dtype=np.float32)
        _check("acb_cond_null_embedding", lib().acb_cond_null_embedding(self.h, out.ctypes.data))
        return out


class Detokenizer:
    """FSQ detokenizer (acb_models.h): detok_ggml_load / detok_ggml_decode of src/fsq-detok.h."""

    def __init__(self, gguf_path: str, device: int = 0):
        self.h = _load_handle("acb_detok_load", gguf_path, device)

    def close(self):
        if getattr(self, "h", None):
            lib().acb_detok_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except (TypeError, AttributeError):  # module globals already torn down at interpreter exit
            pass

    def set_exact(self, exact: bool):
        _check("acb_detok_set_exact", lib().acb_detok_set_exact(self.h, int(bool(exact))))

    def decode(self, codes, channels: int = 64):
        """Host codes [T_5Hz] -> host context latents [T_5Hz * 5][channels]."""
        import numpy as np
        c = np.ascontiguousarray(codes, dtype=np.int32)
        out = np.empty((c.size * 5, channels), dtype=np.float32)
        _check("acb_detok_decode", lib().acb_detok_decode(self.h, c.ctypes.data, c.size, out.ctypes.data))
        return out

    def decode_device(self, codes, out, stream=None):
        _check("acb_detok_decode_device", lib().acb_detok_decode_device(self.h, _ptr(codes), codes.numel(),
                                                                        _ptr(out), _stream(stream)))
        return out


class Tokenizer:
    """FSQ tokenizer (acb_models.h): tok_ggml_load / tok_ggml_encode of src/fsq-tok.h."""

    def __init__(self, gguf_path: str, device: int = 0):
        self.h = _load_handle("acb_tok_load", gguf_path, device)

    def close(self):
        if getattr(self, "h", None):
            lib().acb_tok_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except (TypeError, AttributeError):  # module globals already torn down at interpreter exit
            pass

    def set_exact(self, exact: bool):
        _check("acb_tok_set_exact", lib().acb_tok_set_exact(self.h, int(bool(exact))))

    def encode(self, latents, silence_latent=None):
        """Host latents [T_25Hz][64] (padded to a multiple of 5 from silence_latent) -> codes [T_5Hz]."""
        import numpy as np
        x = np.ascontiguousarray(latents, dtype=np.float32)
        sl = None if silence_latent is None else np.ascontiguousarray(silence_latent, dtype=np.float32)
        codes = np.empty((x.shape[0] + 4) // 5, dtype=np.int32)
        n = C.c_int(0)
        _check("acb_tok_encode", lib().acb_tok_encode(self.h, x.ctypes.data, x.shape[0], codes.ctypes.data,
                                                      None if sl is None else sl.ctypes.data, C.byref(n)))
        assert n.value == codes.size
        return codes

    def encode_device(self, latents, codes, stream=None):
        """Device f32 latents [5 * T_5Hz][64] -> device int32 codes [T_5Hz]."""
        _check("acb_tok_encode_device", lib().acb_tok_encode_device(self.h, _ptr(latents), codes.numel(),
                                                                    _ptr(codes), _stream(stream)))
        return codes


LAYOUT_PLAIN, LAYOUT_GEMM_A, LAYOUT_GEMM_B, LAYOUT_PLANES = 0, 1, 2, 3


def act_quant_ex(x, K, vec_type, layout, up_offset=0, out=None, lo_offset=0, stream=None):
    """acb_act_quant_ex over x [M, >=K] f32 (up_offset > 0: SwiGLU rows)."""
    import torch
    M = x.shape[0]
    dt = torch.bfloat16 if vec_type == BF16 else torch.float16
    width = 3 * K if layout in (LAYOUT_GEMM_A, LAYOUT_GEMM_B) else K
    if out is None:
        out = torch.empty((2 * M if layout == LAYOUT_PLANES else M, width), dtype=dt, device=x.device)
        if layout == LAYOUT_PLANES:
            lo_offset = M * width
    _check("acb_act_quant_ex", lib().acb_act_quant_ex(_ptr(x), x.stride(0), up_offset, M, K, vec_type, layout,
                                                      _ptr(out), dtype_id(out), width, lo_offset, _stream(stream)))
    return out


def norm_quant(x, K, w, eps, vec_type, layout, scale=None, shift=None, rows_per_sample=None, vec_stride=0,
               stream=None):
    """acb_norm_quant over x [M, >=K] f32: RMSNorm (times w) [adaLN with scale/shift] then the
    activation quantiser of act_quant_ex (layouts PLAIN, GEMM_A, PLANES)."""
    import torch
    M = x.shape[0]
    dt = torch.bfloat16 if vec_type == BF16 else torch.float16
    width = 3 * K if layout == LAYOUT_GEMM_A else K
    out = torch.empty((2 * M if layout == LAYOUT_PLANES else M, width), dtype=dt, device=x.device)
    lo_offset = M * width if layout == LAYOUT_PLANES else 0
    rps = rows_per_sample if rows_per_sample is not None else M
    _check("acb_norm_quant", lib().acb_norm_quant(_ptr(x), x.stride(0), M, K, _ptr(w), eps, _ptr(scale), _ptr(shift),
                                                  vec_stride, rps, vec_type, layout, _ptr(out), dtype_id(out), width,
                                                  lo_offset, _stream(stream)))
    return out


def qk_norm_rope_planes(src, n_heads, w, eps, pos=None, rope=None, n_k_heads=0, k_w=None, err=None, stream=None):
    """acb_qk_norm_rope_planes: src [T, >= (n_heads + n_k_heads)*128] -> f16 planes
    [2T, (n_heads + n_k_heads)*128] (hi rows then lo rows); heads past n_heads use k_w."""
    import torch
    T, W = src.shape[0], (n_heads + n_k_heads) * 128
    out = torch.empty((2 * T, W), dtype=torch.float16, device=src.device)
    max_pos = rope.shape[0] if rope is not None else 0
    _check("acb_qk_norm_rope_planes", lib().acb_qk_norm_rope_planes(
        _ptr(src), dtype_id(src), src.stride(0), _ptr(out), W, T * W, T, n_heads, _ptr(w), n_k_heads, _ptr(k_w), 128,
        eps, _ptr(pos), _ptr(rope), max_pos, _ptr(err), _stream(stream)))
    return out


def attn_prefill_split(q, k, v, q_lo, k_lo, v_lo, Nh, Nkv, mask=MASK_NONE, window=0, causal_off=0, out=None,
                       scale=None, flags=0, stream=None):
    """Split-precision attention: q/k/v f16 hi-plane views, *_lo the element offsets of the lo planes."""
    import math

    import torch
    B, Sq = q.shape[0], q.shape[1]
    Skv = k.shape[1]
    if out is None:
        out = torch.empty((B, Sq, Nh * 128), dtype=torch.float32, device=q.device)
    _check("acb_attn_prefill_split", lib().acb_attn_prefill_split(
        _ptr(q), q.stride(0), q.stride(1), _ptr(k), k.stride(0), k.stride(1), _ptr(v), v.stride(0), v.stride(1),
        _ptr(out), dtype_id(out), out.stride(0), out.stride(1), B, Sq, Skv, Nh, Nkv, 128, mask, window, causal_off,
        scale if scale is not None else 1.0 / math.sqrt(128), flags, q_lo, k_lo, v_lo, _stream(stream)))
    return out


class DiT:
    """ACE-Step DiT (acb_models.h): dit_ggml_load / one evaluation / dit_ggml_generate."""

    FIELDS = ["n_layers", "hidden_size", "intermediate_size", "n_heads", "n_kv_heads", "head_dim", "in_channels",
              "out_channels", "patch_size", "sliding_window", "rope_theta", "rms_norm_eps", "enc_hidden_size",
              "has_null_condition"]

    def __init__(self, gguf_path: str, device: int = 0, adapter: str | None = None, adapter_scale: float = 1.0):
        import numpy as np
        self.np = np
        h = C.c_void_p()
        fn = lib().acb_dit_load_ex
        fn.restype, fn.argtypes = C.c_int, [C.c_char_p, C.c_int, C.c_char_p, C.c_float, C.POINTER(C.c_void_p)]
        st = fn(gguf_path.encode(), device, adapter.encode() if adapter else None, float(adapter_scale), C.byref(h))
        if st != 0:
            raise AcbError(f"acb_dit_load_ex ({lib().acb_last_error().decode()})", st)
        self.h = h

        class Cfg(C.Structure):
            _fields_ = [(f, C.c_float if f in ("rope_theta", "rms_norm_eps") else C.c_int) for f in DiT.FIELDS]
        c = Cfg()
        fn = lib().acb_dit_get_config
        fn.restype, fn.argtypes = C.c_int, [C.c_void_p, C.POINTER(Cfg)]
        _check("acb_dit_get_config", fn(self.h, C.byref(c)))
        self.cfg = {f: getattr(c, f) for f in DiT.FIELDS}

    def close(self):
        if getattr(self, "h", None):
            lib().acb_dit_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except (TypeError, AttributeError):  # module globals already torn down at interpreter exit
            pass

    def weight_bytes(self) -> int:
        return lib().acb_dit_weight_bytes(self.h)

    def set_exact(self, exact: bool):
        _check("acb_dit_set_exact", lib().acb_dit_set_exact(self.h, int(bool(exact))))

    def forward(self, x, enc, t, t_r, n_layers_run=-1, out=None, stream=None):
        """x [N, T, in_channels], enc [N, enc_S, enc_hidden] f32 CUDA tensors -> velocity [N, T, out_channels]."""
        import torch
        N, T, _ = x.shape
        if out is None:
            out = torch.empty((N, T, self.cfg["out_channels"]), dtype=torch.float32, device=x.device)
        _check("acb_dit_forward", lib().acb_dit_forward(self.h, _ptr(x), _ptr(enc), N, T, enc.shape[1], float(t),
                                                        float(t_r), _ptr(out), n_layers_run, _stream(stream)))
        return out

    def step_kernels(self) -> int:
        """This library's kernel launches in the last denoise step of the generate / job drivers."""
        return lib().acb_dit_step_kernels(self.h)

    def eval_kernels(self) -> int:
        """Kernel launches in the last captured evaluation graph."""
        return lib().acb_dit_eval_kernels(self.h)

    def set_condition(self, enc, T, stream=None):
        """enc [N, enc_S, enc_hidden] f32 CUDA tensor: embed it and cache the cross K/V."""
        _check("acb_dit_set_condition", lib().acb_dit_set_condition(self.h, _ptr(enc), enc.shape[0], T, enc.shape[1],
                                                                    _stream(stream)))

    def eval(self, x, tt, out, stream=None):
        """One evaluation of x [N, T, in_channels] with tt = device tensor [t, t_r] into out."""
        _check("acb_dit_eval", lib().acb_dit_eval(self.h, _ptr(x), _ptr(tt), _ptr(out), _stream(stream)))
        return out

    SOLVERS = {"euler": 0, "dpm3m": 1}

    def set_lengths(self, real_S=None, real_enc_S=None, stream=None):
        """Padding of the set_condition / eval path: one real length per slot (host ints)."""
        np = self.np
        rs = None if real_S is None else np.ascontiguousarray(real_S, dtype=np.int32)
        re = None if real_enc_S is None else np.ascontiguousarray(real_enc_S, dtype=np.int32)
        _check("acb_dit_set_lengths", lib().acb_dit_set_lengths(
            self.h, None if rs is None else rs.ctypes.data, None if re is None else re.ctypes.data, _stream(stream)))

    def generate_ex(self, noise, context, enc, schedule, guidance_scale=1.0, solver="euler", real_S=None,
                    real_enc_S=None, seeds=None, randn=None, cancel=None, context_switch=None, cover_steps=-1,
                    enc_switch=None, real_enc_S_switch=None, dcw_scaler=0.0, stork_substeps=10, dcw_high_scaler=0.0,
                    dcw_mode="low"):
        """acb_dit_generate_ex (dit_ggml_generate's argument list). randn(seed, n) -> n floats is
        the SDE noise source on the host (None: the reference's Philox stream, drawn on the
        device); cancel(step_count) -> bool is polled before every step. Returns
        (x0, device ms); raises AcbError with status 9 when cancelled."""
        np = self.np
        f32 = lambda a: None if a is None else np.ascontiguousarray(a, dtype=np.float32)
        i32 = lambda a: None if a is None else np.ascontiguousarray(a, dtype=np.int32)
        ptr = lambda a: None if a is None else a.ctypes.data
        noise, context, enc = f32(noise), f32(context), f32(enc)
        cs, es = f32(context_switch), f32(enc_switch)
        rs, re, res = i32(real_S), i32(real_enc_S), i32(real_enc_S_switch)
        sd = None if seeds is None else np.ascontiguousarray(seeds, dtype=np.int64)
        sched = np.ascontiguousarray(schedule, dtype=np.float32)
        N, T, _ = noise.shape
        out = np.empty_like(noise)
        ms = C.c_float(0.0)
        CANCEL = C.CFUNCTYPE(C.c_int, C.c_void_p)
        RANDN = C.CFUNCTYPE(None, C.c_int64, C.POINTER(C.c_float), C.c_int, C.c_void_p)
        calls = [0]

        def _cancel(_):
            calls[0] += 1
            return 1 if cancel(calls[0] - 1) else 0

        def _randn(seed, outp, n, _):
            v = np.ascontiguousarray(randn(int(seed), int(n)), dtype=np.float32)
            C.memmove(outp, v.ctypes.data, 4 * int(n))

        cb_c = CANCEL(_cancel) if cancel is not None else None
        cb_r = RANDN(_randn) if randn is not None else None
        _check("acb_dit_generate_ex", lib().acb_dit_generate_ex(
            self.h, noise.ctypes.data, context.ctypes.data, enc.ctypes.data, enc.shape[1], T, N, sched.size,
            sched.ctypes.data, out.ctypes.data, float(guidance_scale), ptr(cs), int(cover_steps),
            C.cast(cb_c, C.c_void_p) if cb_c else None, None, ptr(rs), ptr(re), ptr(es), ptr(res), ptr(sd), 1,
            float(dcw_scaler), float(dcw_high_scaler), dcw_mode.encode() if dcw_mode else None,
            solver.encode() if solver else None, int(stork_substeps),
            C.cast(cb_r, C.c_void_p) if cb_r else None, None, C.cast(C.pointer(ms), C.c_void_p)))
        return out, ms.value

    def set_stork4_tables(self, tables):
        """ROCK4 tables {ms, fpa [len][6], fpb [len][4], recf} for the "stork4" solver."""
        t = Stork4Tables(tables)
        fn = lib().acb_dit_set_stork4_tables
        fn.restype, fn.argtypes = C.c_int, [C.c_void_p, C.c_void_p]
        _check("acb_dit_set_stork4_tables", fn(self.h, C.byref(t.c)))

    def generate(self, noise, context, enc, schedule, guidance_scale=1.0, solver="euler"):
        """Host arrays: noise [N, T, Oc], context [N, T, in-Oc], enc [N, enc_S, enc_hidden] ->
        (x0 [N, T, Oc], device ms of the step loop). solver: "euler" or "dpm3m"."""
        np = self.np
        noise = np.ascontiguousarray(noise, dtype=np.float32)
        context = np.ascontiguousarray(context, dtype=np.float32)
        enc = np.ascontiguousarray(enc, dtype=np.float32)
        sched = np.ascontiguousarray(schedule, dtype=np.float32)
        N, T, _ = noise.shape
        out = np.empty_like(noise)
        ms = C.c_float(0.0)
        _check("acb_dit_generate_solver", lib().acb_dit_generate_solver(
            self.h, noise.ctypes.data, context.ctypes.data, enc.ctypes.data, enc.shape[1], T, N, sched.size,
            sched.ctypes.data, out.ctypes.data, float(guidance_scale), self.SOLVERS[solver],
            C.cast(C.pointer(ms), C.c_void_p)))
        return out, ms.value


class Comm:
    """acb_comm: the library's NCCL communicator (one process per GPU)."""

    def __init__(self, uid: bytes, world: int, rank: int, device: int = 0, timeout_ms: int = 60000):
        h = C.c_void_p()
        buf = C.create_string_buffer(bytes(uid), 128)
        _check("acb_comm_init", lib().acb_comm_init(buf, world, rank, device, timeout_ms, C.byref(h)))
        self.h = h

    @staticmethod
    def unique_id() -> bytes:
        buf = C.create_string_buffer(128)
        _check("acb_comm_unique_id", lib().acb_comm_unique_id(buf))
        return buf.raw

    def close(self):
        if self.h:
            lib().acb_comm_free(self.h)
            self.h = None


def dit_shard_plan(n_tracks, cfg, world, rank):
    """(track0, n_local, half, peer) of acb_dit_shard_plan."""
    v = [C.c_int() for _ in range(4)]
    _check("acb_dit_shard_plan", lib().acb_dit_shard_plan(n_tracks, int(cfg), world, rank, *[C.byref(x) for x in v]))
    return tuple(x.value for x in v)


def dit_generate_sharded(dit, comm, noise, context, enc, schedule, guidance_scale=1.0, solver="euler", real_S=None,
                         real_enc_S=None, seeds=None, randn=None):
    """acb_dit_generate_sharded: every rank passes the whole job, every rank gets every track's x0."""
    import numpy as np
    f32 = lambda a: None if a is None else np.ascontiguousarray(a, dtype=np.float32)
    i32 = lambda a: None if a is None else np.ascontiguousarray(a, dtype=np.int32)
    ptr = lambda a: None if a is None else a.ctypes.data
    noise, context, enc = f32(noise), f32(context), f32(enc)
    rs, re = i32(real_S), i32(real_enc_S)
    sd = None if seeds is None else np.ascontiguousarray(seeds, dtype=np.int64)
    sched = np.ascontiguousarray(schedule, dtype=np.float32)
    N, T, _ = noise.shape
    out = np.empty_like(noise)
    ms = C.c_float(0.0)
    RANDN = C.CFUNCTYPE(None, C.c_int64, C.POINTER(C.c_float), C.c_int, C.c_void_p)

    def _randn(seed, outp, n, _):
        v = np.ascontiguousarray(randn(int(seed), int(n)), dtype=np.float32)
        C.memmove(outp, v.ctypes.data, 4 * int(n))

    cb_r = RANDN(_randn) if randn is not None else None
    _check("acb_dit_generate_sharded", lib().acb_dit_generate_sharded(
        dit.h, comm.h, noise.ctypes.data, context.ctypes.data, enc.ctypes.data, enc.shape[1], T, N, sched.size,
        sched.ctypes.data, out.ctypes.data, float(guidance_scale), None, -1, None, None, ptr(rs), ptr(re), None, None,
        ptr(sd), solver.encode(), C.cast(cb_r, C.c_void_p) if cb_r else None, None, C.cast(C.pointer(ms), C.c_void_p)))
    return out, ms.value


def turbo_schedule(steps=8, shift=3.0):
    """t_i = shift*t / (1 + (shift - 1)*t) with t = 1 - i/steps (pipeline-synth-ops.cpp:305-309)."""
    import numpy as np
    f = np.float32
    out = []
    for i in range(steps):
        t = f(1.0) - f(i) / f(steps)  # float arithmetic as in the reference
        out.append(float(f(shift) * t / (f(1.0) + (f(shift) - f(1.0)) * t)))
    return out


def dit_apg(cond, uncond, running_avg, first, guidance_scale, out, momentum=-0.75, norm_threshold=2.5, stream=None):
    """APG over cond/uncond [N, T, Oc] CUDA f32 (running_avg float64 [N, T, Oc]) into out."""
    N, T, Oc = cond.shape
    _check("acb_dit_apg", lib().acb_dit_apg(_ptr(cond), _ptr(uncond), _ptr(running_avg), int(first), momentum,
                                            guidance_scale, norm_threshold, N, T, Oc, _ptr(out), _stream(stream)))
    return out


def dit_euler(xt, vt, tt3, last, out=None, stream=None):
    """tt3 = device [t_curr, t_r, t_next]: xt -= vt * (t_curr - t_next), or out = xt - vt * t_curr."""
    _check("acb_dit_euler", lib().acb_dit_euler(_ptr(xt), _ptr(vt), _ptr(tt3), int(last), _ptr(out), xt.numel(),
                                                _stream(stream)))
    return out


def dit_dpm3m(xt, vt, prev_vt, prev_prev_vt, history, tt3, stream=None):
    """DPM++ 3M step in place: xt advances from tt3[0] to tt3[2] with the velocity history
    (history = stored velocities, 0..2), then prev_prev_vt <- prev_vt and prev_vt <- vt."""
    _check("acb_dit_dpm3m", lib().acb_dit_dpm3m(_ptr(xt), _ptr(vt), _ptr(prev_vt), _ptr(prev_prev_vt), int(history),
                                                _ptr(tt3), xt.numel(), _stream(stream)))
    return xt


def dit_sde(xt, vt, noise, tt3, stream=None):
    """SDE ancestral step in place: x0 = xt - vt * tt3[0], then xt = tt3[2] * noise + (1 - tt3[2]) * x0."""
    _check("acb_dit_sde", lib().acb_dit_sde(_ptr(xt), _ptr(vt), _ptr(noise), _ptr(tt3), xt.numel(), _stream(stream)))
    return xt


def dit_sde_philox(xt, vt, step_seeds, tt3, stream=None):
    """SDE ancestral step in place with the noise of track b drawn on the device from the bf16
    Philox stream of step_seeds[b] (device int64 [n_tracks]); xt, vt are [n_tracks, ...]."""
    _check("acb_dit_sde_philox", lib().acb_dit_sde_philox(_ptr(xt), _ptr(vt), _ptr(step_seeds), _ptr(tt3),
                                                          step_seeds.numel(), xt.numel() // step_seeds.numel(),
                                                          _stream(stream)))
    return xt


def philox_randn(seed, n, bf16_round=True, out=None, device="cuda", stream=None):
    """The reference's philox_randn(seed, out, n, bf16_round) (src/philox.h) on the device: a
    float32 tensor [n]."""
    import torch
    if out is None:
        out = torch.empty(int(n), dtype=torch.float32, device=device)
    _check("acb_philox_randn", lib().acb_philox_randn(int(seed), _ptr(out), int(n), 1 if bf16_round else 0,
                                                      _stream(stream)))
    return out


def philox_bits(seed, first, n, device="cuda", stream=None):
    """Raw Philox4x32-10 words of counters {0, 0, first + i}, i < n, under key = seed: uint32 as int32 [n, 4]."""
    import torch
    out = torch.empty((int(n), 4), dtype=torch.int32, device=device)
    _check("acb_philox_bits", lib().acb_philox_bits(int(seed), int(first), int(n), _ptr(out), _stream(stream)))
    return out


def attn_vt(v, Nkv, lo=False, vt_ld=None, out=None, stream=None):
    """v [B, S, >=Nkv*128] (f32 or f16 view) -> V^T f16 [B, Nkv, 128, vt_ld] (and its lo plane:
    returns (vt, lo_offset))."""
    import torch
    B, S = v.shape[0], v.shape[1]
    ld = vt_ld or ((S + 7) // 8 * 8)
    n = B * Nkv * 128 * ld
    if out is None:
        out = torch.zeros((2 if lo else 1) * n, dtype=torch.float16, device=v.device)
    _check("acb_attn_vt", lib().acb_attn_vt(_ptr(v), dtype_id(v), v.stride(0), v.stride(1), B, S, Nkv, 128, _ptr(out),
                                            ld, n if lo else 0, _stream(stream)))
    return out, ld, (n if lo else 0)


def attn_tc(q, k, vt, vt_ld, Nh, Nkv, Sq, Skv, batch, mask=MASK_NONE, window=0, causal_off=0, out=None,
            out_dtype=None, scale=None, q_lo=0, k_lo=0, vt_lo=0, flags=0, err=None, stream=None, quant=None,
            gemm_a=False):
    """q [batch*Sq, q_ts], k [batch*Skv, k_ts] f16 (views allowed), vt from attn_vt -> o [batch*Sq, Nh*128].
    quant=Q8_0 (or F16 / BF16): the output projection's operand instead (16-bit; with gemm_a the
    [hi | hi | lo] layout, 3*Nh*128 columns)."""
    import math

    import torch
    o_type = None
    if quant is not None:
        o_type = quant
        width = (3 if gemm_a else 1) * Nh * 128
        if out is None:
            out = torch.empty((batch * Sq, width), dtype=torch.bfloat16 if quant == BF16 else torch.float16,
                              device=q.device)
        if gemm_a:
            flags |= FLAG_GEMM_A
    if out is None:
        out = torch.empty((batch * Sq, Nh * 128), dtype=out_dtype or torch.float32, device=q.device)
    _check("acb_attn_tc", lib().acb_attn_tc(
        _ptr(q), q.stride(0), _ptr(k), k.stride(0), _ptr(vt), vt_ld, _ptr(out),
        o_type if o_type is not None else dtype_id(out), out.stride(0), batch,
        Sq, Skv, Nh, Nkv, 128, mask, window, causal_off, scale if scale is not None else 1.0 / math.sqrt(128), flags,
        q_lo, k_lo, vt_lo, _ptr(err), _stream(stream)))
    return out
