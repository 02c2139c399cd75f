"""numpy front end of the C oracle (oracle/_build/libacb_oracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline leg, never by the product library. The C sources restate the ggml-CPU arithmetic
of the reference's op-chain (src/qwen3-enc.h, src/qwen3-lm.h, src/dit-graph.h); see
acb_oracle.h for the float rules.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libacb_oracle.so")

F32, F16, Q8_0, Q4_K, Q6_K, Q8_K, BF16 = 0, 1, 8, 12, 14, 15, 30
BLOCK = {F32: (1, 4), F16: (1, 2), BF16: (1, 2), Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210), Q8_K: (256, 292)}

_lib = None


def build() -> str:
    """Compile the oracle with its Makefile (gcc, -ffp-contract=off)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        P, I64, I, F = C.c_void_p, C.c_int64, C.c_int, C.c_float
        sig = {
            "orc_f16_to_f32": (C.c_float, [C.c_uint16]),
            "orc_f32_to_f16": (C.c_uint16, [F]),
            "orc_f32_to_bf16": (C.c_uint16, [F]),
            "orc_row_bytes": (I64, [I, I64]),
            "orc_dequant_row": (I, [I, P, P, I64]),
            "orc_quantize_row_q8_0": (None, [P, P, I64]),
            "orc_quantize_row_q8_K": (None, [P, P, I64]),
            "orc_quantize_row_q4_K": (None, [P, P, I64]),
            "orc_quantize_row_q6_K": (None, [P, P, I64]),
            "orc_get_rows": (I, [I, P, I64, I64, P, I64, P]),
            "orc_rms_norm": (None, [P, P, P, I64, I64, F]),
            "orc_rope_cache": (None, [P, P, I64, I, F]),
            "orc_qk_norm_rope": (None, [P, I64, P, I64, I64, I, I, P, F, P]),
            "orc_swiglu": (None, [P, I64, P, I64, P, I64, I64]),
            "orc_adaln": (None, [P, P, F, P, P, I64, P, I64, I64, I64]),
            "orc_gated_residual": (None, [P, P, P, I64, P, I64, I64, I64]),
            "orc_mul_mat": (I, [I, P, I64, I64, P, I64, P]),
            "orc_attention": (None, [P, I64, P, P, I, I64, I64, P, P, I64, I64, I64, I, I, I, F]),
            "orc_timestep_embedding": (None, [F, I, I, P]),
            "orc_philox4x32_10": (None, [P, C.c_uint32, C.c_uint32, P]),
            "orc_philox_randn": (None, [I64, I64, I, P]),
            "orc_set_threads": (None, [I]),
            "orc_set_mul_mat_mode": (None, [I]),
            "orc_get_mul_mat_mode": (I, []),
            "orc_get_threads": (I, []),
            "orc_fsq_decode_index": (None, [I, P]),
            "orc_fsq_encode_index": (I, [P]),
            "orc_sample_top_k_p": (I, [P, I, F, F, I, F]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def row_bytes(qtype: int, n: int) -> int:
    be, bb = BLOCK[qtype]
    assert n % be == 0
    return n // be * bb


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


def get_threads() -> int:
    return lib().orc_get_threads()


MM_GGML, MM_EXACT = 0, 1


def set_mul_mat_mode(mode: int) -> None:
    """MM_GGML: ggml-CPU quantized mul_mat (activation quantised to Q8_0 / Q8_K); MM_EXACT:
    dequantised weights times the f32 activation in double."""
    lib().orc_set_mul_mat_mode(int(mode))


def get_mul_mat_mode() -> int:
    return lib().orc_get_mul_mat_mode()


class mul_mat_mode:
    """Context manager: `with mul_mat_mode(MM_EXACT): ...` restores the previous mode."""

    def __init__(self, mode):
        self.mode = mode

    def __enter__(self):
        self.prev = get_mul_mat_mode()
        set_mul_mat_mode(self.mode)

    def __exit__(self, *a):
        set_mul_mat_mode(self.prev)


# ---- formats -------------------------------------------------------------------------------

def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even bf16 bits of float32 values (ggml_compute_fp32_to_bf16)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + (0x7FFF + ((u >> 16) & 1))) >> 16).astype(np.uint16)
    return np.where(nan, ((u >> 16) | 64).astype(np.uint16), r)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_bf16(x: np.ndarray) -> np.ndarray:
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


def quantize(x: np.ndarray, qtype: int) -> np.ndarray:
    """Rows of x [..., K] -> raw block bytes [..., row_bytes] (Q8_0, Q8_K, Q4_K, Q6_K, F32, F16, BF16)."""
    x = _f32(x)
    K = x.shape[-1]
    rows = x.reshape(-1, K)
    if qtype == F32:
        return rows.view(np.uint8).reshape(*x.shape[:-1], K * 4)
    if qtype == F16:
        return rows.astype(np.float16).view(np.uint8).reshape(*x.shape[:-1], K * 2)
    if qtype == BF16:
        return f32_to_bf16_bits(rows).view(np.uint8).reshape(*x.shape[:-1], K * 2)
    rb = row_bytes(qtype, K)
    out = np.empty((rows.shape[0], rb), dtype=np.uint8)
    fn = {Q8_0: lib().orc_quantize_row_q8_0, Q8_K: lib().orc_quantize_row_q8_K,
          Q4_K: lib().orc_quantize_row_q4_K, Q6_K: lib().orc_quantize_row_q6_K}[qtype]
    fn(_p(rows), _p(out), rows.size)
    return out.reshape(*x.shape[:-1], rb)


def dequantize(raw: np.ndarray, qtype: int, K: int) -> np.ndarray:
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    rb = row_bytes(qtype, K)
    rows = raw.reshape(-1, rb)
    out = np.empty((rows.shape[0], K), dtype=np.float32)
    rc = lib().orc_dequant_row(qtype, _p(rows), _p(out), rows.shape[0] * K)
    assert rc == 0
    return out.reshape(*raw.shape[:-1], K)


# ---- ops -----------------------------------------------------------------------------------

def get_rows(qtype: int, table: np.ndarray, cols: int, ids: np.ndarray) -> tuple[int, np.ndarray]:
    table = np.ascontiguousarray(table, dtype=np.uint8)
    n_rows = table.size // row_bytes(qtype, cols)
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    out = np.zeros((ids.size, cols), dtype=np.float32)
    rc = lib().orc_get_rows(qtype, _p(table), n_rows, cols, _p(ids), ids.size, _p(out))
    return rc, out


def rms_norm(x, w, eps):
    x = _f32(x)
    cols = x.shape[-1]
    y = np.empty_like(x)
    lib().orc_rms_norm(_p(x), _p(None if w is None else _f32(w)), _p(y), x.size // cols, cols, eps)
    return y


def rope_cache(pos, head_dim, base):
    pos = np.ascontiguousarray(pos, dtype=np.int32)
    c = np.empty((pos.size, head_dim), dtype=np.float32)
    lib().orc_rope_cache(_p(c), _p(pos), pos.size, head_dim, base)
    return c


def qk_norm_rope(x, w, eps, rope):
    """x [T, Hh, D] -> per-head rms_norm*w then NeoX rope with table rows rope[T, D]."""
    x = _f32(x)
    T, Hh, D = x.shape
    y = np.empty_like(x)
    rope = None if rope is None else _f32(rope)
    lib().orc_qk_norm_rope(_p(x), Hh * D, _p(y), Hh * D, T, Hh, D, _p(None if w is None else _f32(w)), eps,
                           _p(rope))
    return y


def swiglu(g, u):
    g, u = _f32(g), _f32(u)
    F = g.shape[-1]
    rows = g.size // F
    out = np.empty_like(g)
    lib().orc_swiglu(_p(g), F, _p(u), F, _p(out), rows, F)
    return out


def adaln(x, w, eps, scale, shift):
    """x [S, T, H]; scale/shift [H] (shared) or [S, H] (per sample)."""
    x = _f32(x)
    S, T, H = x.shape
    scale, shift = _f32(scale), _f32(shift)
    vs = 0 if scale.ndim == 1 else H
    y = np.empty_like(x)
    lib().orc_adaln(_p(x), _p(None if w is None else _f32(w)), eps, _p(scale), _p(shift), vs, _p(y), S, T, H)
    return y


def gated_residual(r, o, gate):
    r, o, gate = _f32(r), _f32(o), _f32(gate)
    S, T, H = r.shape
    vs = 0 if gate.ndim == 1 else H
    out = np.empty_like(r)
    lib().orc_gated_residual(_p(r), _p(o), _p(gate), vs, _p(out), S, T, H)
    return out


def mul_mat(wtype, W_raw, N, K, x):
    x = _f32(x)
    M = x.size // K
    y = np.empty((M, N), dtype=np.float32)
    rc = lib().orc_mul_mat(wtype, _p(np.ascontiguousarray(W_raw)), N, K, _p(x), M, _p(y))
    assert rc == 0
    return y.reshape(*x.shape[:-1], N)


def attention(q, k, v, kv_type, mask, scale, kv_head_major=False):
    """q [Sq, Hq, D] f32; k/v [Skv, Hkv, D] (kv_type F32 float32 or F16 uint16 bits), or
    [Hkv, Skv, D] when kv_head_major. mask [Sq, Skv] additive or None. Returns [Sq, Hq, D]."""
    q = _f32(q)
    Sq, Hq, D = q.shape
    if kv_head_major:
        Hkv, Skv, _ = k.shape
        tok_stride, head_stride = D, Skv * D
    else:
        Skv, Hkv, _ = k.shape
        tok_stride, head_stride = Hkv * D, D
    dt = np.uint16 if kv_type == F16 else np.float32
    k = np.ascontiguousarray(k, dtype=dt)
    v = np.ascontiguousarray(v, dtype=dt)
    out = np.empty_like(q)
    m = None if mask is None else _f32(mask)
    lib().orc_attention(_p(q), Hq * D, _p(k), _p(v), kv_type, tok_stride, head_stride, _p(m), _p(out), Hq * D,
                        Sq, Skv, Hq, Hkv, D, scale)
    return out


def timestep_embedding(t, dim=256, max_period=10000):
    out = np.empty(dim, dtype=np.float32)
    lib().orc_timestep_embedding(t, dim, max_period, _p(out))
    return out


def philox4x32_10(ctr, key):
    """Philox4x32-10 of one counter (4 x u32) under key (2 x u32): 4 x u32 (src/philox.h:50-82)."""
    c = np.ascontiguousarray(ctr, dtype=np.uint32)
    out = np.empty(4, dtype=np.uint32)
    lib().orc_philox4x32_10(_p(c), int(key[0]) & 0xFFFFFFFF, int(key[1]) & 0xFFFFFFFF, _p(out))
    return out


def philox_randn(seed, n, bf16_round=True):
    """philox_randn (src/philox.h:130-136): the reference's seeded N(0, 1) noise, float32 [n]."""
    out = np.empty(n, dtype=np.float32)
    lib().orc_philox_randn(int(seed), int(n), 1 if bf16_round else 0, _p(out))
    return out


# ---- model forwards (acb_oracle_models.h) ----------------------------------------------------

class Tensor(C.Structure):
    _fields_ = [("type", C.c_int), ("data", C.c_void_p), ("K", C.c_int64), ("N", C.c_int64)]


class Qwen3Layer(C.Structure):
    _fields_ = [(n, Tensor) for n in ("attn_norm", "qkv", "q_norm", "k_norm", "o", "post_norm", "gate_up", "down",
                                      "q", "k", "v", "gate", "up")]


class Qwen3(C.Structure):
    _fields_ = [("n_layers", C.c_int), ("H", C.c_int), ("F", C.c_int), ("Nh", C.c_int), ("Nkv", C.c_int),
                ("D", C.c_int), ("V", C.c_int), ("rope_theta", C.c_float), ("eps", C.c_float),
                ("embed", Tensor), ("final_norm", Tensor), ("layers", C.POINTER(Qwen3Layer))]


class KV(C.Structure):
    _fields_ = [("k", C.c_void_p), ("v", C.c_void_p), ("n_sets", C.c_int), ("max_seq", C.c_int)]


class DiTTemb(C.Structure):
    _fields_ = [(n, Tensor) for n in ("l1_w", "l1_b", "l2_w", "l2_b", "tp_w", "tp_b")]


class DiTLayer(C.Structure):
    _fields_ = [(n, Tensor) for n in ("sa_norm", "sa_qkv", "sa_q_norm", "sa_k_norm", "sa_o", "ca_norm", "ca_qkv",
                                      "ca_q_norm", "ca_k_norm", "ca_o", "mlp_norm", "gate_up", "down",
                                      "scale_shift")] + [("layer_type", C.c_int)]


class DiT(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("n_layers", "H", "F", "Nh", "Nkv", "D", "in_ch", "out_ch", "P",
                                       "sliding_window", "H_enc")] + \
               [("rope_theta", C.c_float), ("eps", C.c_float), ("te", DiTTemb), ("te_r", DiTTemb),
                ("proj_in_w", Tensor), ("proj_in_b", Tensor), ("cond_w", Tensor), ("cond_b", Tensor),
                ("layers", C.POINTER(DiTLayer)), ("norm_out", Tensor), ("out_ss", Tensor),
                ("proj_out_w", Tensor), ("proj_out_b", Tensor)]


def _models_lib():
    L = lib()
    if not getattr(L, "_models_bound", False):
        P, I, F = C.c_void_p, C.c_int, C.c_float
        L.orc_qwen3_encode.restype = I
        L.orc_qwen3_encode.argtypes = [C.POINTER(Qwen3), P, I, P]
        L.orc_qwen3_layers.restype = I
        L.orc_qwen3_layers.argtypes = [C.POINTER(Qwen3), P, I, I, I, I, P]
        L.orc_qwen3_layers_ex.restype = I
        L.orc_qwen3_layers_ex.argtypes = [C.POINTER(Qwen3), P, I, I, I, I, I, I, P]
        L.orc_qw3lm_prefill.restype = I
        L.orc_qw3lm_prefill.argtypes = [C.POINTER(Qwen3), C.POINTER(KV), I, I, P, I, P, I, I, P]
        L.orc_qw3lm_decode.restype = I
        L.orc_qw3lm_decode.argtypes = [C.POINTER(Qwen3), C.POINTER(KV), I, P, P, I, P, I, I]
        L.orc_dit_forward.restype = I
        L.orc_dit_forward.argtypes = [C.POINTER(DiT), P, P, I, I, I, F, F, P, I]
        L.orc_dit_forward_masked.restype = I
        L.orc_dit_forward_masked.argtypes = [C.POINTER(DiT), P, P, I, I, I, F, F, P, I, P, P]
        L.orc_dit_begin.restype = P
        L.orc_dit_begin.argtypes = [C.POINTER(DiT), P, P, I, I, I, F, F, P, P]
        L.orc_dit_run_layers.restype = I
        L.orc_dit_run_layers.argtypes = [C.POINTER(DiT), P, I, I]
        L.orc_dit_finish.restype = I
        L.orc_dit_finish.argtypes = [C.POINTER(DiT), P, P]
        L.orc_dit_state_free.restype = None
        L.orc_dit_state_free.argtypes = [P]
        L._models_bound = True
    return L


def tensor(raw: np.ndarray, qtype: int, K: int, N: int, keep: list) -> Tensor:
    """Wrap raw GGUF bytes (or float32 for F32) of a [K, N] tensor; `keep` holds the buffer."""
    a = np.ascontiguousarray(raw)
    keep.append(a)
    return Tensor(qtype, a.ctypes.data, K, N)


class OracleQwen3:
    """Weights dict (name -> (qtype, raw ndarray, K, N)) following the reference's tensor names
    after fusion: embed, final_norm, layers.{i}.{attn_norm,qkv,q_norm,k_norm,o,post_norm,gate_up,down}."""

    def __init__(self, cfg: dict, weights: dict):
        self.keep = []
        self.cfg = cfg
        L = cfg["n_layers"]
        self.layers = (Qwen3Layer * L)()
        for i in range(L):
            for f in Qwen3Layer._fields_:
                key = f"layers.{i}.{f[0]}"
                if key not in weights:  # unfused q/k/v or gate/up absent (or fused ones absent)
                    continue
                qt, raw, K, N = weights[key]
                setattr(self.layers[i], f[0], tensor(raw, qt, K, N, self.keep))
        if "embed" in weights:
            qt, raw, K, N = weights["embed"]
            self.embed_src = (qt, raw, K, N)
            emb = tensor(raw, qt, K, N, self.keep)
        else:  # a stack fed by a projection (condition encoder, FSQ models): no table
            self.embed_src = None
            emb = Tensor(F32, None, 0, 0)
        qt, raw, K, N = weights["final_norm"]
        fn = tensor(raw, qt, K, N, self.keep)
        self.m = Qwen3(L, cfg["H"], cfg["F"], cfg["Nh"], cfg["Nkv"], cfg["D"], cfg["V"], cfg["rope_theta"],
                       cfg["eps"], emb, fn, self.layers)
        self.kv = None

    def encode(self, ids):
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.empty((ids.size, self.cfg["H"]), dtype=np.float32)
        rc = _models_lib().orc_qwen3_encode(C.byref(self.m), _p(ids), ids.size, _p(out))
        assert rc == 0
        return out

    def embed_rows(self, ids):
        """get_rows of the embedding table (the encoder's first hidden states)."""
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        qt, raw, K, _N = self.embed_src
        rc, out = get_rows(qt, raw, K, ids)
        assert rc == 0
        return out

    def run_layers(self, hidden, l0, l1, causal=True, final_norm=False, batch=1, window=0):
        """Layers [l0, l1) from hidden [batch*S][H] (returned updated; with final_norm also the
        normed output): qwen3_build_layers over a layer range, `batch` independent sequences of S
        rows, and on a bidirectional stack with window > 0 the sliding window of the even layers."""
        h = np.array(hidden, dtype=np.float32, copy=True, order="C")
        R = h.shape[0]
        assert R % batch == 0
        out = np.empty_like(h) if final_norm else None
        rc = _models_lib().orc_qwen3_layers_ex(C.byref(self.m), _p(h), batch, R // batch, l0, l1, int(causal),
                                               window, _p(out) if out is not None else None)
        assert rc == 0
        return (h, out) if final_norm else h

    def alloc_kv(self, n_sets: int, max_seq: int):
        c = self.cfg
        shape = (c["n_layers"], n_sets, c["Nkv"], max_seq, c["D"])
        self.kbuf = np.zeros(shape, dtype=np.uint16)
        self.vbuf = np.zeros(shape, dtype=np.uint16)
        self.kv = KV(self.kbuf.ctypes.data, self.vbuf.ctypes.data, n_sets, max_seq)
        self.kv_pos = [0] * n_sets

    def prefill(self, ids, set_=0, lm_offset=0, lm_count=0, want_hidden=False):
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        V = lm_count if lm_count > 0 else self.cfg["V"]
        logits = np.empty(V, dtype=np.float32)
        hid = np.empty((ids.size, self.cfg["H"]), dtype=np.float32) if want_hidden else None
        rc = _models_lib().orc_qw3lm_prefill(C.byref(self.m), C.byref(self.kv), set_, self.kv_pos[set_], _p(ids),
                                             ids.size, _p(logits), lm_offset, lm_count, _p(hid))
        assert rc == 0
        self.kv_pos[set_] += ids.size
        return (logits, hid) if want_hidden else logits

    def decode(self, ids, set0=0, lm_offset=0, lm_count=0):
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        N = ids.size
        pos = np.array(self.kv_pos[set0:set0 + N], dtype=np.int32)
        V = lm_count if lm_count > 0 else self.cfg["V"]
        logits = np.empty((N, V), dtype=np.float32)
        rc = _models_lib().orc_qw3lm_decode(C.byref(self.m), C.byref(self.kv), set0, _p(pos), _p(ids), N,
                                            _p(logits), lm_offset, lm_count)
        assert rc == 0
        for i in range(N):
            self.kv_pos[set0 + i] += 1
        return logits


class OracleDiT:
    """Weights dict (name -> (qtype, raw, K, N)) with names te.*, te_r.*, proj_in_w, proj_in_b,
    cond_w, cond_b, layers.{i}.<DiTLayer field>, norm_out, out_ss, proj_out_w, proj_out_b."""

    def __init__(self, cfg: dict, weights: dict):
        self.keep = []
        self.cfg = cfg
        L = cfg["n_layers"]
        self.layers = (DiTLayer * L)()
        for i in range(L):
            for f in DiTLayer._fields_[:-1]:
                qt, raw, K, N = weights[f"layers.{i}.{f[0]}"]
                setattr(self.layers[i], f[0], tensor(raw, qt, K, N, self.keep))
            self.layers[i].layer_type = 0 if i % 2 == 0 else 1

        def T(name):
            qt, raw, K, N = weights[name]
            return tensor(raw, qt, K, N, self.keep)

        te = DiTTemb(*[T(f"te.{n}") for n, _ in DiTTemb._fields_])
        te_r = DiTTemb(*[T(f"te_r.{n}") for n, _ in DiTTemb._fields_])
        self.m = DiT(L, cfg["H"], cfg["F"], cfg["Nh"], cfg["Nkv"], cfg["D"], cfg["in_ch"], cfg["out_ch"], cfg["P"],
                     cfg["sliding_window"], cfg["H_enc"], cfg["rope_theta"], cfg["eps"], te, te_r,
                     T("proj_in_w"), T("proj_in_b"), T("cond_w"), T("cond_b"), self.layers, T("norm_out"),
                     T("out_ss"), T("proj_out_w"), T("proj_out_b"))

    def forward(self, x, enc, t, t_r, n_layers_run=-1, real_S=None, real_enc_S=None):
        """real_S / real_enc_S: per-sequence real patch positions / condition rows (padding
        masks of dit_ggml_generate), or None."""
        x = _f32(x)
        enc = _f32(enc)
        N, T_, _ = x.shape
        enc_S = enc.shape[1]
        out = np.empty((N, T_, self.cfg["out_ch"]), dtype=np.float32)
        rs = None if real_S is None else np.ascontiguousarray(real_S, dtype=np.int32)
        re = None if real_enc_S is None else np.ascontiguousarray(real_enc_S, dtype=np.int32)
        rc = _models_lib().orc_dit_forward_masked(C.byref(self.m), _p(x), _p(enc), N, T_, enc_S, t, t_r, _p(out),
                                                  n_layers_run, None if rs is None else _p(rs),
                                                  None if re is None else _p(re))
        assert rc == 0
        return out

    def begin(self, x, enc, t, t_r):
        """Start an evaluation whose layers run in slices (run_layers), then finish()."""
        self._x, self._e = _f32(x), _f32(enc)
        self._shape = self._x.shape
        self._st = _models_lib().orc_dit_begin(C.byref(self.m), _p(self._x), _p(self._e), self._shape[0],
                                               self._shape[1], self._e.shape[1], t, t_r, None, None)
        assert self._st

    def run_layers(self, l0, l1):
        assert _models_lib().orc_dit_run_layers(C.byref(self.m), self._st, l0, l1) == 0

    def finish(self):
        out = np.empty((self._shape[0], self._shape[1], self.cfg["out_ch"]), dtype=np.float32)
        rc = _models_lib().orc_dit_finish(C.byref(self.m), self._st, _p(out))
        _models_lib().orc_dit_state_free(self._st)
        self._st = None
        assert rc == 0
        return out


def qwen3_from_gguf_tensors(cfg, tensors, prefix="model."):
    """OracleQwen3 over raw GGUF tensors {name: (qtype, raw, K, N)} with the reference names
    (model.layers.{i}.self_attn.q_proj.weight, ...; prefix "" for the text encoder's
    layers.{i}...), fused like gf_load_qkv_fused / gf_load_pair_fused
    (src/gguf-weights.h:281-354) when the types match."""
    L = cfg["num_hidden_layers"]
    w = {"embed": tensors[f"{prefix}embed_tokens.weight"], "final_norm": tensors[f"{prefix}norm.weight"]}
    for i in range(L):
        p = f"{prefix}layers.{i}"
        w[f"layers.{i}.attn_norm"] = tensors[f"{p}.input_layernorm.weight"]
        w[f"layers.{i}.post_norm"] = tensors[f"{p}.post_attention_layernorm.weight"]
        w[f"layers.{i}.q_norm"] = tensors[f"{p}.self_attn.q_norm.weight"]
        w[f"layers.{i}.k_norm"] = tensors[f"{p}.self_attn.k_norm.weight"]
        w[f"layers.{i}.o"] = tensors[f"{p}.self_attn.o_proj.weight"]
        w[f"layers.{i}.down"] = tensors[f"{p}.mlp.down_proj.weight"]
        q, k, v = (tensors[f"{p}.self_attn.{n}_proj.weight"] for n in "qkv")
        if q[0] == k[0] == v[0]:
            w[f"layers.{i}.qkv"] = (q[0], np.concatenate([q[1], k[1], v[1]]), q[2], q[3] + k[3] + v[3])
        else:
            w[f"layers.{i}.q"], w[f"layers.{i}.k"], w[f"layers.{i}.v"] = q, k, v
        g, u = tensors[f"{p}.mlp.gate_proj.weight"], tensors[f"{p}.mlp.up_proj.weight"]
        if g[0] == u[0]:
            w[f"layers.{i}.gate_up"] = (g[0], np.concatenate([g[1], u[1]]), g[2], g[3] + u[3])
        else:
            w[f"layers.{i}.gate"], w[f"layers.{i}.up"] = g, u
    oc = dict(n_layers=L, H=cfg["hidden_size"], F=cfg["intermediate_size"], Nh=cfg["num_attention_heads"],
              Nkv=cfg["num_key_value_heads"], D=cfg["head_dim"], V=cfg["vocab_size"], rope_theta=cfg["rope_theta"],
              eps=cfg["rms_norm_eps"])
    return OracleQwen3(oc, w)


def dit_from_gguf_tensors(cfg, tensors):
    """OracleDiT over the raw tensors of a DiT GGUF {name: (qtype, raw, K, shape)} with the
    reference's names (decoder.*): Q||K||V and gate||up concatenated by rows, proj_in / proj_out
    pre-permuted to F32 like dit_load_proj_in_w / dit_load_proj_out_w (src/dit.h:142-252).
    cfg uses the acb_dit_config field names."""
    H, L = cfg["hidden_size"], cfg["n_layers"]
    in_ch, oc, P = cfg["in_channels"], cfg["out_channels"], cfg["patch_size"]

    def plain(name):
        qt, raw, K, shape = tensors[name]
        if qt == F32:
            a = np.ascontiguousarray(raw, dtype=np.float32).reshape(-1)
            return (F32, a, K, a.size // K)
        return (qt, raw, K, shape[0])

    def f32_of(name):
        qt, raw, K, shape = tensors[name]
        if qt == BF16:
            return bf16_bits_to_f32(np.asarray(raw).view(np.uint16)).reshape(shape)
        return np.asarray(raw, dtype=np.float32).reshape(shape)

    def cat(names):
        parts = [tensors[n] for n in names]
        assert len({p[0] for p in parts}) == 1, "stacked projections of one type only"
        return (parts[0][0], np.concatenate([p[1] for p in parts]), parts[0][2], sum(p[3][0] for p in parts))

    w = {}
    for pre, key in (("decoder.time_embed", "te"), ("decoder.time_embed_r", "te_r")):
        w[f"{key}.l1_w"] = plain(f"{pre}.linear_1.weight")
        w[f"{key}.l1_b"] = plain(f"{pre}.linear_1.bias")
        w[f"{key}.l2_w"] = plain(f"{pre}.linear_2.weight")
        w[f"{key}.l2_b"] = plain(f"{pre}.linear_2.bias")
        w[f"{key}.tp_w"] = plain(f"{pre}.time_proj.weight")
        w[f"{key}.tp_b"] = plain(f"{pre}.time_proj.bias")
    pin = np.ascontiguousarray(f32_of("decoder.proj_in.1.weight").transpose(0, 2, 1).reshape(H, P * in_ch))
    w["proj_in_w"] = (F32, pin, P * in_ch, H)
    w["proj_in_b"] = plain("decoder.proj_in.1.bias")
    w["cond_w"] = plain("decoder.condition_embedder.weight")
    w["cond_b"] = plain("decoder.condition_embedder.bias")
    for i in range(L):
        p = f"decoder.layers.{i}"
        w[f"layers.{i}.sa_norm"] = plain(f"{p}.self_attn_norm.weight")
        w[f"layers.{i}.sa_qkv"] = cat([f"{p}.self_attn.{n}_proj.weight" for n in "qkv"])
        w[f"layers.{i}.sa_q_norm"] = plain(f"{p}.self_attn.q_norm.weight")
        w[f"layers.{i}.sa_k_norm"] = plain(f"{p}.self_attn.k_norm.weight")
        w[f"layers.{i}.sa_o"] = plain(f"{p}.self_attn.o_proj.weight")
        w[f"layers.{i}.ca_norm"] = plain(f"{p}.cross_attn_norm.weight")
        w[f"layers.{i}.ca_qkv"] = cat([f"{p}.cross_attn.{n}_proj.weight" for n in "qkv"])
        w[f"layers.{i}.ca_q_norm"] = plain(f"{p}.cross_attn.q_norm.weight")
        w[f"layers.{i}.ca_k_norm"] = plain(f"{p}.cross_attn.k_norm.weight")
        w[f"layers.{i}.ca_o"] = plain(f"{p}.cross_attn.o_proj.weight")
        w[f"layers.{i}.mlp_norm"] = plain(f"{p}.mlp_norm.weight")
        w[f"layers.{i}.gate_up"] = cat([f"{p}.mlp.gate_proj.weight", f"{p}.mlp.up_proj.weight"])
        w[f"layers.{i}.down"] = plain(f"{p}.mlp.down_proj.weight")
        sst = f32_of(f"{p}.scale_shift_table").reshape(-1)
        w[f"layers.{i}.scale_shift"] = (F32, sst, H, 6)
    w["norm_out"] = plain("decoder.norm_out.weight")
    w["out_ss"] = (F32, f32_of("decoder.scale_shift_table").reshape(-1), H, 2)
    pout = np.ascontiguousarray(f32_of("decoder.proj_out.1.weight").transpose(2, 1, 0).reshape(P * oc, H))
    w["proj_out_w"] = (F32, pout, H, P * oc)
    w["proj_out_b"] = plain("decoder.proj_out.1.bias")
    oc_cfg = dict(n_layers=L, H=H, F=cfg["intermediate_size"], Nh=cfg["n_heads"], Nkv=cfg["n_kv_heads"],
                  D=cfg["head_dim"], in_ch=in_ch, out_ch=oc, P=P, sliding_window=cfg["sliding_window"],
                  H_enc=cfg["enc_hidden_size"], rope_theta=cfg["rope_theta"], eps=cfg["rms_norm_eps"])
    return OracleDiT(oc_cfg, w)


def dit_generate(od, noise, context, enc, null_emb, schedule, guidance_scale, momentum=-0.75, norm_threshold=2.5,
                 solver="euler", real_S=None, real_enc_S=None, seeds=None, randn=None, context_switch=None,
                 cover_steps=-1, enc_switch=None, real_enc_S_switch=None, stork_tables=None, stork_substeps=10,
                 dcw_scaler=0.0, dcw_high_scaler=0.0, dcw_mode="low"):
    """dit_ggml_generate (src/dit-sampler.h:132-711) over an OracleDiT with the Euler solver,
    DPM++ 3M (solver="dpm3m", solver-dpm.h:14-50) or SDE ancestral (solver="sde",
    solver-sde.h:17-38; randn(seed, n) gives the fresh noise of track b at step k from seed
    seeds[b] + k + 1): batched CFG with APG in double when guidance_scale > 1 and a null
    condition is given; padding masks from real_S / real_enc_S (the unconditional slots use
    their track's lengths, :276-281,300-302); cover mode (:414-449): from step cover_steps on,
    the context of every slot is context_switch and the conditional slots' condition is
    enc_switch (with real_enc_S_switch, for the conditional slots only: the unconditional slots
    keep their cross-attention mask). Returns x0 [N][T][out_ch]."""
    N, T, Oc = noise.shape
    xt = noise.astype(np.float32).copy()
    hist1 = hist2 = None
    cfg_on = guidance_scale > 1.0 and null_emb is not None
    ra = None
    rs = None if real_S is None else np.asarray(real_S, np.int32)
    re = None if real_enc_S is None else np.asarray(real_enc_S, np.int32)
    re_unc = re
    switched = False
    stork = Stork4(stork_tables, stork_substeps) if solver == "stork4" else None
    for step, t in enumerate(schedule):
        if context_switch is not None and cover_steps >= 0 and step >= cover_steps and not switched:
            switched = True
            context = context_switch
            if enc_switch is not None:
                enc = enc_switch
                if real_enc_S_switch is not None:
                    re = np.asarray(real_enc_S_switch, np.int32)
        x_in = np.concatenate([context, xt], axis=2).astype(np.float32)
        rs_g, re_g = rs, re
        if cfg_on:
            x_in = np.concatenate([x_in, x_in])
            e = np.concatenate([enc, np.broadcast_to(null_emb, enc.shape)]).astype(np.float32)
            rs_g = None if rs is None else np.concatenate([rs, rs])
            if re is not None or re_unc is not None:
                full = np.full(N, enc.shape[1], np.int32)
                re_g = np.concatenate([full if re is None else re, full if re_unc is None else re_unc])
        else:
            e = enc
        v = od.forward(x_in, e, float(t), float(t), real_S=rs_g, real_enc_S=re_g)
        if cfg_on:
            cond, unc = v[:N].astype(np.float64), v[N:].astype(np.float64)
            diff = cond - unc
            ra = diff if ra is None else diff + momentum * ra
            n2 = (ra * ra).sum(axis=1, keepdims=True)          # per (sample, channel) over T
            nr = np.sqrt(np.maximum(n2, 0.0))
            s = np.where(nr > 1e-60, np.minimum(1.0, norm_threshold / np.where(nr > 1e-60, nr, 1.0)), 1.0)
            d = np.where(s < 1.0, ra * s, ra)
            v2 = (cond * cond).sum(axis=1, keepdims=True)
            inv = np.where(v2 > 1e-60, 1.0 / np.sqrt(np.where(v2 > 1e-60, v2, 1.0)), 0.0)
            dot = (d * (cond * inv)).sum(axis=1, keepdims=True)
            orth = d - dot * (cond * inv)
            v = (cond + (guidance_scale - 1.0) * orth).astype(np.float32)
        if step == len(schedule) - 1:
            return (xt - v * np.float32(t)).astype(np.float32)
        if solver == "dpm3m":
            xt, hist1, hist2 = dpm3m_step(xt, v, hist1, hist2, t, schedule[step + 1])
        elif stork is not None:
            xt = stork.step(xt, v, t, schedule[step + 1])
        elif solver == "sde":
            fresh = np.stack([np.asarray(randn(int(seeds[b]) + step + 1, T * Oc), np.float32).reshape(T, Oc)
                              for b in range(N)])
            xt = sde_step(xt, v, fresh, t, schedule[step + 1])
            continue  # SDE injects noise: no DCW
        else:
            dt = np.float32(np.float32(t) - np.float32(schedule[step + 1]))
            xt = (xt - v * dt).astype(np.float32)
        if dcw_scaler > 0.0 or dcw_high_scaler > 0.0:
            xt = dcw_step(xt, v, t, schedule[step + 1], dcw_scaler, dcw_high_scaler, dcw_mode)
    return xt


def _haar_fwd(x):
    """dwt_haar_fwd_tc (src/dwt-haar.h:24-50) along axis 1 of [N][T][C] f32 (zero-padded odd T)."""
    f, r = np.float32, np.float32(0.70710678118654752440)
    N, T, C = x.shape
    a = x[:, 0::2]
    b = np.zeros_like(a)
    b[:, :x[:, 1::2].shape[1]] = x[:, 1::2]
    L = ((a + b).astype(f) * r).astype(f)
    H = ((a - b).astype(f) * r).astype(f)
    if T % 2:  # the lone last frame: L = H = a / sqrt(2)
        L[:, -1] = (a[:, -1] * r).astype(f)
        H[:, -1] = (a[:, -1] * r).astype(f)
    return L, H


def _haar_inv(L, H, T):
    """dwt_haar_inv_tc (:54-75): exactly T frames."""
    f, r = np.float32, np.float32(0.70710678118654752440)
    out = np.empty((L.shape[0], T, L.shape[2]), np.float32)
    out[:, 0::2] = ((L + H).astype(f) * r).astype(f)
    out[:, 1::2] = (((L - H).astype(f) * r).astype(f))[:, :T // 2]
    return out


def dcw_step(xt, v, t_curr, t_next, dcw_scaler, dcw_high_scaler, mode):
    """DCW after an ODE solver step (src/dit-sampler.h:613-666, src/dwt-haar.h): denoised = xt -
    v * t_next from the updated xt; modes low (s = t_curr * scaler on the low band), high ((1 -
    t_curr) * scaler, high band), double (both, the high one with dcw_high_scaler), pix (xt +=
    scaler * (xt - denoised), no transform); an unknown mode is low. A zero effective scale leaves
    xt untouched (the reference returns before the transform)."""
    f = np.float32
    t_curr, t_next = f(t_curr), f(t_next)
    mode = mode if mode in ("low", "high", "double", "pix") else "low"
    s_low = f(t_curr * f(dcw_scaler))
    s_high = f((f(1.0) - t_curr) * f(dcw_scaler))
    s_dh = f((f(1.0) - t_curr) * f(dcw_high_scaler))
    den = (xt - (v * t_next).astype(f)).astype(f)
    if mode == "pix":
        s = f(dcw_scaler)
        return xt if s == 0 else (xt + (s * (xt - den).astype(f)).astype(f)).astype(f)
    if (mode == "low" and s_low == 0) or (mode == "high" and s_high == 0) or \
            (mode == "double" and s_low == 0 and s_dh == 0):
        return xt
    xL, xH = _haar_fwd(xt)
    yL, yH = _haar_fwd(den)
    if mode in ("low", "double") and s_low != 0:
        xL = (xL + (s_low * (xL - yL).astype(f)).astype(f)).astype(f)
    if mode == "high":
        xH = (xH + (s_high * (xH - yH).astype(f)).astype(f)).astype(f)
    if mode == "double" and s_dh != 0:
        xH = (xH + (s_dh * (xH - yH).astype(f)).astype(f)).astype(f)
    return _haar_inv(xL, xH, xt.shape[1])


def dpm3m_step(xt, vt, prev_vt, prev_prev_vt, t_curr, t_next):
    """One DPM++ 3M step (src/solvers/solver-dpm.h:14-50), in float32 with every product and sum
    rounded in the reference's source order: third-order Adams-Bashforth with two stored
    velocities, second order with one (prev_prev_vt None), Euler with none (prev_vt None).
    Returns (xt, prev_vt, prev_prev_vt) after the step: the history moves down by one."""
    f = np.float32
    vt = np.asarray(vt, dtype=np.float32)
    dt = f(f(t_curr) - f(t_next))
    if prev_vt is not None and prev_prev_vt is not None:
        c0, c1, c2 = f(23.0) / f(12.0), f(16.0) / f(12.0), f(5.0) / f(12.0)
        v = ((c0 * vt).astype(np.float32) - (c1 * prev_vt).astype(np.float32)).astype(np.float32)
        v = (v + (c2 * prev_prev_vt).astype(np.float32)).astype(np.float32)
    elif prev_vt is not None:
        v = ((f(1.5) * vt).astype(np.float32) - (f(0.5) * prev_vt).astype(np.float32)).astype(np.float32)
    else:
        v = vt
    xt = (np.asarray(xt, dtype=np.float32) - (v * dt).astype(np.float32)).astype(np.float32)
    return xt, vt.copy(), (None if prev_vt is None else np.asarray(prev_vt, dtype=np.float32).copy())


def sde_step(xt, vt, noise, t_curr, t_next):
    """One SDE ancestral step (src/solvers/solver-sde.h:17-38) in float32, rounded in the
    reference's order: x0 = xt - vt * t_curr; xt = t_next * noise + (1 - t_next) * x0. The noise
    (Philox N(0,1) rounded to bf16 in the reference) is an input."""
    f = np.float32
    x0 = (np.asarray(xt, np.float32) - (np.asarray(vt, np.float32) * f(t_curr)).astype(np.float32)).astype(np.float32)
    a = (f(t_next) * np.asarray(noise, np.float32)).astype(np.float32)
    b = ((f(1.0) - f(t_next)) * x0).astype(np.float32)
    return (a + b).astype(np.float32)


# ---- condition encoder and FSQ models (src/cond-enc.h, src/fsq-detok.h, src/fsq-tok.h) ----------

def fsq_decode_index(index: int) -> np.ndarray:
    out = np.empty(6, dtype=np.float32)
    lib().orc_fsq_decode_index(int(index), _p(out))
    return out


def fsq_encode_index(raw6) -> int:
    r = np.ascontiguousarray(raw6, dtype=np.float32)
    return int(lib().orc_fsq_encode_index(_p(r)))


def stack_from_gguf_tensors(tensors, prefix):
    """OracleQwen3 (no embedding table) over the stack `prefix`layers.{i}.* / `prefix`norm.weight,
    sizes from the tensor shapes; tensors {name: (qtype, raw, K, shape)} as synthetic's keep."""
    L = 0
    while f"{prefix}layers.{L}.input_layernorm.weight" in tensors:
        L += 1
    D = tensors[f"{prefix}layers.0.self_attn.q_norm.weight"][2]
    H = tensors[f"{prefix}norm.weight"][2]

    def rows(t):
        return int(np.prod(t[3])) // t[2]

    cfg = dict(num_hidden_layers=L, hidden_size=H, head_dim=D,
               intermediate_size=rows(tensors[f"{prefix}layers.0.mlp.gate_proj.weight"]),
               num_attention_heads=rows(tensors[f"{prefix}layers.0.self_attn.q_proj.weight"]) // D,
               num_key_value_heads=rows(tensors[f"{prefix}layers.0.self_attn.k_proj.weight"]) // D,
               vocab_size=0, rope_theta=1000000.0, rms_norm_eps=1e-6)
    w = {}
    for i in range(L):
        p = f"{prefix}layers.{i}"
        w[f"layers.{i}.attn_norm"] = _t4(tensors[f"{p}.input_layernorm.weight"])
        w[f"layers.{i}.post_norm"] = _t4(tensors[f"{p}.post_attention_layernorm.weight"])
        w[f"layers.{i}.q_norm"] = _t4(tensors[f"{p}.self_attn.q_norm.weight"])
        w[f"layers.{i}.k_norm"] = _t4(tensors[f"{p}.self_attn.k_norm.weight"])
        w[f"layers.{i}.o"] = _t4(tensors[f"{p}.self_attn.o_proj.weight"])
        w[f"layers.{i}.down"] = _t4(tensors[f"{p}.mlp.down_proj.weight"])
        for n in "qkv":
            w[f"layers.{i}.{n}"] = _t4(tensors[f"{p}.self_attn.{n}_proj.weight"])
        w[f"layers.{i}.gate"] = _t4(tensors[f"{p}.mlp.gate_proj.weight"])
        w[f"layers.{i}.up"] = _t4(tensors[f"{p}.mlp.up_proj.weight"])
    w["final_norm"] = _t4(tensors[f"{prefix}norm.weight"])
    oc = dict(n_layers=L, H=H, F=cfg["intermediate_size"], Nh=cfg["num_attention_heads"],
              Nkv=cfg["num_key_value_heads"], D=D, V=0, rope_theta=cfg["rope_theta"], eps=cfg["rms_norm_eps"])
    return OracleQwen3(oc, w)


def _t4(t):
    """(qtype, raw, K, shape) -> (qtype, raw, K, N) for OracleQwen3."""
    qt, raw, K, shape = t
    return qt, raw, K, int(np.prod(shape)) // K


def _linear(t, x, bias=None):
    """ggml_mul_mat(W, x) (+ ggml_add(bias)) for a tensor (qtype, raw, K, shape)."""
    qt, raw, K, shape = t
    N = int(np.prod(shape)) // K
    y = mul_mat(qt, raw, N, K, np.ascontiguousarray(x, dtype=np.float32).reshape(-1, K))
    if bias is not None:
        y = y + _f32_of(bias).reshape(1, N)
    return y


def _f32_of(t):
    """A small tensor as float32 (gf_load_tensor_f32, or ggml_cast of a quantised one)."""
    qt, raw, K, shape = t
    if qt == F32:
        return np.asarray(raw, dtype=np.float32).reshape(-1, K)
    if qt == BF16:
        return bf16_bits_to_f32(np.asarray(raw, dtype=np.uint16)).reshape(-1, K)
    if qt == F16:
        return np.asarray(raw, dtype=np.uint16).view(np.float16).astype(np.float32).reshape(-1, K)
    return dequantize(np.asarray(raw).reshape(-1, row_bytes(qt, K)), qt, K)


class OracleCond:
    """cond_ggml_forward (src/cond-enc.h:171-381) over raw tensors: lyric stack with the window
    128 mask on even layers, timbre stack (CLS prepended when timbre_cls), text projector."""

    def __init__(self, tensors, timbre_cls=False):
        self.t = tensors
        self.cls = timbre_cls
        self.lyric = stack_from_gguf_tensors(tensors, "encoder.lyric_encoder.")
        self.timbre = stack_from_gguf_tensors(tensors, "encoder.timbre_encoder.")

    def forward(self, text, lyric, timbre=None, window=128):
        t = self.t
        h = _linear(t["encoder.lyric_encoder.embed_tokens.weight"], lyric,
                    t["encoder.lyric_encoder.embed_tokens.bias"])
        _, lyr = self.lyric.run_layers(h, 0, self.lyric.cfg["n_layers"], causal=False, final_norm=True,
                                       window=window)
        parts = [lyr]
        if timbre is not None and len(timbre) > 0:
            th = _linear(t["encoder.timbre_encoder.embed_tokens.weight"], timbre,
                         t["encoder.timbre_encoder.embed_tokens.bias"])
            if self.cls:
                th = np.concatenate([_f32_of(t["encoder.timbre_encoder.special_token"]).reshape(1, -1), th])
            _, tim = self.timbre.run_layers(th, 0, self.timbre.cfg["n_layers"], causal=False, final_norm=True,
                                            window=window)
            parts.append(tim[:1])
        parts.append(_linear(t["encoder.text_projector.weight"], text))
        return np.concatenate(parts).astype(np.float32)


class OracleDetok:
    """detok_ggml_decode (src/fsq-detok.h:128-212), all groups as one batch of 5-row sequences."""

    def __init__(self, tensors):
        self.t = tensors
        self.stack = stack_from_gguf_tensors(tensors, "detokenizer.")

    def decode(self, codes):
        t = self.t
        G = len(codes)
        x = np.stack([fsq_decode_index(c) for c in codes])
        q = _linear(t["tokenizer.quantizer.project_out.weight"], x, t["tokenizer.quantizer.project_out.bias"])
        e = _linear(t["detokenizer.embed_tokens.weight"], q, t["detokenizer.embed_tokens.bias"])
        sp = _f32_of(t["detokenizer.special_tokens"])
        h = (e[:, None, :] + sp[None, :, :]).reshape(G * 5, -1).astype(np.float32)
        _, y = self.stack.run_layers(h, 0, self.stack.cfg["n_layers"], causal=False, final_norm=True, batch=G)
        return _linear(t["detokenizer.proj_out.weight"], y, t["detokenizer.proj_out.bias"])


class OracleTok:
    """tok_ggml_encode (src/fsq-tok.h:133-238) on latents already padded to 5 * G frames; returns
    (codes [G], pre-activation values [G][6])."""

    def __init__(self, tensors):
        self.t = tensors
        self.stack = stack_from_gguf_tensors(tensors, "tokenizer.attention_pooler.")

    def encode(self, latents):
        t = self.t
        G = latents.shape[0] // 5
        p = _linear(t["tokenizer.audio_acoustic_proj.weight"], latents, t["tokenizer.audio_acoustic_proj.bias"])
        e = _linear(t["tokenizer.attention_pooler.embed_tokens.weight"], p,
                    t["tokenizer.attention_pooler.embed_tokens.bias"])
        cls = _f32_of(t["tokenizer.attention_pooler.special_token"]).reshape(1, 1, -1)
        H = e.shape[1]
        h = np.concatenate([np.broadcast_to(cls, (G, 1, H)), e.reshape(G, 5, H)], axis=1).reshape(G * 6, H)
        _, y = self.stack.run_layers(np.ascontiguousarray(h, dtype=np.float32), 0, self.stack.cfg["n_layers"],
                                     causal=False, final_norm=True, batch=G)
        raw = _linear(t["tokenizer.quantizer.project_in.weight"], y[0::6], t["tokenizer.quantizer.project_in.bias"])
        return np.array([fsq_encode_index(r) for r in raw], dtype=np.int32), raw


def sample_top_k_p(logits, temperature, top_p, top_k, u) -> int:
    """sample_top_k_p (src/sampling.h:30-133) on a copy of one logits row; u the canonical uniform."""
    x = np.array(logits, dtype=np.float32, copy=True)
    return int(lib().orc_sample_top_k_p(_p(x), x.size, temperature, top_p, top_k, u))


def lm_compact_cfg(lc, lu, cfg_scale, eos_idx, code_offset, n_codes):
    """The phase-2 targeted CFG and compaction (src/pipeline-lm.cpp:474-490): [EOS, codes...] of
    lu + cfg * (lc - lu) (every step one f32 rounding), or of lc alone when lu is None."""
    cols = np.concatenate([[eos_idx], code_offset + np.arange(n_codes)])
    c = np.asarray(lc, dtype=np.float32)[cols]
    if lu is None:
        return c
    u = np.asarray(lu, dtype=np.float32)[cols]
    return (u + np.float32(cfg_scale) * (c - u)).astype(np.float32)


class Stork4:
    """solver_stork4_step (src/solvers/solver-stork.h:270-315) in float32 with every product and sum
    rounded in the reference's order (d2v in float64), over the caller's ROCK4 tables
    {ms, fpa [len][6], fpb [len][4], recf}."""

    def __init__(self, tables, substeps=10):
        self.ms = [int(v) for v in tables["ms"]]
        self.fpa = np.asarray(tables["fpa"], np.float64).reshape(-1, 6)
        self.fpb = np.asarray(tables["fpb"], np.float64).reshape(-1, 4)
        self.recf = np.asarray(tables["recf"], np.float64)
        self.substeps = substeps
        self.step_index = 0
        self.hist = []  # (vt, dt), newest last, at most 3

    def _push(self, vt, dt):
        self.hist.append((np.array(vt, np.float32, copy=True), np.float32(dt)))
        self.hist = self.hist[-3:]

    def _derivs(self, vt):
        """_stork_compute_derivatives (solver-stork.h:72-127): (order, dv, d2v)."""
        f = np.float32
        if not self.hist:
            return 0, None, None
        v1, h1 = self.hist[-1]
        if h1 == 0:
            return 0, None, None
        dv = ((v1 - vt) / h1).astype(np.float32)
        n = vt.size
        vt_rms = np.sqrt(np.sum(vt.astype(np.float64) ** 2) / n)
        dv_rms = np.sqrt(np.sum(dv.astype(np.float64) ** 2) / n)
        if vt_rms > 0 and dv_rms * abs(float(h1)) > 5.0 * vt_rms:
            return 0, dv, None
        if len(self.hist) < 2:
            return 1, dv, None
        v2, h2 = self.hist[-2]
        if h2 == 0:
            return 1, dv, None
        h1d, h2d = float(h1), float(h2)
        denom = h1d * h2d * (h1d + h2d)
        if abs(denom) < 1e-30:
            return 1, dv, None
        coeff = 2.0 / denom
        d2v = (coeff * ((v2.astype(np.float64) * h1d - v1.astype(np.float64) * (h1d + h2d))
                        + vt.astype(np.float64) * h2d)).astype(np.float32)
        d2v_rms = np.sqrt(np.sum(d2v.astype(np.float64) ** 2) / n)
        if vt_rms > 0 and d2v_rms * float(h1) * float(h1) > 5.0 * vt_rms:
            return 1, dv, d2v
        return 2, dv, d2v

    @staticmethod
    def _taylor(order, diff, v, dv, d2v):
        f = np.float32
        if order >= 1 and dv is not None:
            if order >= 2 and d2v is not None:
                half = f(f(f(0.5) * diff) * diff)
                return ((v + diff * dv) + half * d2v).astype(np.float32)
            return (v + diff * dv).astype(np.float32)
        return v.copy()

    def _mdegr(self, s):
        mp1 = 1
        for i, m in enumerate(self.ms):
            if m >= s:
                return m, i, mp1 - 1
            mp1 += m * 2 - 1
        return self.ms[-1], len(self.ms) - 1, mp1 - 1

    def _substep(self, xt, vt, s, t_curr, t_prev, order, dv, d2v):
        """_rock4_substep (solver-stork.h:160-268): (x_next, finite)."""
        with np.errstate(over="ignore", invalid="ignore"):
            return self._substep_body(xt, vt, s, t_curr, t_prev, order, dv, d2v)

    def _substep_body(self, xt, vt, s, t_curr, t_prev, order, dv, d2v):
        f = np.float32
        s = min(s, self.ms[-1])
        mdeg, mz, mr = self._mdegr(s)
        t_curr, t_prev = f(t_curr), f(t_prev)
        dt = f(t_curr - t_prev)
        R = self.recf
        t1 = f(-dt * f(R[mr]))
        ci1 = f(t_curr + t1)
        ci2, ci3 = ci1, t_curr
        y1 = (xt + t1 * vt).astype(np.float32)
        y2 = xt.copy()
        for j in range(2, mdeg + 1):
            diff = f(ci1 - t_curr)
            vel = self._taylor(order, diff, vt, dv, d2v)
            temp1 = f(-dt * f(R[mr + 2 * (j - 2) + 1]))
            temp3 = f(-f(R[mr + 2 * (j - 2) + 2]))
            temp2 = f(f(1.0) - temp3)
            cn = f(f(temp1 + f(temp2 * ci2)) + f(temp3 * ci3))
            y = ((temp1 * vel + temp2 * y1) + temp3 * y2).astype(np.float32)
            y2, y1 = y1, y
            ci3, ci2, ci1 = ci2, cn, cn
        A, B = self.fpa[mz], self.fpb[mz]
        fa = [f(-dt * f(a)) for a in A]
        fb = [f(-dt * f(b)) for b in B]
        F1 = self._taylor(order, f(ci1 - t_curr), vt, dv, d2v)
        F2 = self._taylor(order, f(f(ci1 + fa[0]) - t_curr), vt, dv, d2v)
        F3 = self._taylor(order, f(f(f(ci1 + fa[1]) + fa[2]) - t_curr), vt, dv, d2v)
        F4 = self._taylor(order, f(f(f(f(ci1 + fa[3]) + fa[4]) + fa[5]) - t_curr), vt, dv, d2v)
        out = ((((y1 + fb[0] * F1) + fb[1] * F2) + fb[2] * F3) + fb[3] * F4).astype(np.float32)
        return out, bool(np.all(np.isfinite(out)))

    def step(self, xt, vt, t_curr, t_prev):
        f = np.float32
        xt = np.asarray(xt, np.float32)
        vt = np.asarray(vt, np.float32)
        dt = f(f(t_curr) - f(t_prev))
        if self.step_index == 0:
            out = (xt - vt * dt).astype(np.float32)
            self._push(vt, dt)
            self.step_index = 1
            return out
        order, dv, d2v = self._derivs(vt)
        s = max(self.substeps, 2)
        out = None
        while s >= 2:
            nxt, ok = self._substep(xt, vt, s, t_curr, t_prev, order, dv, d2v)
            if ok:
                out = nxt
                break
            s //= 2
        if out is None:
            out = (xt - vt * dt).astype(np.float32)
        self._push(vt, dt)
        self.step_index += 1
        return out


# ---- LoRA merge (src/adapter-merge.h:482-672) --------------------------------------------------

def lora_scaling(alpha, rank, scale) -> np.float32:
    """(alpha / rank) * scale in f32, as adapter_merge_lora computes it."""
    f = np.float32
    return f(f(f(alpha) / f(rank)) * f(scale))


def lora_merge(entry, A, B, scaling):
    """One tensor of adapter_merge_lora: entry (qtype, raw, K, shape) -> (qtype, merged raw [N][row
    bytes or K], merged f32 [N][K]). A [rank][K], B [N][rank] are rounded to bf16 (PEFT); the delta
    B.A is formed from those exact products in double, rounded to f32, scaled, rounded to bf16 and
    added to the dequantised base; the sum is requantised to the base type."""
    qt, raw, K, shape = entry
    N = int(np.prod(shape)) // K
    base = _f32_of(entry).reshape(N, K)
    a = round_bf16(np.asarray(A, np.float32)).astype(np.float64)
    b = round_bf16(np.asarray(B, np.float32)).astype(np.float64)
    d = (b @ a).astype(np.float32)
    d = round_bf16((d * np.float32(scaling)).astype(np.float32))
    merged = (base + d).astype(np.float32)
    if qt == F32:
        out = merged
    elif qt == BF16:
        out = f32_to_bf16_bits(merged)
    elif qt == F16:
        out = merged.astype(np.float16).view(np.uint16)
    else:
        out = quantize(merged, qt)
    return qt, out, merged


def lokr_factors(w1, alpha, rank, w2=None, w2a=None, w2b=None):
    """adapter_merge_lokr's two Kronecker factors (src/adapter-merge.h:674-958): w1s = w1 * (alpha /
    rank) in f32, and W2 = w2 (monolithic) or w2_a . w2_b (factorised) with the exact products of
    the f32 factors summed in float64 in ascending rank and rounded to f32 once."""
    f = np.float32
    scaling = f(f(alpha) / f(rank))
    w1s = (np.asarray(w1, np.float32) * scaling).astype(np.float32)
    if w2 is not None:
        W2 = np.asarray(w2, np.float32)
    else:
        a, b = np.asarray(w2a, np.float32), np.asarray(w2b, np.float32)
        acc = np.zeros((a.shape[0], b.shape[1]), np.float64)
        for q in range(a.shape[1]):
            acc += a[:, q:q + 1].astype(np.float64) * b[q:q + 1, :].astype(np.float64)
        W2 = acc.astype(np.float32)
    return w1s, W2


def lokr_merge(entry, w1s, W2, user_scale, dora_scale=None):
    """One tensor of adapter_merge_lokr + adapter_merge_on_backend (:357-472): delta = kron(w1s, W2)
    (f32 products) rounded to bf16; without DoRA base + delta * user_scale; with a DoRA magnitude
    vector m = base + delta, each row scaled by ds / (|m| + 2^-7), mixed with 1 by user_scale when
    it is not 1 (|m| from the f32 squares summed in float64, rounded once, f32 sqrt). Returns
    (qtype, merged raw, merged f32) like lora_merge."""
    f = np.float32
    qt, raw, K, shape = entry
    N = int(np.prod(shape)) // K
    base = _f32_of(entry).reshape(N, K)
    delta = round_bf16(np.kron(w1s.astype(np.float32), W2.astype(np.float32)).astype(np.float32))
    assert delta.shape == (N, K)
    if dora_scale is None:
        merged = (base + (delta * f(user_scale)).astype(np.float32)).astype(np.float32)
    else:
        m = (base + delta).astype(np.float32)
        ss = (m * m).astype(np.float32).astype(np.float64).sum(axis=1).astype(np.float32)
        rn = (np.sqrt(ss).astype(np.float32) + f(0.0078125)).astype(np.float32)
        sc = (np.asarray(dora_scale, np.float32).reshape(N) / rn).astype(np.float32)
        if f(user_scale) != f(1.0):
            sc = ((sc * f(user_scale)).astype(np.float32) + f(f(1.0) - f(user_scale))).astype(np.float32)
        merged = (m * sc[:, None]).astype(np.float32)
    if qt == F32:
        out = merged
    elif qt == BF16:
        out = f32_to_bf16_bits(merged)
    elif qt == F16:
        out = merged.astype(np.float16).view(np.uint16)
    else:
        out = quantize(merged, qt)
    return qt, out, merged


# ---- VAE decoder (src/vae.h) ----------------------------------------------------------------------

class OracleVAE:
    """vae_ggml_load + vae_ggml_build_graph (src/vae.h:167-369) in numpy over the GGUF's bf16 bits
    {name: uint16 array in PyTorch shape}: weight norm fused in f32 with a sequential sum of squares
    (vae_fuse_wn, :64-93) and rounded to f16; snake in f32 (five separately rounded ops); every conv
    as an im2col of f16-cast activations times the f16 weights, exact products summed in float64
    and rounded to f32 (ggml_conv_1d's operand types; the sum order of ggml is not reproduced);
    ConvTranspose as that GEMM plus the overlap-add in ascending kernel tap, then the bias."""

    def __init__(self, bits: dict):
        f = lambda n: bf16_bits_to_f32(bits[n]).reshape(bits[n].shape)
        self.f = f
        self.c1 = self._conv(f, "decoder.conv1", bias=True)
        self.blocks = []
        i = 0
        while f"decoder.block.{i}.conv_t1.weight_v" in bits:
            p = f"decoder.block.{i}"
            g, v = f(f"{p}.conv_t1.weight_g"), f(f"{p}.conv_t1.weight_v")  # v [IC, OC, K]
            w = self._wn(g.reshape(-1), v).astype(np.float16)
            ru = []
            for r in range(1, 4):
                rp = f"{p}.res_unit{r}"
                ru.append(dict(s1=self._snake(f, f"{rp}.snake1"), c1=self._conv(f, f"{rp}.conv1", True),
                               s2=self._snake(f, f"{rp}.snake2"), c2=self._conv(f, f"{rp}.conv2", True),
                               dil=(1, 3, 9)[r - 1]))
            self.blocks.append(dict(sn=self._snake(f, f"{p}.snake1"), ct=w, ctb=f(f"{p}.conv_t1.bias").reshape(-1),
                                    stride=v.shape[2] // 2, ru=ru))
            i += 1
        self.sn = self._snake(f, "decoder.snake1")
        self.c2 = self._conv(f, "decoder.conv2", bias=False)
        self.up = int(np.prod([b["stride"] for b in self.blocks]))

    @staticmethod
    def _wn(g, v):
        d0 = v.shape[0]
        vv = v.reshape(d0, -1).astype(np.float32)
        sq = (vv * vv).astype(np.float32)
        nsq = np.add.accumulate(sq, axis=1, dtype=np.float32)[:, -1]  # sequential f32 sum
        s = (g.astype(np.float32) / (np.sqrt(nsq).astype(np.float32) + np.float32(1e-12))).astype(np.float32)
        return (vv * s[:, None]).astype(np.float32).reshape(v.shape)

    def _conv(self, f, pfx, bias):
        v = f(f"{pfx}.weight_v")  # [OC, IC, K]
        w = self._wn(f(f"{pfx}.weight_g").reshape(-1), v).astype(np.float16)
        return dict(w=w, b=f(f"{pfx}.bias").reshape(-1) if bias else None)

    @staticmethod
    def _snake(f, pfx):
        a = f(f"{pfx}.alpha").reshape(-1)
        b = f(f"{pfx}.beta").reshape(-1)
        return np.exp(a).astype(np.float32), (np.float32(1.0) / np.exp(b).astype(np.float32)).astype(np.float32)

    @staticmethod
    def snake(x, sn):
        ea, ib = sn
        ax = (x * ea).astype(np.float32)
        s = np.sin(ax).astype(np.float32)
        return (x + ((s * s).astype(np.float32) * ib).astype(np.float32)).astype(np.float32)

    @staticmethod
    def conv(x, c, dil=1, pad=None, res=None):
        """x [T][IC] f32 -> [T][OC]: f16 im2col, exact f16 products summed in float64."""
        w = c["w"]  # [OC, IC, K] f16
        OC, IC, K = w.shape
        pad = (K // 2) * dil if pad is None else pad
        T = x.shape[0]
        xh = x.astype(np.float16).astype(np.float64)
        xp = np.zeros((T + 2 * pad, IC))
        xp[pad:pad + T] = xh
        y = np.zeros((T, OC))
        wf = w.astype(np.float64)
        for k in range(K):
            y += xp[k * dil:k * dil + T] @ wf[:, :, k].T
        y = y.astype(np.float32)
        if c["b"] is not None:
            y = (y + c["b"]).astype(np.float32)
        if res is not None:
            y = (res + y).astype(np.float32)
        return y

    def decode(self, latent):
        """latent [T][64] -> audio [2][T * up]."""
        x = self.conv(np.asarray(latent, np.float32), self.c1)
        for b in self.blocks:
            h = self.snake(x, b["sn"]).astype(np.float16).astype(np.float64)
            w = b["ct"].astype(np.float64)  # [IC, OC, K]
            IC, OC, K = w.shape
            s = b["stride"]
            col = np.tensordot(h, w, axes=([1], [0])).astype(np.float32)  # [T][OC][K]
            T = x.shape[0]
            pad = (K - s) // 2
            full = np.zeros(((T - 1) * s + K, OC), np.float32)
            for k in range(K):  # overlap-add in ascending tap: input t lands on t*s + k
                full[k:k + (T - 1) * s + 1:s] += col[:, :, k]
            y = full[pad:pad + (T - 1) * s + K - 2 * pad]
            x = (y + b["ctb"]).astype(np.float32)
            for r in b["ru"]:
                h1 = self.conv(self.snake(x, r["s1"]), r["c1"], dil=r["dil"])
                x = self.conv(self.snake(h1, r["s2"]), r["c2"], res=x)
        y = self.conv(self.snake(x, self.sn), self.c2)  # [T][2]
        return np.ascontiguousarray(y.T)

    def decode_tiled(self, latent, chunk_size=256, overlap=64):
        """vae_ggml_decode_tiled (src/vae.h:467-565) over decode()."""
        T = latent.shape[0]
        while chunk_size - 2 * overlap <= 0 and overlap > 0:
            overlap //= 2
        if T <= chunk_size:
            return self.decode(latent)
        stride = chunk_size - 2 * overlap
        outs, upf = [], None
        for i in range((T + stride - 1) // stride):
            c0, c1 = i * stride, min(i * stride + stride, T)
            w0, w1 = max(c0 - overlap, 0), min(c1 + overlap, T)
            a = self.decode(latent[w0:w1])
            if upf is None:
                upf = np.float32(a.shape[1]) / np.float32(w1 - w0)
            t0 = int(np.round(np.float32(c0 - w0) * upf))
            t1 = int(np.round(np.float32(w1 - c1) * upf))
            outs.append(a[:, t0:(a.shape[1] - t1 if t1 > 0 else a.shape[1])])
        return np.concatenate(outs, axis=1)
