"""GPU parity of the op-chain kernels (through the C ABI) against the CPU oracle.

Bars: get_rows, rms_norm, q/k-norm+RoPE, adaLN modulate and the gated residual are compared
bit-for-bit (the oracle and the kernels perform the same separately rounded float operations,
with the norm's sum of squares in double); SwiGLU uses CUDA's expf, so it is held to a
relative error of 1e-6 (f32 I/O) or one bf16 rounding step (bf16 I/O). Shapes include the
BASELINE config-2 shapes and ragged / unaligned cases.
"""
import numpy as np
import pytest

import acb
import oracle as O
from helpers import assert_bitexact, assert_nearly_exact, max_rel

pytestmark = pytest.mark.gpu


def T(a, dev, dtype=None):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return t if dtype is None else t.to(dtype)


def to_np32(t):
    import torch
    return t.float().cpu().numpy() if t.dtype != torch.float32 else t.cpu().numpy()


def io_cast(x, io):
    """Input as seen by the kernel: bf16 rounds the f32 values first."""
    return O.round_bf16(x) if io == "bf16" else x


def torch_dtype(io):
    import torch
    return {"f32": torch.float32, "bf16": torch.bfloat16}[io]


def round_out(y, io):
    return O.round_bf16(y) if io == "bf16" else y


# ---------------------------------------------------------------------------------------------

@pytest.mark.parametrize("io", ["f32", "bf16"])
@pytest.mark.parametrize("rows,cols", [(8192, 2048), (256, 1024), (3, 2560), (5, 100), (1, 128)])
def test_rms_norm(cuda, io, rows, cols):
    rng = np.random.default_rng(rows * 7 + cols)
    x = io_cast(rng.standard_normal((rows, cols)).astype(np.float32), io)
    w = (1 + 0.01 * rng.standard_normal(cols)).astype(np.float32)
    y = acb.rms_norm(T(x, cuda, torch_dtype(io)), T(w, cuda), 1e-6)
    ref = round_out(O.rms_norm(x, w, 1e-6), io)
    assert_nearly_exact(to_np32(y), ref, 1e-6, 0.9999, f"rms_norm {io} {rows}x{cols}")


@pytest.mark.parametrize("io", ["f32", "bf16"])
def test_qk_norm_rope_microbench_shape(cuda, io):
    """config 2b: [B=4, T=1024, H=16, D=128], positions 0..T-1 per batch, theta 1e6."""
    import torch
    B, Tn, Hh, D = 4, 1024, 16, 128
    rng = np.random.default_rng(11)
    x = io_cast(rng.standard_normal((B * Tn, Hh, D)).astype(np.float32), io)
    w = (1 + 0.01 * rng.standard_normal(D)).astype(np.float32)
    pos = np.tile(np.arange(Tn, dtype=np.int32), B)
    table = acb.rope_table(Tn, D, 1e6)
    y = acb.qk_norm_rope(T(x.reshape(B * Tn, Hh * D), cuda, torch_dtype(io)), Hh, D, T(w, cuda), 1e-6,
                         T(pos, cuda), table.to(cuda))
    rope_rows = O.rope_cache(pos, D, 1e6)
    ref = round_out(O.qk_norm_rope(x, w, 1e-6, rope_rows), io)
    assert_bitexact(to_np32(y).reshape(ref.shape), ref, f"qk_norm_rope {io}")


def test_qk_norm_rope_from_fused_qkv_into_f16_cache(cuda):
    """LM decode pattern: k heads read from the fused QKV row, written (f16) into a KV cache
    [n_sets][Nkv][max_seq][D] at per-sequence positions; v copied without norm/rope."""
    import torch
    Nh, Nkv, D, max_seq, N = 16, 8, 128, 512, 4
    qkvd = (Nh + 2 * Nkv) * D
    rng = np.random.default_rng(5)
    qkv = rng.standard_normal((N, qkvd)).astype(np.float32)
    w = (1 + 0.01 * rng.standard_normal(D)).astype(np.float32)
    pos = np.array([0, 17, 255, 511], dtype=np.int32)
    table = acb.rope_table(max_seq, D, 1e6).to(cuda)
    cache_k = torch.zeros((N, Nkv, max_seq, D), dtype=torch.float16, device=cuda)
    cache_v = torch.zeros_like(cache_k)
    src = T(qkv, cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    dpos = T(pos, cuda)
    # k: columns [Nh*D, Nh*D + Nkv*D) of each fused row
    acb.qk_norm_rope(src[:, Nh * D:], Nkv, D, T(w, cuda), 1e-6, dpos, table, out=cache_k,
                     src_tok_stride=qkvd, dst_tok_stride=Nkv * max_seq * D, dst_head_stride=max_seq * D,
                     dst_pos_stride=D, n_tok=N, err=err)
    acb.qk_norm_rope(src[:, (Nh + Nkv) * D:], Nkv, D, None, 1e-6, dpos, None, out=cache_v,
                     src_tok_stride=qkvd, dst_tok_stride=Nkv * max_seq * D, dst_head_stride=max_seq * D,
                     dst_pos_stride=D, n_tok=N, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    kref = O.qk_norm_rope(qkv[:, Nh * D:(Nh + Nkv) * D].reshape(N, Nkv, D), w, 1e-6, O.rope_cache(pos, D, 1e6))
    vref = qkv[:, (Nh + Nkv) * D:].reshape(N, Nkv, D)
    ck, cv = cache_k.cpu().numpy(), cache_v.cpu().numpy()
    for i in range(N):
        assert np.array_equal(ck[i, :, pos[i], :].view(np.uint16), kref[i].astype(np.float16).view(np.uint16))
        assert np.array_equal(cv[i, :, pos[i], :].view(np.uint16), vref[i].astype(np.float16).view(np.uint16))
    # nothing else written
    mask = np.ones((N, max_seq), bool)
    mask[np.arange(N), pos] = False
    assert not ck.transpose(0, 2, 1, 3)[mask].any() and not cv.transpose(0, 2, 1, 3)[mask].any()


def test_qk_norm_rope_position_out_of_range_sets_flag(cuda):
    import torch
    D = 128
    x = torch.randn(3, 2 * D, device=cuda)
    table = acb.rope_table(16, D, 1e6).to(cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    pos = torch.tensor([0, 16, 3], dtype=torch.int32, device=cuda)  # 16 is out of range
    acb.qk_norm_rope(x, 2, D, None, 1e-6, pos, table, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) & 2


@pytest.mark.parametrize("io", ["f32", "bf16"])
@pytest.mark.parametrize("rows,F", [(8192, 6144), (7, 3072), (3, 100)])
def test_swiglu(cuda, io, rows, F):
    rng = np.random.default_rng(rows + F)
    gu = io_cast(rng.standard_normal((rows, 2 * F)).astype(np.float32) * 3, io)
    y = acb.swiglu(T(gu, cuda, torch_dtype(io)), F)
    ref = O.swiglu(gu[:, :F], gu[:, F:])
    if io == "f32":
        assert max_rel(to_np32(y), ref) < 1e-6
        assert np.abs(to_np32(y) - ref).max() <= 4e-7 * np.abs(ref).max() + 1e-30
    else:
        got = to_np32(y)
        refb = O.round_bf16(ref)
        # at most one bf16 step apart, and almost always identical
        step = np.abs(refb) * 2.0 ** -7 + 1e-30
        assert (np.abs(got - refb) <= step).all()
        assert np.mean(got == refb) > 0.999


@pytest.mark.parametrize("io", ["f32", "bf16"])
@pytest.mark.parametrize("per_sample", [True, False])
@pytest.mark.parametrize("with_norm", [False, True])
def test_adaln_modulate(cuda, io, per_sample, with_norm):
    """config 2d: x [8, 750, 2048], per-sample shift/scale [8, 2048] (or shared [2048])."""
    S, Tn, H = 8, 750, 2048
    rng = np.random.default_rng(21)
    x = io_cast(rng.standard_normal((S, Tn, H)).astype(np.float32), io)
    shp = (S, H) if per_sample else (H,)
    scale = (0.1 * rng.standard_normal(shp)).astype(np.float32)
    shift = (0.1 * rng.standard_normal(shp)).astype(np.float32)
    w = (1 + 0.01 * rng.standard_normal(H)).astype(np.float32) if with_norm else None
    y = acb.adaln_modulate(T(x, cuda, torch_dtype(io)), None if w is None else T(w, cuda), 1e-6, T(scale, cuda),
                           T(shift, cuda))
    ref = round_out(O.adaln(x, w, 1e-6, scale, shift), io)
    assert_bitexact(to_np32(y), ref, "adaln")


@pytest.mark.parametrize("io", ["f32", "bf16"])
@pytest.mark.parametrize("shape", [(8, 750, 2048), (2, 3, 100)])
def test_gated_residual(cuda, io, shape):
    S, Tn, H = shape
    rng = np.random.default_rng(31)
    r = io_cast(rng.standard_normal(shape).astype(np.float32), io)
    o = io_cast(rng.standard_normal(shape).astype(np.float32), io)
    gate = rng.standard_normal((S, H)).astype(np.float32)
    y = acb.gated_residual(T(r, cuda, torch_dtype(io)), T(o, cuda, torch_dtype(io)), T(gate, cuda))
    ref = round_out(O.gated_residual(r, o, gate), io)
    assert_bitexact(to_np32(y), ref, "gated")


@pytest.mark.parametrize("qt", [O.Q8_0, O.Q4_K, O.Q6_K, O.BF16, O.F16, O.F32])
@pytest.mark.parametrize("out", ["f32", "bf16"])
def test_get_rows_types(cuda, qt, out):
    import torch
    rng = np.random.default_rng(qt)
    n_rows, cols = 1000, 2560
    tab = (rng.standard_normal((n_rows, cols)) * 0.02).astype(np.float32)
    raw = O.quantize(tab, qt)
    ids = rng.integers(0, n_rows, size=300).astype(np.int32)
    ids[:3] = [0, n_rows - 1, 5]
    y = acb.get_rows(T(raw, cuda), qt, n_rows, cols, T(ids, cuda), out_dtype=torch_dtype(out))
    rc, ref = O.get_rows(qt, raw, cols, ids)
    assert rc == 0
    assert_bitexact(to_np32(y), round_out(ref, out), f"get_rows {qt}")


def test_get_rows_microbench_shape(cuda):
    """config 2e: 8192 random ids into a [217472 x 2048] Q8_0 table (473 MB)."""
    import torch
    V, H, n = 217472, 2048, 8192
    g = torch.Generator(device=cuda).manual_seed(7)
    # random Q8_0 rows made on the device: random int8 quants and modest positive f16 scales
    raw = torch.randint(0, 256, (V, 2176), dtype=torch.uint8, device=cuda, generator=g)
    d = (torch.rand((V, 64), device=cuda, generator=g) * 1e-3 + 1e-5).to(torch.float16)
    raw.view(V, 64, 34)[:, :, 0:2] = d.view(torch.uint8).view(V, 64, 2)
    ids = torch.randint(0, V, (n,), dtype=torch.int32, device=cuda, generator=g)
    for out_dt in (torch.float32, torch.bfloat16):
        y = acb.get_rows(raw, O.Q8_0, V, H, ids, out_dtype=out_dt)
        ids_np = ids.cpu().numpy()
        rows = raw[ids.long()].cpu().numpy()
        ref = O.dequantize(rows, O.Q8_0, H)
        assert_bitexact(to_np32(y), ref if out_dt == torch.float32 else O.round_bf16(ref), "get_rows micro")
        assert ids_np.shape == (n,)


def test_get_rows_bad_id_sets_flag_and_zeroes_row(cuda):
    import torch
    rng = np.random.default_rng(9)
    tab = rng.standard_normal((10, 64)).astype(np.float32)
    raw = O.quantize(tab, O.Q8_0)
    ids = np.array([1, 10, -1, 2], dtype=np.int32)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    y = acb.get_rows(T(raw, cuda), O.Q8_0, 10, 64, T(ids, cuda), err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 1
    yn = y.cpu().numpy()
    assert not yn[1].any() and not yn[2].any()
    _, ref = O.get_rows(O.Q8_0, raw, 64, np.array([1, 2], np.int32))
    assert_bitexact(yn[[0, 3]], ref, "good rows")
