"""GPU: the activation operand of the tensor-core linears (acb_act_quant, acb_act_quant_swiglu)
against the oracle's ggml activation quantisers. The kernel writes fp16(d*q) for each element
of each Q8_0 / Q8_K block: the oracle's quantise -> dequantise values rounded to f16 must match
bit for bit (integer and scale arithmetic identical, one rounding at the end)."""
import numpy as np
import pytest

import acb
import oracle as O
from helpers import assert_bitexact

pytestmark = pytest.mark.gpu


def ref_fq(x, vt):
    """Oracle: ggml from_float for vec_type vt, dequantised to f32, then rounded to the operand type."""
    if vt == O.Q8_0:
        return O.dequantize(O.quantize(x, O.Q8_0), O.Q8_0, x.shape[1]).astype(np.float16)
    if vt == O.Q8_K:
        raw = O.quantize(x, O.Q8_K).reshape(x.shape[0], -1, 292)
        d = raw[:, :, 0:4].copy().view(np.float32)             # [rows, blocks, 1]
        q = raw[:, :, 4:260].view(np.int8).astype(np.float32)  # [rows, blocks, 256]
        return (d * q).astype(np.float32).reshape(x.shape).astype(np.float16)
    if vt == O.F16:
        return x.astype(np.float16)
    return O.bf16_bits_to_f32(O.f32_to_bf16_bits(x))


@pytest.mark.parametrize("vt", [O.Q8_0, O.Q8_K, O.F16, O.BF16])
@pytest.mark.parametrize("M,K", [(1, 256), (77, 1024), (256, 3072), (33, 6144)])
def test_act_quant_matches_oracle(cuda, vt, M, K):
    import torch
    rng = np.random.default_rng(M * K + vt)
    x = (rng.standard_normal((M, K)) * rng.uniform(0.1, 30, (M, 1))).astype(np.float32)
    x[0, :64] = 0.0  # an all-zero Q8_0 block (d = 0)
    if K == 256:
        x[-1, :] = 0.0  # an all-zero Q8_K block
    y = acb.act_quant(torch.from_numpy(x).to(cuda), vt)
    want = ref_fq(x, vt)
    got = y.cpu()
    got = got.float().numpy() if vt == O.BF16 else got.numpy()
    assert_bitexact(got, want, f"act_quant vt={vt}")


@pytest.mark.parametrize("vt", [O.Q8_0, O.Q8_K])
def test_act_quant_swiglu_matches_oracle(cuda, vt):
    import torch
    rng = np.random.default_rng(vt)
    M, F = 65, 3072
    gu = (rng.standard_normal((M, 2 * F)) * 2).astype(np.float32)
    y = acb.act_quant_swiglu(torch.from_numpy(gu).to(cuda), F, vt)
    h = O.swiglu(gu[:, :F], gu[:, F:])
    assert_bitexact(y.cpu().numpy(), ref_fq(h, vt), "act_quant_swiglu")


def test_vec_dot_types():
    assert acb.vec_dot_type(acb.Q8_0) == acb.Q8_0
    assert acb.vec_dot_type(acb.Q4_K) == acb.Q8_K and acb.vec_dot_type(acb.Q6_K) == acb.Q8_K
    assert acb.vec_dot_type(acb.F16) == acb.F16 and acb.vec_dot_type(acb.BF16) == acb.BF16
    assert acb.vec_dot_type(acb.F32) == acb.F32 and acb.vec_dot_type(acb.Q8_K) == -1


def _split(v):
    hi = v.astype(np.float16)
    lo = (v - hi.astype(np.float32)).astype(np.float16)
    return hi, lo


@pytest.mark.parametrize("layout", [acb.LAYOUT_GEMM_A, acb.LAYOUT_GEMM_B, acb.LAYOUT_PLANES])
@pytest.mark.parametrize("vt", [O.Q8_0, O.Q8_K, O.F16])
def test_act_quant_exact_layouts(cuda, layout, vt):
    """Exact layouts: hi = f16(v), lo = f16(v - hi) of the same operand values, and hi + lo == v
    exactly for the dequantised activations (<= 18 significant bits)."""
    import torch
    rng = np.random.default_rng(layout * 31 + vt)
    M, K = 19, 512
    x = (rng.standard_normal((M, K)) * 3).astype(np.float32)
    y = acb.act_quant_ex(torch.from_numpy(x).to(cuda), K, vt, layout).cpu().numpy()
    if vt == O.Q8_0:  # the dequantised operand values, unrounded
        v = O.dequantize(O.quantize(x, O.Q8_0), O.Q8_0, K)
    elif vt == O.Q8_K:
        raw = O.quantize(x, O.Q8_K).reshape(M, -1, 292)
        d = raw[:, :, 0:4].copy().view(np.float32)
        q = raw[:, :, 4:260].view(np.int8).astype(np.float32)
        v = (d * q).astype(np.float32).reshape(M, K)
    else:
        v = x
    hi, lo = _split(v)
    if layout == acb.LAYOUT_GEMM_A:
        want = np.concatenate([hi, hi, lo], axis=1)
    elif layout == acb.LAYOUT_GEMM_B:
        want = np.concatenate([hi, lo, hi], axis=1)
    else:
        want = np.concatenate([hi, lo], axis=0)
    assert_bitexact(y, want, f"layout {layout}")
    if vt == O.Q8_0:  # f16 scale times a 7-bit integer: the split is exact
        assert np.array_equal(hi.astype(np.float32) + lo.astype(np.float32), v)


@pytest.mark.parametrize("vt", [O.Q8_0, O.Q8_K, O.F16, O.BF16])
@pytest.mark.parametrize("layout", [acb.LAYOUT_PLAIN, acb.LAYOUT_GEMM_A, acb.LAYOUT_PLANES])
@pytest.mark.parametrize("K", [1024, 2048, 2560])
def test_norm_quant_matches_unfused(cuda, vt, layout, K):
    """acb_norm_quant (RMSNorm x w [+ adaLN] fused into the activation quantiser) is bit-identical
    to acb_rms_norm / acb_adaln_modulate with f32 output followed by acb_act_quant_ex."""
    import torch
    if vt == O.BF16 and layout != acb.LAYOUT_PLAIN:
        pytest.skip("the split layouts are f16")
    rng = np.random.default_rng(K + vt * 7 + layout)
    S, T = 3, 37
    M = S * T
    x = torch.from_numpy((rng.standard_normal((M, K)) * rng.uniform(0.1, 30, (M, 1))).astype(np.float32)).to(cuda)
    w = torch.from_numpy((1 + 0.1 * rng.standard_normal(K)).astype(np.float32)).to(cuda)
    sc = torch.from_numpy((0.2 * rng.standard_normal((S, K))).astype(np.float32)).to(cuda)
    sh = torch.from_numpy((0.2 * rng.standard_normal((S, K))).astype(np.float32)).to(cuda)
    # RMSNorm x w
    got = acb.norm_quant(x, K, w, 1e-6, vt, layout)
    want = acb.act_quant_ex(acb.rms_norm(x, w, 1e-6), K, vt, layout)
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    # adaLN: per-sample scale / shift
    got = acb.norm_quant(x, K, w, 1e-6, vt, layout, scale=sc, shift=sh, rows_per_sample=T, vec_stride=K)
    xm = acb.adaln_modulate(x.view(S, T, K), w, 1e-6, sc, sh).reshape(M, K)
    want = acb.act_quant_ex(xm, K, vt, layout)
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))


@pytest.mark.parametrize("rope", [False, True])
def test_qk_norm_rope_planes_matches_unfused(cuda, rope):
    """acb_qk_norm_rope_planes (q heads and k heads with their own weights, one launch) ==
    acb_qk_norm_rope (f32) per head group followed by acb_act_quant_ex PLANES, bit for bit."""
    import torch
    rng = np.random.default_rng(5 + rope)
    T, Nq, Nk, D = 300, 3, 2, 128
    src = torch.from_numpy(rng.standard_normal((T, (Nq + Nk) * D + 64)).astype(np.float32) * 3).to(cuda)
    wq = torch.from_numpy((1 + 0.1 * rng.standard_normal(D)).astype(np.float32)).to(cuda)
    wk = torch.from_numpy((1 + 0.1 * rng.standard_normal(D)).astype(np.float32)).to(cuda)
    pos = torch.from_numpy(rng.integers(0, 512, T).astype(np.int32)).to(cuda) if rope else None
    tab = acb.rope_table(512, D, 1e6).to(cuda) if rope else None
    got = acb.qk_norm_rope_planes(src, Nq, wq, 1e-6, pos=pos, rope=tab, n_k_heads=Nk, k_w=wk)
    rq = acb.qk_norm_rope(src, Nq, D, wq, 1e-6, pos, tab, out_dtype=torch.float32).reshape(T, Nq * D)
    rk = acb.qk_norm_rope(src[:, Nq * D:], Nk, D, wk, 1e-6, pos, tab, out_dtype=torch.float32).reshape(T, Nk * D)
    ref32 = torch.cat([rq, rk], dim=1).contiguous()
    want = acb.act_quant_ex(ref32, (Nq + Nk) * D, O.F16, acb.LAYOUT_PLANES)
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    # q heads only (the cross-attention form)
    got = acb.qk_norm_rope_planes(src, Nq, wq, 1e-6)
    want = acb.act_quant_ex(acb.qk_norm_rope(src, Nq, D, wq, 1e-6, None, None, out_dtype=torch.float32)
                            .reshape(T, Nq * D).contiguous(), Nq * D, O.F16, acb.LAYOUT_PLANES)
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
