"""GPU: prefill / DiT attention (acb_attn_prefill) against a plain PyTorch fp32 softmax attention on
the same bf16 Q/K/V, and against the oracle's ggml-CPU attention. The kernel rounds the
probabilities to bf16 for the P.V product and uses exp2, so the bar is the bf16 tier:
cosine >= 0.9999 and max_rel <= 1e-2 per output."""
import math

import numpy as np
import pytest

import acb
import oracle as O
from helpers import cos_sim, max_rel

pytestmark = pytest.mark.gpu


def torch_ref(q, k, v, Nh, Nkv, mask, window, causal_off):
    import torch
    B, Sq, _ = q.shape
    Skv = k.shape[1]
    G = Nh // Nkv
    qf = q.float().view(B, Sq, Nh, 128).permute(0, 2, 1, 3)
    kf = k.float().view(B, Skv, Nkv, 128).permute(0, 2, 1, 3).repeat_interleave(G, dim=1)
    vf = v.float().view(B, Skv, Nkv, 128).permute(0, 2, 1, 3).repeat_interleave(G, dim=1)
    s = (qf @ kf.transpose(-1, -2)) / math.sqrt(128)
    i = torch.arange(Sq, device=q.device)[:, None]
    j = torch.arange(Skv, device=q.device)[None, :]
    if mask == acb.MASK_CAUSAL:
        s = s.masked_fill(~(j <= i + causal_off), float("-inf"))
    elif mask == acb.MASK_WINDOW:
        s = s.masked_fill(~((i - j).abs() <= window), float("-inf"))
    p = torch.softmax(s, dim=-1)
    return (p @ vf).permute(0, 2, 1, 3).reshape(B, Sq, Nh * 128)


@pytest.mark.parametrize("B,Sq,Skv,Nh,Nkv,mask,window", [
    (1, 256, 256, 16, 8, acb.MASK_CAUSAL, 0),       # text encoder (config 1)
    (8, 750, 750, 16, 8, acb.MASK_WINDOW, 128),     # DiT self-attention, even layers
    (8, 750, 750, 16, 8, acb.MASK_NONE, 0),         # DiT self-attention, odd layers
    (8, 750, 512, 16, 8, acb.MASK_NONE, 0),         # DiT cross-attention
    (2, 77, 33, 4, 2, acb.MASK_NONE, 0),            # ragged tails
    (1, 100, 300, 16, 8, acb.MASK_CAUSAL, 200),     # prefill continuing a cache (causal offset)
])
def test_attn_prefill_matches_fp32(cuda, B, Sq, Skv, Nh, Nkv, mask, window):
    import torch
    g = torch.Generator(device=cuda).manual_seed(Sq + Skv + mask)
    q = (torch.randn(B, Sq, Nh * 128, device=cuda, generator=g) * 1.5).bfloat16()
    k = (torch.randn(B, Skv, Nkv * 128, device=cuda, generator=g) * 1.5).bfloat16()
    v = torch.randn(B, Skv, Nkv * 128, device=cuda, generator=g).bfloat16()
    causal_off = 200 if (mask == acb.MASK_CAUSAL and Skv > Sq) else 0
    o = acb.attn_prefill(q, k, v, Nh, Nkv, mask=mask, window=window, causal_off=causal_off, out_dtype=torch.float32)
    ref = torch_ref(q, k, v, Nh, Nkv, mask, window, causal_off)
    got, want = o.cpu().numpy(), ref.cpu().numpy()
    for b in range(B):
        c, r = cos_sim(got[b], want[b]), max_rel(got[b], want[b])
        assert c >= 0.9999 and r <= 1e-2, (b, c, r)


def test_attn_prefill_views_of_fused_qkv_and_oracle(cuda):
    """Q, K, V as column views of one fused bf16 QKV row (the GEMM output layout), compared with
    the oracle's ggml-CPU attention (f32 path of qwen3_attn_f32, causal mask)."""
    import torch
    Nh, Nkv, S = 16, 8, 200
    qkvd = (Nh + 2 * Nkv) * 128
    g = torch.Generator(device=cuda).manual_seed(9)
    qkv = torch.randn(1, S, qkvd, device=cuda, generator=g).bfloat16()
    q, k, v = qkv[:, :, :Nh * 128], qkv[:, :, Nh * 128:(Nh + Nkv) * 128], qkv[:, :, (Nh + Nkv) * 128:]
    o = acb.attn_prefill(q, k, v, Nh, Nkv, mask=acb.MASK_CAUSAL, out_dtype=torch.float32)
    qn = q.float().cpu().numpy().reshape(S, Nh, 128)
    kn = k.float().cpu().numpy().reshape(S, Nkv, 128)
    vn = v.float().cpu().numpy().reshape(S, Nkv, 128)
    mask = np.where(np.arange(S)[None, :] <= np.arange(S)[:, None], 0.0, -np.inf).astype(np.float32)
    ref = O.attention(qn, kn, vn, O.F32, mask, 1.0 / math.sqrt(128)).reshape(S, Nh * 128)
    got = o[0].cpu().numpy()
    assert cos_sim(got, ref) >= 0.9999 and max_rel(got, ref) <= 1e-2


@pytest.mark.parametrize("B,Sq,Skv,Nh,Nkv,mask,window", [
    (1, 256, 256, 16, 8, acb.MASK_CAUSAL, 0),
    (8, 750, 750, 16, 8, acb.MASK_WINDOW, 128),
    (8, 750, 512, 16, 8, acb.MASK_NONE, 0),
    (2, 77, 33, 4, 2, acb.MASK_NONE, 0),
])
def test_attn_prefill_f16_operands(cuda, B, Sq, Skv, Nh, Nkv, mask, window):
    """ACB_FLAG_F16: f16 Q/K/V and f16 probabilities (11-bit significands): bar cosine >= 0.99999
    and max_rel <= 2e-3 against the fp32 softmax attention of the same operands."""
    import torch
    g = torch.Generator(device=cuda).manual_seed(Sq * 3 + Skv + mask)
    q = (torch.randn(B, Sq, Nh * 128, device=cuda, generator=g) * 1.5).half()
    k = (torch.randn(B, Skv, Nkv * 128, device=cuda, generator=g) * 1.5).half()
    v = torch.randn(B, Skv, Nkv * 128, device=cuda, generator=g).half()
    o = acb.attn_prefill(q, k, v, Nh, Nkv, mask=mask, window=window, out_dtype=torch.float32)
    ref = torch_ref(q, k, v, Nh, Nkv, mask, window, 0)
    got, want = o.cpu().numpy(), ref.cpu().numpy()
    for b in range(B):
        c, r = cos_sim(got[b], want[b]), max_rel(got[b], want[b])
        assert c >= 0.99999 and r <= 2e-3, (b, c, r)
    oh = acb.attn_prefill(q, k, v, Nh, Nkv, mask=mask, window=window, out_dtype=torch.float16)
    assert max_rel(oh.float().cpu().numpy(), got) <= 2.0 ** -10


@pytest.mark.parametrize("B,Sq,Skv,Nh,Nkv,mask,window", [
    (1, 256, 256, 16, 8, acb.MASK_CAUSAL, 0),
    (8, 750, 750, 16, 8, acb.MASK_WINDOW, 128),
    (4, 750, 512, 16, 8, acb.MASK_NONE, 0),
    (2, 77, 33, 4, 2, acb.MASK_NONE, 0),
])
def test_attn_prefill_split_is_fp32_accurate(cuda, B, Sq, Skv, Nh, Nkv, mask, window):
    """acb_attn_prefill_split on hi/lo planes of f32 Q/K/V: fp32 softmax attention of the f32
    operands to max_rel <= 1e-5 (the f32 reference CPU attention, qwen3_attn_f32; fp32
    accumulation order and exp2 give ~3e-6)."""
    import torch
    g = torch.Generator(device=cuda).manual_seed(Sq * 5 + Skv + mask)
    q = torch.randn(B, Sq, Nh * 128, device=cuda, generator=g) * 1.5
    k = torch.randn(B, Skv, Nkv * 128, device=cuda, generator=g) * 1.5
    v = torch.randn(B, Skv, Nkv * 128, device=cuda, generator=g)

    def planes(t):
        flat = t.reshape(-1, t.shape[-1])
        pl = acb.act_quant_ex(flat, flat.shape[1], acb.F16, acb.LAYOUT_PLANES)
        n = flat.shape[0]
        return pl[:n].view(t.shape), n * flat.shape[1]

    qh, ql = planes(q)
    kh, kl = planes(k)
    vh, vl = planes(v)
    o = acb.attn_prefill_split(qh, kh, vh, ql, kl, vl, Nh, Nkv, mask=mask, window=window)
    torch.backends.cuda.matmul.allow_tf32 = False
    ref = torch_ref(q.double(), k.double(), v.double(), Nh, Nkv, mask, window, 0)
    got, want = o.double().cpu().numpy(), ref.cpu().numpy()
    for b in range(B):
        assert max_rel(got[b], want[b]) <= 1e-5, (b, max_rel(got[b], want[b]))


TC_CASES = [
    (1, 256, 256, 16, 8, acb.MASK_CAUSAL, 0, 0),
    (8, 750, 750, 16, 8, acb.MASK_WINDOW, 128, 0),
    (8, 750, 750, 16, 8, acb.MASK_NONE, 0, 0),
    (8, 750, 512, 16, 8, acb.MASK_NONE, 0, 0),
    (2, 77, 33, 4, 2, acb.MASK_NONE, 0, 0),
    (1, 100, 300, 16, 8, acb.MASK_CAUSAL, 0, 200),
]


@pytest.mark.parametrize("B,Sq,Skv,Nh,Nkv,mask,window,causal_off", TC_CASES)
def test_attn_tc_matches_reference(cuda, B, Sq, Skv, Nh, Nkv, mask, window, causal_off):
    """acb_attn_tc (tcgen05): f16 operands against the fp32 attention of the same f16 values
    (cosine >= 0.99999, max_rel <= 2e-3); hi/lo split operands against float64 attention of the
    f32 values (max_rel <= 1e-5) and against the mma.sync split kernel."""
    import torch
    g = torch.Generator(device=cuda).manual_seed(Sq * 7 + Skv + mask)
    q = torch.randn(B, Sq, Nh * 128, device=cuda, generator=g) * 1.5
    k = torch.randn(B, Skv, Nkv * 128, device=cuda, generator=g) * 1.5
    v = torch.randn(B, Skv, Nkv * 128, device=cuda, generator=g)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    # f16 operands
    qh, kh, vh = q.half(), k.half(), v.half()
    vt, ld, _ = acb.attn_vt(vh, Nkv)
    o = acb.attn_tc(qh.view(B * Sq, -1), kh.view(B * Skv, -1), vt, ld, Nh, Nkv, Sq, Skv, B, mask=mask, window=window,
                    causal_off=causal_off, err=err)
    ref = torch_ref(qh, kh, vh, Nh, Nkv, mask, window, causal_off).reshape(B * Sq, -1)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    got, want = o.view(B, Sq, -1).cpu().numpy(), ref.view(B, Sq, -1).cpu().numpy()
    for b in range(B):
        c, r = cos_sim(got[b], want[b]), max_rel(got[b], want[b])
        assert c >= 0.99999 and r <= 2e-3, ("f16", b, c, r)
    # hi/lo split operands
    def planes(t):
        flat = t.reshape(-1, t.shape[-1])
        pl = acb.act_quant_ex(flat, flat.shape[1], acb.F16, acb.LAYOUT_PLANES)
        return pl, flat.numel()
    qp, qlo = planes(q)
    kp, klo = planes(k)
    vts, ld, vlo = acb.attn_vt(v, Nkv, lo=True)
    o2 = acb.attn_tc(qp[: B * Sq], kp[: B * Skv], vts, ld, Nh, Nkv, Sq, Skv, B, mask=mask, window=window,
                     causal_off=causal_off, q_lo=qlo, k_lo=klo, vt_lo=vlo, err=err)
    torch.backends.cuda.matmul.allow_tf32 = False
    ref2 = torch_ref(q.double(), k.double(), v.double(), Nh, Nkv, mask, window, causal_off)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    got2, want2 = o2.view(B, Sq, -1).double().cpu().numpy(), ref2.cpu().numpy()
    for b in range(B):
        assert max_rel(got2[b], want2[b]) <= 1e-5, ("split", b, max_rel(got2[b], want2[b]))
    if causal_off == 0:
        hq = qp[: B * Sq].view(B, Sq, -1)
        hk = kp[: B * Skv].view(B, Skv, -1)
        vp, _ = planes(v)
        hv = vp[: B * Skv].view(B, Skv, -1)
        o3 = acb.attn_prefill_split(hq, hk, hv, qlo, klo, v.numel(), Nh, Nkv, mask=mask, window=window)
        assert max_rel(o2.view(B, Sq, -1).cpu().numpy(), o3.cpu().numpy()) <= 1e-5


@pytest.mark.parametrize("split,gemm_a,quant", [(True, True, O.Q8_0), (False, False, O.Q8_0), (True, True, O.F16),
                                                (False, False, O.BF16)])
def test_attn_tc_quantised_output(cuda, split, gemm_a, quant):
    """acb_attn_tc writing the output projection's operand (o_type Q8_0 / F16 / BF16, optionally the
    exact [hi|hi|lo] layout) == the f32 output followed by acb_act_quant_ex, bit for bit."""
    import torch
    B, Sq, Skv, Nh, Nkv = 2, 300, 200, 4, 2
    g = torch.Generator(device=cuda).manual_seed(77 + split)
    q = torch.randn(B * Sq, Nh * 128, device=cuda, generator=g)
    k = torch.randn(B * Skv, Nkv * 128, device=cuda, generator=g)
    v = torch.randn(B, Skv, Nkv * 128, device=cuda, generator=g)
    if split:
        qp = acb.act_quant_ex(q, Nh * 128, acb.F16, acb.LAYOUT_PLANES)
        kp = acb.act_quant_ex(k, Nkv * 128, acb.F16, acb.LAYOUT_PLANES)
        vt, ld, vlo = acb.attn_vt(v, Nkv, lo=True)
        lo = dict(q_lo=q.numel(), k_lo=k.numel(), vt_lo=vlo)
        qq, kk = qp[: B * Sq], kp[: B * Skv]
    else:
        vt, ld, _ = acb.attn_vt(v.half(), Nkv)
        lo = {}
        qq, kk = q.half(), k.half()
    o32 = acb.attn_tc(qq, kk, vt, ld, Nh, Nkv, Sq, Skv, B, **lo)
    got = acb.attn_tc(qq, kk, vt, ld, Nh, Nkv, Sq, Skv, B, quant=quant, gemm_a=gemm_a, **lo)
    layout = acb.LAYOUT_GEMM_A if gemm_a else acb.LAYOUT_PLAIN
    want = acb.act_quant_ex(o32, Nh * 128, quant, layout)
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
