"""GPU: the tcgen05 tensor-core GEMM (acb_gemm_bf16) against a plain PyTorch fp32 reference of
the same op on the same bf16 operands. Only the fp32 accumulation order differs, so the bar is
max_rel <= 1e-5 (relative to max |C|) for f32 output and one bf16 rounding step for bf16 output.
Shapes cover single tiles, ragged M/N tails, the DiT layer shapes at 8 x 750 tokens and K=6144."""
import numpy as np
import pytest

import acb
import oracle as O
from helpers import max_rel

pytestmark = pytest.mark.gpu


def ref_mm(A, B):
    """fp32 reference (TF32 off) of the same bf16 operands."""
    import torch
    torch.backends.cuda.matmul.allow_tf32 = False
    return A.float() @ B.float().T


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 128), (77, 300, 128), (129, 257, 192),
                                   (6000, 4096, 2048), (6000, 2048, 6144), (1, 256, 64)])
def test_gemm_plain(cuda, M, N, K):
    import torch
    g = torch.Generator(device=cuda).manual_seed(M * 7 + N + K)
    A = torch.randn(M, K, device=cuda, generator=g).bfloat16()
    B = (torch.randn(N, K, device=cuda, generator=g) * 0.05).bfloat16()
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    C = acb.gemm_bf16(A, B, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref = ref_mm(A, B)
    r = max_rel(C.cpu().numpy(), ref.cpu().numpy())
    assert r <= 1e-5, r


def test_gemm_epilogues(cuda):
    import torch
    g = torch.Generator(device=cuda).manual_seed(3)
    S, T, K, N = 4, 250, 512, 768
    M = S * T
    A = torch.randn(M, K, device=cuda, generator=g).bfloat16()
    B = (torch.randn(N, K, device=cuda, generator=g) * 0.05).bfloat16()
    bias = torch.randn(N, device=cuda, generator=g)
    res = torch.randn(M, N, device=cuda, generator=g)
    gate = torch.randn(S, N, device=cuda, generator=g)
    base = ref_mm(A, B)
    # bias only, f32
    C = acb.gemm_bf16(A, B, bias=bias)
    assert max_rel(C.cpu().numpy(), (base + bias).cpu().numpy()) <= 1e-5
    # residual add (in place on an f32 buffer aliasing res)
    out = res.clone()
    acb.gemm_bf16(A, B, out=out, res=out)
    assert max_rel((out - res).cpu().numpy(), base.cpu().numpy()) <= 1e-5
    # DiT gated residual: res + (acc + bias) * gate[sample]
    out = res.clone()
    acb.gemm_bf16(A, B, out=out, bias=bias, res=out, gate=gate, rows_per_sample=T)
    want = res + (base + bias) * gate.repeat_interleave(T, dim=0)
    assert max_rel((out - res).cpu().numpy(), (want - res).cpu().numpy()) <= 1e-5
    # bf16 output
    Cb = acb.gemm_bf16(A, B, out_dtype=torch.bfloat16)
    d = (Cb.float() - base).abs()
    assert (d <= base.abs() * 2.0 ** -8 + 1e-6).all()


@pytest.mark.parametrize("M,N,K", [(256, 4096, 1024), (77, 300, 128), (6000, 2048, 6144)])
def test_gemm_f16_operands(cuda, M, N, K):
    """ACB_FLAG_F16: the same GEMM on f16 operands (the reference-faithful dense path), f32 and
    f16 output."""
    import torch
    g = torch.Generator(device=cuda).manual_seed(M + N + K)
    A = torch.randn(M, K, device=cuda, generator=g).half()
    B = (torch.randn(N, K, device=cuda, generator=g) * 0.05).half()
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    C = acb.gemm_bf16(A, B, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref = ref_mm(A, B)
    assert max_rel(C.cpu().numpy(), ref.cpu().numpy()) <= 1e-5
    Ch = acb.gemm_bf16(A, B, out_dtype=torch.float16)
    d = (Ch.float() - ref).abs()
    assert (d <= ref.abs() * 2.0 ** -10 + 2e-5 * ref.abs().max()).all()


@pytest.mark.parametrize("M,N,K", [(256, 1024, 3072), (256, 1024, 2048), (77, 1024, 2048), (256, 4096, 1024),
                                   (256, 6144, 1024), (1, 2048, 6144)])
def test_gemm_split_k(cuda, M, N, K):
    """Small-M shapes split K over CTAs (acb_gemm_tc with a workspace): same bars as the unsplit
    GEMM, every epilogue, and bit-identical results on repeat (partials summed in split order)."""
    import torch
    ws_bytes = acb.gemm_workspace_bytes(M, N, K)
    assert ws_bytes > 0, "these shapes are meant to split"
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=cuda)
    g = torch.Generator(device=cuda).manual_seed(M + N * 3 + K)
    A = torch.randn(M, K, device=cuda, generator=g).half()
    B = (torch.randn(N, K, device=cuda, generator=g) * 0.05).half()
    bias = torch.randn(N, device=cuda, generator=g)
    res = torch.randn(M, N, device=cuda, generator=g)
    gate = torch.randn(2, N, device=cuda, generator=g)
    base = ref_mm(A, B)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    C1 = acb.gemm_bf16(A, B, workspace=ws, err=err)
    C2 = acb.gemm_bf16(A, B, workspace=ws)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert max_rel(C1.cpu().numpy(), base.cpu().numpy()) <= 1e-5
    assert torch.equal(C1, C2)
    out = res.clone()
    rps = max(1, (M + 1) // 2)
    acb.gemm_bf16(A, B, out=out, bias=bias, res=out, gate=gate, rows_per_sample=rps, workspace=ws)
    want = res + (base + bias) * gate.repeat_interleave(rps, dim=0)[:M]
    assert max_rel((out - res).cpu().numpy(), (want - res).cpu().numpy()) <= 1e-5
    Ch = acb.gemm_bf16(A, B, out_dtype=torch.float16, workspace=ws)
    d = (Ch.float() - base).abs()
    assert (d <= base.abs() * 2.0 ** -10 + 2e-5 * base.abs().max()).all()


def test_gemm_split_k_shared_workspace(cuda):
    """Split GEMMs of different shapes take turns on one workspace (as a model's linears do): the
    tile counters keep their place whatever the partials of the other shapes cover, so every call
    still matches its own result on a fresh workspace, bit for bit."""
    import torch
    shapes = [(77, 1024, 2048), (256, 6144, 1024), (1, 2048, 6144), (256, 1024, 3072)]
    need = max(acb.gemm_workspace_bytes(*s) for s in shapes)
    ws = torch.zeros(need, dtype=torch.uint8, device=cuda)
    g = torch.Generator(device=cuda).manual_seed(7)
    ops = [(torch.randn(M, K, device=cuda, generator=g).half(),
            (torch.randn(N, K, device=cuda, generator=g) * 0.05).half()) for M, N, K in shapes]
    want = []
    for (A, B), s in zip(ops, shapes):
        own = torch.zeros(acb.gemm_workspace_bytes(*s), dtype=torch.uint8, device=cuda)
        want.append(acb.gemm_bf16(A, B, workspace=own))
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    for rep in range(3):
        for i in (list(range(len(shapes))) if rep % 2 == 0 else reversed(range(len(shapes)))):
            A, B = ops[i]
            got = acb.gemm_bf16(A, B, workspace=ws, err=err)
            assert torch.equal(got, want[i]), (rep, shapes[i])
    torch.cuda.synchronize()
    assert int(err.item()) == 0


@pytest.mark.parametrize("M,N,K", [(256, 1024, 3072), (300, 512, 1024)])
def test_gemm_exact_split_products(cuda, M, N, K):
    """GEMM over K' = 3K with A' = [hi|hi|lo] and B' = [hi|lo|hi] (acb_act_quant_ex layouts): the
    product of dequantised Q8_0 activations and weights to fp32 accuracy (max_rel <= 2e-6
    against float64)."""
    import torch
    rng = np.random.default_rng(M + N + K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    W = O.quantize((rng.standard_normal((N, K)) * 0.02).astype(np.float32), O.Q8_0)
    wd = O.dequantize(W, O.Q8_0, K)
    xd = O.dequantize(O.quantize(x, O.Q8_0), O.Q8_0, K)
    A = acb.act_quant_ex(torch.from_numpy(x).to(cuda), K, O.Q8_0, acb.LAYOUT_GEMM_A)
    B = acb.act_quant_ex(torch.from_numpy(wd).to(cuda), K, O.F16, acb.LAYOUT_GEMM_B)
    ws = torch.zeros(max(1, acb.gemm_workspace_bytes(M, N, 3 * K)), dtype=torch.uint8, device=cuda)
    C = acb.gemm_bf16(A, B, workspace=ws).double().cpu().numpy()
    ref = xd.astype(np.float64) @ wd.astype(np.float64).T
    assert max_rel(C, ref) <= 2e-6, max_rel(C, ref)


@pytest.mark.parametrize("f16", [False, True])
def test_gemm_cta_pairs(cuda, f16):
    """Unsplit GEMMs with M > 128 run on CTA pairs (256 x 256 tiles over two SMs). Ragged M and N
    leave the second CTA of the last pair tiles partly (rows 2432..2499) or wholly out of range,
    and 80 tiles over the resident pairs make some pairs reuse both TMEM accumulators. Every
    epilogue, against the fp32 reference; repeat runs are bit-identical."""
    import torch
    assert acb.gemm_pair_clusters(f16) > 0, "the CTA-pair kernel should be available on B200"
    dt = torch.float16 if f16 else torch.bfloat16
    g = torch.Generator(device=cuda).manual_seed(11 + f16)
    S, T, K, N = 4, 625, 1024, 2000
    M = S * T
    A = torch.randn(M, K, device=cuda, generator=g).to(dt)
    B = (torch.randn(N, K, device=cuda, generator=g) * 0.05).to(dt)
    bias = torch.randn(N, device=cuda, generator=g)
    res = torch.randn(M, N, device=cuda, generator=g)
    gate = torch.randn(S, N, device=cuda, generator=g)
    base = ref_mm(A, B)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    C1 = acb.gemm_bf16(A, B, err=err)
    C2 = acb.gemm_bf16(A, B, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert max_rel(C1.cpu().numpy(), base.cpu().numpy()) <= 1e-5
    assert torch.equal(C1, C2)
    out = res.clone()
    acb.gemm_bf16(A, B, out=out, bias=bias, res=out, gate=gate, rows_per_sample=T)
    want = res + (base + bias) * gate.repeat_interleave(T, dim=0)
    assert max_rel((out - res).cpu().numpy(), (want - res).cpu().numpy()) <= 1e-5
    Cb = acb.gemm_bf16(A, B, out_dtype=dt)
    d = (Cb.float() - base).abs()
    ulp = 2.0 ** -10 if f16 else 2.0 ** -8
    assert (d <= base.abs() * ulp + 2e-5 * base.abs().max()).all()


@pytest.mark.parametrize("M,F,K,f16,vt,layout,bias", [
    (2500, 1024, 1024, True, O.Q8_0, acb.LAYOUT_GEMM_A, False),
    (6000, 3072, 2048, True, O.Q8_0, acb.LAYOUT_PLAIN, False),
    (300, 1024, 512, False, O.Q8_0, acb.LAYOUT_GEMM_A, True),
    (1000, 1024, 1024, True, O.F16, acb.LAYOUT_PLAIN, True),
    (1000, 1024, 1024, False, O.BF16, acb.LAYOUT_PLAIN, False)])
def test_gemm_swiglu_quant_matches_unfused(cuda, M, F, K, f16, vt, layout, bias):
    """acb_gemm_swiglu_quant (SwiGLU and the down projection's quantisation in the gate/up GEMM's
    epilogue) == acb_gemm_tc (f32 out, same bias) + acb_act_quant_ex(up_offset = F), bit for bit."""
    import torch
    dt = torch.float16 if f16 else torch.bfloat16
    g = torch.Generator(device=cuda).manual_seed(M + F + K)
    A = torch.randn(M, K, device=cuda, generator=g).to(dt)
    B = (torch.randn(2 * F, K, device=cuda, generator=g) * 0.05).to(dt)
    bv = torch.randn(2 * F, device=cuda, generator=g) if bias else None
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    got = acb.gemm_swiglu_quant(A, B, F, vt, layout, bias=bv, err=err)
    gu = acb.gemm_bf16(A, B, bias=bv)
    want = acb.act_quant_ex(gu, F, vt, layout, up_offset=F)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))


@pytest.mark.parametrize("lo,rope", [(True, True), (False, True), (True, False)])
def test_gemm_qkv_planes_matches_unfused(cuda, lo, rope):
    """acb_gemm_qkv_planes (q/k RMSNorm + RoPE into attention operand planes and V^T planes in the
    qkv GEMM's epilogue) == acb_gemm_tc (f32) + acb_qk_norm_rope_planes + acb_attn_vt, bit for bit.
    300 tokens per sequence put sequence boundaries inside 32-row epilogue groups."""
    import torch
    Bs, S, nq, nk, K = 3, 300, 4, 2, 512
    M = Bs * S
    g = torch.Generator(device=cuda).manual_seed(31 + lo + 2 * rope)
    A = torch.randn(M, K, device=cuda, generator=g).half()
    B = (torch.randn((nq + 2 * nk) * 128, K, device=cuda, generator=g) * 0.05).half()
    qw = 1 + 0.1 * torch.randn(128, device=cuda, generator=g)
    kw = 1 + 0.1 * torch.randn(128, device=cuda, generator=g)
    pos = torch.arange(S, dtype=torch.int32, device=cuda).repeat(Bs) if rope else None
    tab = acb.rope_table(512, 128, 1e6).to(cuda) if rope else None
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    qk, vt, ld, vlo = acb.gemm_qkv_planes(A, B, nq, nk, qw, kw, 1e-6, S, pos=pos, rope=tab, lo=lo, err=err)
    C = acb.gemm_bf16(A, B)
    W = (nq + nk) * 128
    want_qk = acb.qk_norm_rope_planes(C, nq, qw, 1e-6, pos=pos, rope=tab, n_k_heads=nk, k_w=kw)
    want_vt, ld2, vlo2 = acb.attn_vt(C[:, W:].reshape(Bs, S, nk * 128), nk, lo=lo)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    if lo:
        assert torch.equal(qk.view(torch.int16), want_qk.view(torch.int16))
    else:
        assert torch.equal(qk.view(torch.int16), want_qk[:M].view(torch.int16))
    assert ld == ld2 and vlo == vlo2
    assert torch.equal(vt.view(torch.int16), want_vt.view(torch.int16))
