"""GPU parity of the decode path (configs 3 and 5) through the C ABI against the oracle.

GEMV: every block contributes (float)isum * (d_w*d_x) exactly as in the oracle (activation
quantised in-kernel to Q8_0 / Q8_K with the ggml rules, integer dot products), and the terms of
a row are added in double and rounded once, on the GPU and in the oracle: the outputs are
bit-identical. Attention reproduces the f16 rounding of q and of the probabilities, sums its
dot products and P.V terms in double and uses the library's exponential (acb_exp.h) on both
sides: bit-identical too. (A double sum can differ in its last bit between two orders when its
terms span more than ~20 binades; the float result then differs only if that bit decides a
rounding to float, about one element in 10^8.) The LM must give the same greedy tokens as the
oracle's greedy loop, and the same logits.
"""
import numpy as np
import pytest

import acb
import oracle as O
from helpers import assert_bitexact, cos_sim, max_rel
from lm_fixtures import TINY, make_tensors, oracle_greedy, oracle_model, policy_all, policy_q4_k_m, write_gguf

pytestmark = pytest.mark.gpu


def T(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def TW(raw, dev):
    """Weight rows on the device with 256 readable bytes after the last row (acb_gemv reads
    whole 16-byte units)."""
    import torch
    flat = np.ascontiguousarray(raw).reshape(-1)
    buf = torch.zeros(flat.size + 256, dtype=torch.uint8, device=dev)
    buf[:flat.size] = torch.from_numpy(flat).to(dev)
    return buf


@pytest.mark.parametrize("qt", [O.Q8_0, O.Q4_K, O.Q6_K])
@pytest.mark.parametrize("M", [1, 3, 8])
@pytest.mark.parametrize("N,K", [(77, 256), (1000, 2048), (333, 2560), (2048, 6144)])
def test_gemv_plain(cuda, qt, M, N, K):
    rng = np.random.default_rng(N + K + M + qt)
    W = O.quantize((rng.standard_normal((N, K)) * 0.02).astype(np.float32), qt)
    x = rng.standard_normal((M, K)).astype(np.float32)
    y = acb.gemv(TW(W, cuda), qt, N, K, T(x, cuda), M=M)
    ref = O.mul_mat(qt, W, N, K, x)
    assert_bitexact(y.cpu().numpy(), ref, "gemv")


@pytest.mark.parametrize("qt", [O.Q8_0, O.Q4_K, O.Q6_K])
def test_gemv_rmsnorm_prologue_and_residual(cuda, qt):
    rng = np.random.default_rng(qt)
    M, N, K = 4, 512, 2048
    W = O.quantize((rng.standard_normal((N, K)) * 0.02).astype(np.float32), qt)
    h = rng.standard_normal((M, K)).astype(np.float32) * 3
    w = (1 + 0.01 * rng.standard_normal(K)).astype(np.float32)
    res = rng.standard_normal((M, N)).astype(np.float32)
    y = acb.gemv(TW(W, cuda), qt, N, K, T(h, cuda), M=M, prologue=acb.PRO_RMSNORM, norm_w=T(w, cuda),
                 epilogue=acb.EPI_ADD, res=T(res, cuda), flags=acb.FLAG_PDL)
    ref = (res + O.mul_mat(qt, W, N, K, O.rms_norm(h, w, 1e-6))).astype(np.float32)
    assert_bitexact(y.cpu().numpy(), ref, "gemv rmsnorm + residual")


def test_gemv_swiglu_and_split_prologues(cuda):
    rng = np.random.default_rng(7)
    M, N, K = 2, 256, 3072
    W = O.quantize((rng.standard_normal((N, K)) * 0.02).astype(np.float32), O.Q8_0)
    gu = rng.standard_normal((M, 2 * K)).astype(np.float32)
    y = acb.gemv(TW(W, cuda), O.Q8_0, N, K, T(gu, cuda), M=M, prologue=acb.PRO_SWIGLU, x_stride=2 * K)
    ref = O.mul_mat(O.Q8_0, W, N, K, O.swiglu(gu[:, :K], gu[:, K:]))
    # the SiLU of both sides uses the library's exponential: identical activations
    assert_bitexact(y.cpu().numpy(), ref, "gemv swiglu")
    ns = 5
    parts = rng.standard_normal((M, ns, K))  # double partials (acb_attn_decode's)
    y = acb.gemv(TW(W, cuda), O.Q8_0, N, K, T(parts, cuda), M=M, prologue=acb.PRO_SUM_SPLITS, x_stride=ns * K,
                 n_split=ns)
    x = parts.sum(axis=1).astype(np.float32)
    assert_bitexact(y.cpu().numpy(), O.mul_mat(O.Q8_0, W, N, K, x), "gemv split sum")


@pytest.mark.parametrize("qt", [O.Q8_0, O.Q4_K, O.Q6_K])
def test_device_quantize_matches_oracle_encoders(cuda, qt):
    import torch
    rng = np.random.default_rng(11)
    x = (rng.standard_normal((64, 2560 if qt != O.Q8_0 else 2048)) * 0.02).astype(np.float32)
    x[3, :256] = 0.0
    K = x.shape[1]
    rb = acb.lib().acb_row_bytes(qt, K)
    out = torch.empty((64, rb), dtype=torch.uint8, device=cuda)
    acb._check("q", acb.lib().acb_quantize(T(x, cuda).data_ptr(), 64, K, qt, out.data_ptr(), acb._stream(None)))
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), O.quantize(x, qt))


@pytest.mark.parametrize("n_tok,set_per_tok", [(1, 1), (4, 1), (37, 0)])
def test_qkv_post_and_attention(cuda, n_tok, set_per_tok):
    import torch
    Nh, Nkv, D, max_seq, n_sets = 16, 8, 128, 1024, 4
    rng = np.random.default_rng(n_tok)
    qkvd = (Nh + 2 * Nkv) * D
    # a cache already holding random history
    kc = (rng.standard_normal((n_sets, Nkv, max_seq, D)) * 0.5).astype(np.float16)
    vc = rng.standard_normal((n_sets, Nkv, max_seq, D)).astype(np.float16)
    if set_per_tok:
        pos = rng.integers(0, max_seq, size=n_tok).astype(np.int32)
        pos[0] = 0
    else:
        pos = (300 + np.arange(n_tok)).astype(np.int32)
    qkv = rng.standard_normal((n_tok, qkvd)).astype(np.float32)
    qn = (1 + 0.01 * rng.standard_normal(D)).astype(np.float32)
    kn = (1 + 0.01 * rng.standard_normal(D)).astype(np.float32)
    rope = acb.rope_table(max_seq, D, 1e6)
    d_kc, d_vc = T(kc.view(np.uint16), cuda), T(vc.view(np.uint16), cuda)
    q_out = torch.empty((n_tok, Nh * D), dtype=torch.float32, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    d_pos = T(pos, cuda)
    acb.qkv_post(T(qkv, cuda), n_tok, Nh, Nkv, D, T(qn, cuda), T(kn, cuda), 1e-6, d_pos, rope.to(cuda), q_out, d_kc,
                 d_vc, max_seq, 0, set_per_tok, flags=acb.FLAG_PDL, err=err)
    ns = acb.attn_decode_splits(n_tok, Nkv)
    scores = torch.empty((n_tok, Nh, max_seq), dtype=torch.float32, device=cuda)
    smax = torch.empty((n_tok, Nh, ns), dtype=torch.float32, device=cuda)
    part = torch.empty((n_tok, ns, Nh * D), dtype=torch.float64, device=cuda)
    out = torch.empty((n_tok, Nh * D), dtype=torch.float32, device=cuda)
    tickets = torch.zeros((n_tok, Nkv), dtype=torch.int32, device=cuda)
    acb.attn_decode(q_out, n_tok, Nh, Nkv, D, d_pos, d_kc, d_vc, max_seq, 0, set_per_tok, 1.0 / np.sqrt(D), ns,
                    scores, smax, part, out=out, tickets=tickets, flags=acb.FLAG_PDL)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    # in-kernel combine == the double split partials added and rounded once; tickets back to zero
    pn = part.cpu().numpy()
    comb = pn.sum(axis=1).astype(np.float32)
    assert_bitexact(out.cpu().numpy(), comb, "combine")
    assert not tickets.cpu().numpy().any()
    # oracle: q/k norm + rope, cache write, attention over [0, pos]
    rt = O.rope_cache(pos, D, 1e6)
    qr = O.qk_norm_rope(qkv[:, :Nh * D].reshape(n_tok, Nh, D), qn, 1e-6, rt)
    kr = O.qk_norm_rope(qkv[:, Nh * D:(Nh + Nkv) * D].reshape(n_tok, Nkv, D), kn, 1e-6, rt)
    vr = qkv[:, (Nh + Nkv) * D:].reshape(n_tok, Nkv, D)
    assert_bitexact(q_out.cpu().numpy().reshape(n_tok, Nh, D), qr, "q")
    kc2, vc2 = kc.copy(), vc.copy()
    for t in range(n_tok):
        s = t if set_per_tok else 0
        kc2[s, :, pos[t]] = kr[t].astype(np.float16)
        vc2[s, :, pos[t]] = vr[t].astype(np.float16)
    assert np.array_equal(d_kc.cpu().numpy(), kc2.view(np.uint16))
    assert np.array_equal(d_vc.cpu().numpy(), vc2.view(np.uint16))
    got = out.cpu().numpy()
    for t in range(n_tok):
        s = t if set_per_tok else 0
        L = pos[t] + 1
        ref = O.attention(qr[t:t + 1], kc2[s, :, :L].view(np.uint16), vc2[s, :, :L].view(np.uint16), O.F16, None,
                          1.0 / np.sqrt(D), kv_head_major=True)
        # same exponential, double sums on both sides: the split count does not matter
        assert_bitexact(got[t], ref.reshape(-1), f"attention token {t} (kv_len {L})")


def test_argmax(cuda):
    import torch
    rng = np.random.default_rng(5)
    lg = rng.standard_normal((3, 217472)).astype(np.float32)
    lg[1, 1234] = lg[1, 99] = 50.0  # tie -> lowest index
    ids = torch.empty(3, dtype=torch.int32, device=cuda)
    marg = torch.empty(3, dtype=torch.float32, device=cuda)
    scratch = acb.argmax(T(lg, cuda), ids, margin=marg)
    torch.cuda.synchronize()
    assert ids.cpu().numpy().tolist() == [int(np.argmax(r)) for r in lg]
    s = np.sort(lg, axis=1)
    assert np.allclose(marg.cpu().numpy(), s[:, -1] - s[:, -2])
    # the scratch (ticket counters) is reusable: a second call on new data with the same scratch
    lg2 = rng.standard_normal((3, 217472)).astype(np.float32)
    acb.argmax(T(lg2, cuda), ids, scratch=scratch)
    torch.cuda.synchronize()
    assert ids.cpu().numpy().tolist() == [int(np.argmax(r)) for r in lg2]
    # odd length (scalar tail path)
    lg3 = rng.standard_normal((1, 1001)).astype(np.float32)
    acb.argmax(T(lg3, cuda), ids[:1])
    torch.cuda.synchronize()
    assert int(ids[0].item()) == int(np.argmax(lg3))


def test_argmax_scratch_reused_across_shapes(cuda):
    """One scratch buffer sized for the largest shape serves calls of other shapes in any order:
    the row counters sit at a fixed offset, never where an earlier call left a partial."""
    import torch
    rng = np.random.default_rng(6)
    big = acb.lib().acb_argmax_scratch_bytes(32, 217472)
    scratch = torch.zeros(big, dtype=torch.uint8, device=cuda)
    for rows, V in ((3, 217472), (1, 151936), (32, 217472), (1, 8192), (7, 1001), (2, 217472)):
        lg = rng.standard_normal((rows, V)).astype(np.float32)
        ids = torch.full((rows,), -1, dtype=torch.int32, device=cuda)
        marg = torch.empty(rows, dtype=torch.float32, device=cuda)
        acb.argmax(T(lg, cuda), ids, margin=marg, scratch=scratch)
        torch.cuda.synchronize()
        assert ids.cpu().numpy().tolist() == [int(np.argmax(r)) for r in lg], (rows, V)
        srt = np.sort(lg, axis=1)
        assert np.array_equal(marg.cpu().numpy(), srt[:, -1] - srt[:, -2]), (rows, V)
    assert not scratch[:4096].any()  # every counter back at zero


# ---- whole LM ----------------------------------------------------------------------------------

def _models(tmp_path, policy, seed):
    p = str(tmp_path / "lm.gguf")
    t = make_tensors(TINY, policy, seed=seed, embed_std=0.5)
    write_gguf(p, TINY, t)
    gpu = acb.QW3LM(p, max_seq_len=256, n_kv_sets=4)
    ora = oracle_model(TINY, t)
    ora.alloc_kv(4, 256)
    return gpu, ora


@pytest.mark.parametrize("policy", [policy_all(O.Q8_0), policy_q4_k_m], ids=["q8_0", "q4_k_m"])
def test_lm_prefill_and_greedy_decode(cuda, tmp_path, policy):
    gpu, ora = _models(tmp_path, policy, seed=21)
    rng = np.random.default_rng(0)
    prompt = rng.integers(0, TINY["vocab_size"], size=40).astype(np.int32)
    lg = gpu.forward(prompt, kv_set=0)
    lr = ora.prefill(prompt, set_=0)
    assert cos_sim(lg, lr) > 0.99999 and max_rel(lg, lr) < 1e-3, (cos_sim(lg, lr), max_rel(lg, lr))
    assert gpu.kv_pos(0) == 40
    # greedy: the device loop continues from the prefill's argmax
    n = 24
    first = int(np.argmax(lg))
    toks, marg, _ = gpu.generate_greedy([first], 0, n, want_margins=True)
    ora2 = oracle_model(TINY, make_tensors(TINY, policy, seed=21, embed_std=0.5))
    ora2.alloc_kv(1, 256)
    rtoks, rmarg = oracle_greedy(ora2, prompt, n)
    assert toks[0].tolist() == rtoks, (toks[0].tolist(), rtoks, rmarg)
    assert gpu.kv_pos(0) == 40 + n
    gpu.close()


def test_lm_forward_batch_ragged_sets(cuda, tmp_path):
    gpu, ora = _models(tmp_path, policy_all(O.Q8_0), seed=5)
    rng = np.random.default_rng(1)
    lens = [7, 19, 3]
    for s, L in enumerate(lens):
        p = rng.integers(0, TINY["vocab_size"], size=L).astype(np.int32)
        gpu.forward(p, kv_set=s)
        ora.prefill(p, set_=s)
    for step in range(3):
        ids = rng.integers(0, TINY["vocab_size"], size=3).astype(np.int32)
        g = gpu.forward_batch(ids, [0, 1, 2])
        r = ora.decode(ids, set0=0)
        for i in range(3):
            assert cos_sim(g[i], r[i]) > 0.99999 and max_rel(g[i], r[i]) < 1e-3, \
                (step, i, cos_sim(g[i], r[i]), max_rel(g[i], r[i]))
    # partial head: rows [lm_offset, V)
    gpu.build_partial_head(600)
    ids = np.array([5, 6, 7], np.int32)
    g = gpu.forward_batch(ids, [0, 1, 2], lm_offset=600, lm_count=400)
    r = ora.decode(ids, set0=0, lm_offset=600, lm_count=400)
    # after several steps the two KV caches differ by f16 rounding flips: bf16-tier bar
    assert g.shape == (3, 400) and max_rel(g, r) < 1e-2 and cos_sim(g, r) > 0.99999, (max_rel(g, r), cos_sim(g, r))
    # copy_kv then decode from the copy equals decoding the original
    gpu.copy_kv(1, 3)
    a = gpu.forward_batch(np.array([9], np.int32), [3])
    b = gpu.forward_batch(np.array([9], np.int32), [1])
    assert np.array_equal(a, b)
    gpu.close()


def test_lm_errors(cuda, tmp_path):
    gpu, _ = _models(tmp_path, policy_all(O.Q8_0), seed=2)
    with pytest.raises(acb.AcbError) as e:
        gpu.forward(np.array([TINY["vocab_size"]], np.int32))
    assert e.value.status == 4
    with pytest.raises(acb.AcbError):
        gpu.forward_batch(np.array([1, 2], np.int32), [0, 2])  # sets not consecutive
    with pytest.raises(acb.AcbError) as e:
        gpu.forward(np.zeros(300, np.int32))  # exceeds max_seq 256
    assert e.value.status == 4
    gpu.close()


@pytest.mark.parametrize("M,N,K", [(1, 4096, 2048), (1, 2048, 6144), (3, 512, 2048), (8, 256, 9728), (1, 1024, 2560)])
def test_gemv_q8_0_tiles(cuda, M, N, K):
    """Q8_0 weights repacked into tensor-core tiles (acb_q8_0_to_tiles, w_type Q8_0_TILES): the
    int8 mma path against the oracle's quantised mul_mat (same per-block integer sums and
    scales, block terms added in double), with every prologue and the residual epilogue."""
    rng = np.random.default_rng(N + K + M)
    W = O.quantize((rng.standard_normal((N, K)) * 0.02).astype(np.float32), O.Q8_0)
    Wt = acb.q8_0_to_tiles(TW(W, cuda), N, K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    y = acb.gemv(Wt, acb.Q8_0_TILES, N, K, T(x, cuda), M=M)
    assert_bitexact(y.cpu().numpy(), O.mul_mat(O.Q8_0, W, N, K, x), "tiles gemv")
    w = (1 + 0.01 * rng.standard_normal(K)).astype(np.float32)
    res = rng.standard_normal((M, N)).astype(np.float32)
    y = acb.gemv(Wt, acb.Q8_0_TILES, N, K, T(x * 3, cuda), M=M, prologue=acb.PRO_RMSNORM, norm_w=T(w, cuda),
                 epilogue=acb.EPI_ADD, res=T(res, cuda), flags=acb.FLAG_PDL)
    ref = (res + O.mul_mat(O.Q8_0, W, N, K, O.rms_norm(x * 3, w, 1e-6))).astype(np.float32)
    assert_bitexact(y.cpu().numpy(), ref, "tiles gemv rmsnorm + residual")
    gu = rng.standard_normal((M, 2 * K)).astype(np.float32)
    y = acb.gemv(Wt, acb.Q8_0_TILES, N, K, T(gu, cuda), M=M, prologue=acb.PRO_SWIGLU, x_stride=2 * K)
    ref = O.mul_mat(O.Q8_0, W, N, K, O.swiglu(gu[:, :K], gu[:, K:]))
    assert_bitexact(y.cpu().numpy(), ref, "tiles gemv swiglu")


# ---- single-sequence decode as one persistent launch (acb_lm_decode_step) ----------------------

def _persist_pair(tmp_path, cfg, seed, max_seq=512):
    """One GGUF loaded twice: persistent single-sequence decode, and the per-op graph."""
    import os
    p = str(tmp_path / "lm16.gguf")
    t = make_tensors(cfg, policy_all(O.Q8_0), seed=seed, embed_std=0.5)
    write_gguf(p, cfg, t)
    a = acb.QW3LM(p, max_seq_len=max_seq, n_kv_sets=2)
    os.environ["ACB_LM_PERSIST"] = "0"
    try:
        b = acb.QW3LM(p, max_seq_len=max_seq, n_kv_sets=2)
    finally:
        del os.environ["ACB_LM_PERSIST"]
    return a, b, t


# vocabulary a multiple of 16 (the head is tiled); q heads per kv head 2, 4, 1; one wide layer
# (ffn 6144: three activation chunks per thread in the down projection's prologue)
PERSIST_CFGS = {
    "g2": dict(TINY, vocab_size=1008),
    "g4": dict(TINY, vocab_size=1008, num_key_value_heads=1),
    "g1": dict(TINY, vocab_size=1008, num_key_value_heads=4),
    "wide": dict(TINY, vocab_size=2048, hidden_size=2048, intermediate_size=6144, num_hidden_layers=1,
                 num_attention_heads=16, num_key_value_heads=8),
}


@pytest.mark.parametrize("name", list(PERSIST_CFGS))
def test_lm_persistent_greedy(cuda, tmp_path, name):
    cfg = PERSIST_CFGS[name]
    per, ref, t = _persist_pair(tmp_path, cfg, seed=31)
    assert per.persistent_decode() and not ref.persistent_decode()
    rng = np.random.default_rng(3)
    prompt = rng.integers(0, cfg["vocab_size"], size=150).astype(np.int32)
    lg = per.forward(prompt, kv_set=0)
    ref.forward(prompt, kv_set=0)
    n = 24
    first = int(np.argmax(lg))
    toks, marg, _ = per.generate_greedy([first], 0, n, want_margins=True)
    rtoks, rmarg, _ = ref.generate_greedy([first], 0, n, want_margins=True)
    assert toks[0].tolist() == rtoks[0].tolist(), (toks, rtoks)
    assert np.allclose(marg, rmarg, rtol=1e-3, atol=1e-4)
    ora = oracle_model(cfg, t)
    ora.alloc_kv(1, 512)
    otoks, omarg = oracle_greedy(ora, prompt, n)
    assert toks[0].tolist() == otoks, (toks[0].tolist(), otoks, omarg)
    assert per.kv_pos(0) == 150 + n
    per.close()
    ref.close()


def test_lm_persistent_forward_batch(cuda, tmp_path):
    cfg = PERSIST_CFGS["g2"]
    per, ref, t = _persist_pair(tmp_path, cfg, seed=32)
    ora = oracle_model(cfg, t)
    ora.alloc_kv(2, 512)
    rng = np.random.default_rng(4)
    p = rng.integers(0, cfg["vocab_size"], size=77).astype(np.int32)
    per.forward(p, kv_set=1)
    ref.forward(p, kv_set=1)
    ora.prefill(p, set_=1)
    for step in range(4):
        ids = rng.integers(0, cfg["vocab_size"], size=1).astype(np.int32)
        g = per.forward_batch(ids, [1])
        h = ref.forward_batch(ids, [1])
        r = ora.decode(ids, set0=1)
        assert cos_sim(g[0], r[0]) > 0.99999 and max_rel(g[0], r[0]) < 1e-3, (step, cos_sim(g[0], r[0]))
        assert cos_sim(g[0], h[0]) > 0.999999 and max_rel(g[0], h[0]) < 1e-4, (step, max_rel(g[0], h[0]))
    assert per.kv_pos(1) == 81 and per.kv_pos(0) == 0
    per.close()
    ref.close()


def test_lm_greedy_batch_then_single_same_handle(cuda, tmp_path):
    """Q4_K_M weights (per-op graph, K-quant GEMVs): a greedy run of 4 sequences, then one of a
    single sequence on the same handle (the argmax scratch is reused with fewer rows and the
    other step graph), both equal to the oracle's greedy loops."""
    gpu, _ = _models(tmp_path, policy_q4_k_m, seed=23)
    t = make_tensors(TINY, policy_q4_k_m, seed=23, embed_std=0.5)
    rng = np.random.default_rng(8)
    prompts = [rng.integers(0, TINY["vocab_size"], size=n).astype(np.int32) for n in (30, 11, 47, 5)]
    firsts = []
    for s, p in enumerate(prompts):
        firsts.append(int(np.argmax(gpu.forward(p, kv_set=s))))
    n = 12
    toks, _, _ = gpu.generate_greedy(firsts, 0, n)
    for s, p in enumerate(prompts):
        ora = oracle_model(TINY, t)
        ora.alloc_kv(1, 256)
        rtoks, _ = oracle_greedy(ora, p, n)
        assert toks[s].tolist() == rtoks, (s, toks[s].tolist(), rtoks)
    # a single sequence after the batch of four
    gpu.reset_kv(0)
    p = prompts[2]
    first = int(np.argmax(gpu.forward(p, kv_set=0)))
    toks1, _, _ = gpu.generate_greedy([first], 0, n)
    ora = oracle_model(TINY, t)
    ora.alloc_kv(1, 256)
    rtoks, _ = oracle_greedy(ora, p, n)
    assert toks1[0].tolist() == rtoks, (toks1[0].tolist(), rtoks)
    gpu.close()


# config 3 (28 layers, hidden 2048, 16/8 heads of 128, FFN 6144, vocabulary 217,472, Q8_0
# weights N(0, 0.02), tied head); ACB_TEST_C3_LAYERS=<n> runs a shallower copy on slow hosts
C3_LAYERS = int(__import__("os").environ.get("ACB_TEST_C3_LAYERS", "28"))
C3 = dict(vocab_size=217472, hidden_size=2048, intermediate_size=6144, num_hidden_layers=C3_LAYERS,
          num_attention_heads=16, num_key_value_heads=8, head_dim=128, rope_theta=1000000.0, rms_norm_eps=1e-6,
          tie_word_embeddings=True)


def test_lm_greedy_256_tokens_identical_config3_shape(cuda, tmp_path):
    """greedy decode gives the same token stream as the reference arithmetic for
    the first 256 tokens. Config 3's widths, a 512-token random prompt; both GPU decode paths
    (the persistent single-sequence step and the per-op graph) against the oracle's greedy
    loop. The prefill logits are bit-identical too, and so are the two paths' margins."""
    import os
    p = str(tmp_path / "c3.gguf")
    t = make_tensors(C3, policy_all(O.Q8_0), seed=33)
    write_gguf(p, C3, t)
    per = acb.QW3LM(p, max_seq_len=1024, n_kv_sets=1)
    os.environ["ACB_LM_PERSIST"] = "0"
    try:
        ref = acb.QW3LM(p, max_seq_len=1024, n_kv_sets=1)
    finally:
        del os.environ["ACB_LM_PERSIST"]
    assert per.persistent_decode() and not ref.persistent_decode()
    rng = np.random.default_rng(512)
    prompt = rng.integers(0, C3["vocab_size"], size=512).astype(np.int32)
    lg = per.forward(prompt, kv_set=0)
    lg2 = ref.forward(prompt, kv_set=0)
    ora = oracle_model(C3, t)
    ora.alloc_kv(1, 1024)
    lr = ora.prefill(prompt, set_=0)
    assert_bitexact(lg, lr, "prefill logits (persistent handle)")
    assert_bitexact(lg2, lr, "prefill logits (per-op handle)")
    n = 256
    first = int(np.argmax(lr))
    toks, marg, _ = per.generate_greedy([first], 0, n, want_margins=True)
    rtoks, rmarg, _ = ref.generate_greedy([first], 0, n, want_margins=True)
    otoks, omarg = [], []
    nxt = first
    for _ in range(n):
        lo = ora.decode(np.array([nxt], np.int32), set0=0)[0]
        nxt = int(np.argmax(lo))
        srt = np.sort(lo)
        otoks.append(nxt)
        omarg.append(float(srt[-1] - srt[-2]))
    first_diff = lambda a, b: next((i for i, (x, y) in enumerate(zip(a, b)) if x != y), None)
    assert toks[0].tolist() == otoks, ("persistent vs oracle", first_diff(toks[0].tolist(), otoks))
    assert rtoks[0].tolist() == otoks, ("per-op vs oracle", first_diff(rtoks[0].tolist(), otoks))
    assert np.array_equal(np.asarray(marg, np.float32).ravel(), np.asarray(rmarg, np.float32).ravel())
    assert np.array_equal(np.asarray(marg, np.float32).ravel(), np.asarray(omarg, np.float32))
    per.close()
    ref.close()
