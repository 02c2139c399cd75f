"""GPU: the condition encoder and the FSQ detokenizer / tokenizer (acb_cond_*, acb_detok_*,
acb_tok_* of acb_models.h) against the oracle's restatement of cond_ggml_forward
(src/cond-enc.h:171-381), detok_ggml_decode (src/fsq-detok.h:128-212) and tok_ggml_encode
(src/fsq-tok.h:133-238), through the C ABI, on synthetic GGUFs with the reference's tensor names.

Bars: the float outputs (packed encoder states, context latents) at cosine >= 0.9999 and
max_rel <= 1e-2 per segment; the small ops bit-exact (FSQ decode + project_out, the FSQ index of
given pre-activations, the row packing kernels); the tokenizer's codes equal to the oracle's
except where the oracle's own level value lies within 1e-3 of a rounding boundary (a code is a
floor of a float computed through two encoder layers: a difference in the last bits there is a
different, equally valid code).

Shapes cover the sliding window of the even layers (S_lyric 200 > 129), the XL timbre CLS token,
no timbre input, ragged frame counts padded from the silence latent, and K-quant weights whose
64-wide inputs stay BF16."""
import os

import numpy as np
import pytest

import acb
import oracle as O
from helpers import assert_bitexact, cos_sim, max_rel

pytestmark = pytest.mark.gpu

DIT_TINY = dict(n_layers=1, hidden_size=256, intermediate_size=512, n_heads=4, n_kv_heads=2, head_dim=128,
                in_channels=192, out_channels=64, patch_size=2, sliding_window=16, rope_theta=1000000.0,
                rms_norm_eps=1e-6, enc_hidden_size=256)


def _bars(got, ref, what):
    c, e = cos_sim(got, ref), max_rel(got, ref)
    assert c >= 0.9999 and e <= 1e-2, (what, c, e)


@pytest.fixture(scope="module")
def models(tmp_path_factory, cuda):
    import synthetic
    out = {}
    for name, qt, xl in (("q8", synthetic.Q8_0, False), ("q8xl", synthetic.Q8_0, True),
                         ("q4k", synthetic.Q4_K, False)):
        path = os.path.join(str(tmp_path_factory.mktemp(name)), "dit.gguf")
        keep = {}
        synthetic.write_dit_gguf(path, DIT_TINY, qt, seed=41, device="cuda", keep=keep, cond=synthetic.COND_TINY,
                                 timbre_cls=xl, decoder=False)
        out[name] = (path, keep, xl)
    return out


# ---- the small ops -----------------------------------------------------------------------------

def test_fsq_project_out_bitexact(cuda):
    import torch
    rng = np.random.default_rng(3)
    G, N = 300, 256
    codes = np.concatenate([[0, 63999, 32036], rng.integers(0, 64000, G - 3)]).astype(np.int32)
    for wt in (acb.BF16, acb.F16, acb.F32):
        w32 = (rng.standard_normal((N, 6)) * 0.5).astype(np.float32)
        if wt == acb.BF16:
            w = O.f32_to_bf16_bits(w32)
        elif wt == acb.F16:
            w = w32.astype(np.float16).view(np.uint16)
        else:
            w = w32
        b = (rng.standard_normal(N) * 0.1).astype(np.float32)
        x = np.stack([O.fsq_decode_index(c) for c in codes])
        ref = O.mul_mat(wt, w, N, 6, x) + b
        d_codes = torch.from_numpy(codes).cuda()
        d_w = torch.from_numpy(np.ascontiguousarray(w)).cuda()
        d_b = torch.from_numpy(b).cuda()
        out = torch.empty((G, N), dtype=torch.float32, device="cuda")
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        acb._check("acb_fsq_project_out", acb.lib().acb_fsq_project_out(
            d_codes.data_ptr(), G, d_w.data_ptr(), wt, N, d_b.data_ptr(), out.data_ptr(), N, err.data_ptr(),
            acb._stream(None)))
        torch.cuda.synchronize()
        assert err.item() == 0
        assert_bitexact(out.cpu().numpy(), ref.astype(np.float32), f"project_out type {wt}")


def test_fsq_project_out_negative_code_flags(cuda):
    import torch
    codes = torch.tensor([5, -1, 7], dtype=torch.int32, device="cuda")
    w = torch.zeros((8, 6), dtype=torch.float32, device="cuda")
    out = torch.full((3, 8), 7.0, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    acb._check("acb_fsq_project_out", acb.lib().acb_fsq_project_out(
        codes.data_ptr(), 3, w.data_ptr(), acb.F32, 8, None, out.data_ptr(), 8, err.data_ptr(), acb._stream(None)))
    torch.cuda.synchronize()
    assert err.item() == 8  # ACB_DEVERR_CODE_RANGE
    assert torch.all(out[1] == 0)


def test_fsq_quantize_matches_oracle(cuda):
    import torch
    rng = np.random.default_rng(4)
    G = 5000
    raw = (rng.standard_normal((G, 8)) * 1.5).astype(np.float32)
    bias = (rng.standard_normal(6) * 0.2).astype(np.float32)
    ref = np.array([O.fsq_encode_index(raw[g, :6] + bias) for g in range(G)], dtype=np.int32)
    d_raw = torch.from_numpy(raw).cuda()
    d_b = torch.from_numpy(bias).cuda()
    codes = torch.empty(G, dtype=torch.int32, device="cuda")
    acb._check("acb_fsq_quantize", acb.lib().acb_fsq_quantize(d_raw.data_ptr(), 8, d_b.data_ptr(), G,
                                                              codes.data_ptr(), acb._stream(None)))
    torch.cuda.synchronize()
    assert np.array_equal(codes.cpu().numpy(), ref)


def test_rows_repeat_add_and_prepend(cuda):
    import torch
    G, P, H = 70, 5, 256
    a = torch.randn((G, H), device="cuda")
    b = torch.randn((P, H), device="cuda")
    out = torch.empty((G * P, H), device="cuda")
    acb._check("acb_rows_repeat_add", acb.lib().acb_rows_repeat_add(
        a.data_ptr(), H, b.data_ptr(), H, G, P, H, out.data_ptr(), H, acb._stream(None)))
    ref = (a[:, None, :] + b[None, :, :]).reshape(G * P, H)
    assert torch.equal(out, ref)
    src = torch.randn((G * P, H), device="cuda")
    head = torch.randn(H, device="cuda")
    out2 = torch.empty((G * (P + 1), H), device="cuda")
    acb._check("acb_rows_prepend", acb.lib().acb_rows_prepend(
        head.data_ptr(), src.data_ptr(), H, G, P, H, out2.data_ptr(), H, acb._stream(None)))
    ref2 = torch.cat([head.expand(G, 1, H), src.reshape(G, P, H)], dim=1).reshape(G * (P + 1), H)
    assert torch.equal(out2, ref2)


# ---- the models --------------------------------------------------------------------------------

@pytest.mark.parametrize("name", ["q8", "q8xl", "q4k"])
def test_cond_forward_matches_oracle(models, name):
    path, keep, xl = models[name]
    import synthetic
    cc = synthetic.COND_TINY
    m = acb.CondEncoder(path)
    assert m.cfg["timbre_cls"] == int(xl) and m.cfg["window"] == 128
    assert m.cfg["lyric_layers"] == cc["lyric_layers"] and m.cfg["hidden_size"] == cc["hidden_size"]
    oc = O.OracleCond(keep, timbre_cls=xl)
    rng = np.random.default_rng(9)
    S_text, S_lyric, S_ref = 37, 200, 50
    text = rng.standard_normal((S_text, cc["text_dim"])).astype(np.float32)
    lyric = rng.standard_normal((S_lyric, cc["lyric_dim"])).astype(np.float32)
    timbre = rng.standard_normal((S_ref, cc["latent_dim"])).astype(np.float32)
    for tb in (timbre, None):
        got = m.forward(text, lyric, tb)
        ref = oc.forward(text, lyric, tb)
        assert got.shape == ref.shape
        _bars(got[:S_lyric], ref[:S_lyric], f"{name} lyric")
        n_t = 1 if tb is not None else 0
        if n_t:
            _bars(got[S_lyric], ref[S_lyric], f"{name} timbre")
        _bars(got[S_lyric + n_t:], ref[S_lyric + n_t:], f"{name} text")
    # the window matters at this length: the unmasked oracle disagrees
    if name == "q8":
        unmasked = oc.forward(text, lyric, timbre, window=0)
        assert cos_sim(unmasked[:S_lyric], ref[:S_lyric]) < 0.9999 or max_rel(unmasked[:S_lyric], ref[:S_lyric]) > 1e-2
    null = m.null_embedding()
    assert_bitexact(null, O._f32_of(keep["null_condition_emb"]).ravel(), "null_condition_emb")
    m.close()


def test_cond_short_lyric_and_repeat(models):
    path, keep, xl = models["q8"]
    import synthetic
    cc = synthetic.COND_TINY
    m = acb.CondEncoder(path)
    oc = O.OracleCond(keep, timbre_cls=xl)
    rng = np.random.default_rng(10)
    for S_text, S_lyric, S_ref in ((1, 1, 1), (9, 64, 3), (37, 200, 50), (5, 20, 7)):
        text = rng.standard_normal((S_text, cc["text_dim"])).astype(np.float32)
        lyric = rng.standard_normal((S_lyric, cc["lyric_dim"])).astype(np.float32)
        timbre = rng.standard_normal((S_ref, cc["latent_dim"])).astype(np.float32)
        got = m.forward(text, lyric, timbre)
        _bars(got, oc.forward(text, lyric, timbre), (S_text, S_lyric, S_ref))
        again = m.forward(text, lyric, timbre)
        assert np.array_equal(got, again)  # deterministic across calls and scratch sizes
    m.close()


@pytest.mark.parametrize("name", ["q8", "q4k"])
def test_detok_matches_oracle(models, name):
    path, keep, _ = models[name]
    m = acb.Detokenizer(path)
    od = O.OracleDetok(keep)
    rng = np.random.default_rng(11)
    for G in (1, 7, 61):
        codes = rng.integers(0, 64000, G).astype(np.int32)
        codes[0] = 63999 if G > 1 else 0
        got = m.decode(codes)
        ref = od.decode(codes)
        assert got.shape == (G * 5, 64)
        for g in range(G):  # every group on its own (groups are independent sequences)
            _bars(got[g * 5:(g + 1) * 5], ref[g * 5:(g + 1) * 5], (name, G, g))
    with pytest.raises(acb.AcbError) as e:
        m.decode(np.array([3, -2], dtype=np.int32))
    assert e.value.status == 4  # ACB_ERR_OUT_OF_RANGE
    m.close()


def _level_margin(raw_row):
    """Distance of the oracle's level value (L-1)(tanh(x)+1)/2 + 0.5 from the nearest integer."""
    L = np.array([8, 8, 8, 5, 5, 5], dtype=np.float64)
    s = (L - 1) * (np.tanh(raw_row.astype(np.float64)) + 1) / 2 + 0.5
    return np.abs(s - np.round(s)).min()


@pytest.mark.parametrize("name", ["q8", "q4k"])
def test_tok_matches_oracle(models, name):
    path, keep, _ = models[name]
    m = acb.Tokenizer(path)
    ot = O.OracleTok(keep)
    rng = np.random.default_rng(12)
    silence = rng.standard_normal((16, 64)).astype(np.float32)
    used = set()
    for T in (5, 23, 5 * 40 + 3):
        lat = rng.standard_normal((T, 64)).astype(np.float32)
        got = m.encode(lat, silence)
        pad = (5 - T % 5) % 5
        padded = np.concatenate([lat, silence[:pad]]) if pad else lat
        ref, raw = ot.encode(padded)
        raw_b = raw + 0  # project_in output with its bias (the oracle adds it)
        assert got.shape == ref.shape
        for g in range(got.size):
            if got[g] != ref[g]:
                assert _level_margin(raw_b[g]) < 1e-3, (name, T, g, got[g], ref[g])
        used.update(int(c) for c in got)
    assert len(used) > 5  # the codes spread over the alphabet
    with pytest.raises(acb.AcbError):
        m.encode(rng.standard_normal((7, 64)).astype(np.float32), None)  # ragged without silence
    m.close()


def test_tok_detok_device_entry_points(models, cuda):
    import torch
    path, keep, _ = models["q8"]
    tok, det = acb.Tokenizer(path), acb.Detokenizer(path)
    rng = np.random.default_rng(13)
    lat = rng.standard_normal((50, 64)).astype(np.float32)
    host_codes = tok.encode(lat)
    d_codes = torch.empty(10, dtype=torch.int32, device="cuda")
    tok.encode_device(torch.from_numpy(lat).cuda(), d_codes)
    torch.cuda.synchronize()
    assert np.array_equal(d_codes.cpu().numpy(), host_codes)
    out = torch.empty((50, 64), dtype=torch.float32, device="cuda")
    det.decode_device(d_codes, out)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), det.decode(host_codes))
    tok.close()
    det.close()
