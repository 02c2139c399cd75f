"""GPU parity of the DiT (configs 4 and 5: src/dit.h, src/dit-graph.h, src/dit-sampler.h) through
the C ABI against the oracle's restatement of dit_ggml_build_graph and dit_ggml_generate.

Exact mode (the default) forms every linear's products from hi/lo f16 splits of the reference's
dequantised operands and runs attention the same way, so values reach each activation quantiser
at fp32 summation-order distance from the reference; bars per sample: cosine >= 0.9999 and
max_rel (max |out - ref| / max |ref|) <= 1e-2 on the velocity of one evaluation and on the x0 of
a whole CFG + APG generate. Fast mode (single f16 operands) is checked with looser bars.
"""
import os

import numpy as np
import pytest

import acb
import oracle as O
from helpers import cos_sim, max_rel

pytestmark = pytest.mark.gpu

DIT_TINY = dict(n_layers=2, hidden_size=256, intermediate_size=512, n_heads=4, n_kv_heads=2, head_dim=128,
                in_channels=64, out_channels=32, patch_size=2, sliding_window=16, rope_theta=1000000.0,
                rms_norm_eps=1e-6, enc_hidden_size=256)


def _model(tmp_path, cfg, seed, null_condition=True):
    import synthetic
    keep = {}
    path = os.path.join(str(tmp_path), "dit.gguf")
    synthetic.write_dit_gguf(path, cfg, synthetic.Q8_0, seed=seed, device="cuda", keep=keep,
                             null_condition=null_condition)
    return path, keep


def _check(out, ref, cos_bar, rel_bar, what):
    for b in range(ref.shape[0]):
        c, r = cos_sim(out[b], ref[b]), max_rel(out[b], ref[b])
        assert c >= cos_bar and r <= rel_bar, f"{what} sample {b}: cosine {c:.7f}, max_rel {r:.3g}"


@pytest.mark.parametrize("t,t_r", [(0.7, 0.7), (0.9, 0.3)])
def test_dit_forward_matches_oracle(cuda, tmp_path, t, t_r):
    import torch
    cfg = DIT_TINY
    path, keep = _model(tmp_path, cfg, seed=1)
    dit = acb.DiT(path)
    for k in ("n_layers", "hidden_size", "in_channels", "out_channels", "patch_size", "sliding_window"):
        assert dit.cfg[k] == cfg[k], k
    assert dit.cfg["enc_hidden_size"] == cfg["enc_hidden_size"] and dit.cfg["has_null_condition"] == 1
    rng = np.random.default_rng(3)
    N, T, enc_S = 2, 80, 24  # S = 40 > sliding window 16: layer 0 is windowed
    x = rng.standard_normal((N, T, cfg["in_channels"])).astype(np.float32)
    enc = rng.standard_normal((N, enc_S, cfg["enc_hidden_size"])).astype(np.float32)
    od = O.dit_from_gguf_tensors(cfg, keep)
    xd, ed = torch.from_numpy(x).to(cuda), torch.from_numpy(enc).to(cuda)
    for nl in (1, -1):
        got = dit.forward(xd, ed, t, t_r, n_layers_run=nl).cpu().numpy()
        ref = od.forward(x, enc, t, t_r, n_layers_run=nl)
        assert np.isfinite(got).all()
        _check(got, ref, 0.9999, 1e-2, f"exact, {nl} layers")
    dit.set_exact(False)
    got = dit.forward(xd, ed, t, t_r).cpu().numpy()
    _check(got, od.forward(x, enc, t, t_r), 0.999, 5e-2, "fast")
    dit.close()


def test_dit_generate_cfg_apg_matches_oracle(cuda, tmp_path):
    cfg = DIT_TINY
    path, keep = _model(tmp_path, cfg, seed=2)
    dit = acb.DiT(path)
    rng = np.random.default_rng(5)
    N, T, enc_S, Oc = 2, 80, 24, cfg["out_channels"]
    noise = rng.standard_normal((N, T, Oc)).astype(np.float32)
    ctx = rng.standard_normal((N, T, cfg["in_channels"] - Oc)).astype(np.float32)
    enc = rng.standard_normal((N, enc_S, cfg["enc_hidden_size"])).astype(np.float32)
    sched = acb.turbo_schedule(4)
    od = O.dit_from_gguf_tensors(cfg, keep)
    null = keep["null_condition_emb"][1].astype(np.float32)
    for g in (1.0, 3.0):
        x0, ms = dit.generate(noise, ctx, enc, sched, guidance_scale=g)
        ref = O.dit_generate(od, noise, ctx, enc, null, sched, g)
        assert np.isfinite(x0).all() and ms > 0
        _check(x0, ref, 0.9999, 1e-2, f"generate guidance {g}")
    # DPM++ 3M through the same driver (Euler, second and third order steps, then the x0 step)
    x0d, _ = dit.generate(noise, ctx, enc, sched, guidance_scale=3.0, solver="dpm3m")
    _check(x0d, O.dit_generate(od, noise, ctx, enc, null, sched, 3.0, solver="dpm3m"), 0.9999, 1e-2,
           "generate dpm3m")
    # repeat: the captured step graphs give identical results
    x0b, _ = dit.generate(noise, ctx, enc, sched, guidance_scale=3.0)
    x0c, _ = dit.generate(noise, ctx, enc, sched, guidance_scale=3.0)
    assert np.array_equal(x0b, x0c)
    dit.close()


def test_dit_without_null_condition_runs_without_cfg(cuda, tmp_path):
    cfg = DIT_TINY
    path, keep = _model(tmp_path, cfg, seed=4, null_condition=False)
    dit = acb.DiT(path)
    assert dit.cfg["has_null_condition"] == 0
    rng = np.random.default_rng(9)
    N, T, enc_S, Oc = 1, 40, 8, cfg["out_channels"]
    noise = rng.standard_normal((N, T, Oc)).astype(np.float32)
    ctx = rng.standard_normal((N, T, cfg["in_channels"] - Oc)).astype(np.float32)
    enc = rng.standard_normal((N, enc_S, cfg["enc_hidden_size"])).astype(np.float32)
    a, _ = dit.generate(noise, ctx, enc, [1.0, 0.5], guidance_scale=5.0)  # CFG disabled, like the reference
    b, _ = dit.generate(noise, ctx, enc, [1.0, 0.5], guidance_scale=1.0)
    assert np.array_equal(a, b)
    dit.close()


def test_dit_padding_masks_match_oracle(cuda, tmp_path):
    """dit_ggml_generate's padding masks (dit-sampler.h:244-304) on ragged tracks: sequence b
    attends only among its real_S[b] patch positions (inside the window on the sliding layers;
    padded query rows get a zero attention output) and to its real_enc_S[b] condition rows. One
    evaluation through set_condition / set_lengths / eval, against the oracle's masked forward."""
    import torch
    cfg = DIT_TINY
    path, keep = _model(tmp_path, cfg, seed=12)
    dit = acb.DiT(path)
    od = O.dit_from_gguf_tensors(cfg, keep)
    rng = np.random.default_rng(13)
    N, T, enc_S = 3, 80, 24  # S = 40 > window 16
    real_S, real_enc_S = [40, 29, 7], [24, 13, 1]
    x = rng.standard_normal((N, T, cfg["in_channels"])).astype(np.float32)
    enc = rng.standard_normal((N, enc_S, cfg["enc_hidden_size"])).astype(np.float32)
    xd, ed = torch.from_numpy(x).to(cuda), torch.from_numpy(enc).to(cuda)
    out = torch.empty((N, T, cfg["out_channels"]), dtype=torch.float32, device=cuda)
    tt = torch.tensor([0.8, 0.8], dtype=torch.float32, device=cuda)
    dit.set_condition(ed, T)
    dit.set_lengths(real_S, real_enc_S)
    got = dit.eval(xd, tt, out).cpu().numpy()
    ref = od.forward(x, enc, 0.8, 0.8, real_S=real_S, real_enc_S=real_enc_S)
    assert np.isfinite(got).all()
    _check(got, ref, 0.9999, 1e-2, "masked evaluation")
    # the masks change the result (they are not ignored), and all-real lengths are the unmasked model
    plain = od.forward(x, enc, 0.8, 0.8)
    assert cos_sim(ref[1], plain[1]) < 0.999
    dit.set_lengths([40, 40, 40], [24, 24, 24])
    _check(dit.eval(xd, tt, out).cpu().numpy(), plain, 0.9999, 1e-2, "all-real lengths")
    dit.close()


def _np_randn(seed, n):
    """A stand-in noise source for the SDE solver (the reference passes its Philox generator)."""
    return np.random.default_rng(seed).standard_normal(n).astype(np.float32)


def test_dit_generate_ex_matches_oracle(cuda, tmp_path):
    """acb_dit_generate_ex with dit_ggml_generate's arguments: ragged tracks (real_S, real_enc_S),
    batched CFG + APG, the SDE solver with per-track seeds, and cover mode (context and condition
    switched at step 2, the conditional slots' condition lengths with them), against the oracle's
    generate over the same inputs and noise."""
    cfg = DIT_TINY
    path, keep = _model(tmp_path, cfg, seed=14)
    dit = acb.DiT(path)
    od = O.dit_from_gguf_tensors(cfg, keep)
    null = keep["null_condition_emb"][1].astype(np.float32)
    rng = np.random.default_rng(15)
    N, T, enc_S, Oc = 2, 80, 24, cfg["out_channels"]
    noise = rng.standard_normal((N, T, Oc)).astype(np.float32)
    ctx = rng.standard_normal((N, T, cfg["in_channels"] - Oc)).astype(np.float32)
    ctx2 = rng.standard_normal((N, T, cfg["in_channels"] - Oc)).astype(np.float32)
    enc = rng.standard_normal((N, enc_S, cfg["enc_hidden_size"])).astype(np.float32)
    enc2 = rng.standard_normal((N, enc_S, cfg["enc_hidden_size"])).astype(np.float32)
    sched = acb.turbo_schedule(4)
    seeds = [1234, 98765]
    kw = dict(real_S=[40, 31], real_enc_S=[24, 17])
    for solver in ("euler", "sde", "dpm3m"):
        x0, ms = dit.generate_ex(noise, ctx, enc, sched, guidance_scale=3.0, solver=solver, seeds=seeds,
                                 randn=_np_randn, **kw)
        ref = O.dit_generate(od, noise, ctx, enc, null, sched, 3.0, solver=solver, seeds=seeds, randn=_np_randn, **kw)
        assert np.isfinite(x0).all() and ms > 0
        _check(x0, ref, 0.9999, 1e-2, f"generate_ex {solver}")
    cover = dict(context_switch=ctx2, cover_steps=2, enc_switch=enc2, real_enc_S_switch=[9, 24])
    x0, _ = dit.generate_ex(noise, ctx, enc, sched, guidance_scale=3.0, **kw, **cover)
    ref = O.dit_generate(od, noise, ctx, enc, null, sched, 3.0, **kw, **cover)
    _check(x0, ref, 0.9999, 1e-2, "generate_ex cover mode")
    dit.close()


def test_dit_generate_ex_cancel_and_unsupported(cuda, tmp_path):
    """The cancel callback is polled before every step; a cancelled run returns ACB_ERR_CANCELLED
    and the model stays usable. STORK4 without its tables is reported as unsupported, nothing runs."""
    cfg = DIT_TINY
    path, keep = _model(tmp_path, cfg, seed=16)
    dit = acb.DiT(path)
    rng = np.random.default_rng(17)
    N, T, enc_S, Oc = 1, 40, 8, cfg["out_channels"]
    noise = rng.standard_normal((N, T, Oc)).astype(np.float32)
    ctx = rng.standard_normal((N, T, cfg["in_channels"] - Oc)).astype(np.float32)
    enc = rng.standard_normal((N, enc_S, cfg["enc_hidden_size"])).astype(np.float32)
    sched = acb.turbo_schedule(8)
    polls = []
    with pytest.raises(acb.AcbError) as e:
        dit.generate_ex(noise, ctx, enc, sched, guidance_scale=3.0, cancel=lambda k: polls.append(k) or k == 3)
    assert e.value.status == 9 and polls == [0, 1, 2, 3]
    a, _ = dit.generate_ex(noise, ctx, enc, sched, guidance_scale=3.0, cancel=lambda k: False)
    b, _ = dit.generate(noise, ctx, enc, sched, guidance_scale=3.0)
    assert np.array_equal(a, b)
    with pytest.raises(acb.AcbError) as e:
        dit.generate_ex(noise, ctx, enc, sched, guidance_scale=3.0, solver="stork4")
    assert e.value.status == 2
    dit.close()


def test_dit_generate_dcw_matches_oracle(cuda, tmp_path):
    """DCW (dit-sampler.h:613-666, dwt-haar.h) through acb_dit_generate_ex: the four modes after
    Euler steps, low after DPM++ 3M steps, all against the oracle's generate; DCW changes the
    result, and with the SDE solver it is not applied. (Frame counts are multiples of the patch
    size, so the transform's odd-T padding is pinned on the CPU, tests/test_solver_cpu.py.)"""
    cfg = DIT_TINY
    path, keep = _model(tmp_path, cfg, seed=18)
    dit = acb.DiT(path)
    od = O.dit_from_gguf_tensors(cfg, keep)
    null = keep["null_condition_emb"][1].astype(np.float32)
    rng = np.random.default_rng(19)
    N, T, enc_S, Oc = 2, 78, 12, cfg["out_channels"]  # 39 tokens: frame pairs of the transform = tokens
    noise = rng.standard_normal((N, T, Oc)).astype(np.float32)
    ctx = rng.standard_normal((N, T, cfg["in_channels"] - Oc)).astype(np.float32)
    enc = rng.standard_normal((N, enc_S, cfg["enc_hidden_size"])).astype(np.float32)
    sched = acb.turbo_schedule(4)
    plain, _ = dit.generate_ex(noise, ctx, enc, sched, guidance_scale=3.0)
    cases = [("euler", "low", 0.3, 0.0), ("euler", "high", 0.3, 0.0), ("euler", "double", 0.3, 0.2),
             ("euler", "pix", 0.1, 0.0), ("dpm3m", "low", 0.3, 0.0)]
    for solver, mode, sc, hs in cases:
        x0, _ = dit.generate_ex(noise, ctx, enc, sched, guidance_scale=3.0, solver=solver, dcw_scaler=sc,
                                dcw_high_scaler=hs, dcw_mode=mode)
        ref = O.dit_generate(od, noise, ctx, enc, null, sched, 3.0, solver=solver, dcw_scaler=sc,
                             dcw_high_scaler=hs, dcw_mode=mode)
        assert np.isfinite(x0).all()
        _check(x0, ref, 0.9999, 1e-2, f"dcw {solver} {mode}")
        if solver == "euler":
            assert max_rel(x0, plain) > 1e-3, mode  # the correction is applied
    seeds = [5, 6]
    a, _ = dit.generate_ex(noise, ctx, enc, sched, guidance_scale=3.0, solver="sde", seeds=seeds, randn=_np_randn,
                           dcw_scaler=0.3)
    b, _ = dit.generate_ex(noise, ctx, enc, sched, guidance_scale=3.0, solver="sde", seeds=seeds, randn=_np_randn)
    assert np.array_equal(a, b)
    dit.close()


@pytest.mark.parametrize("t,t_r", [(1.0, 1.0), (0.75, 0.25), (0.3, 0.0), (0.0, 0.0)])
def test_dit_sinusoid_matches_oracle(cuda, t, t_r):
    """acb_dit_sinusoid (dit_ggml_build_temb, dit-graph.h:81-117): row 0 embeds t * 1000, row 1
    (t - t_r) * 1000, cos half then sin half. The device's expf/cosf/sinf and the host libm's may
    differ by a few ulp; with arguments up to 1000 that moves a channel by at most ~4e-4, so the
    bar is 1e-3 absolute. At t = 1 both rows also match the reference's CPU-backend dump
    (tests/CPU-Q8_0.log:162-163) to that bar."""
    import torch
    tt = torch.tensor([t, t_r], dtype=torch.float32, device=cuda)
    out = torch.empty((2, 256), dtype=torch.float32, device=cuda)
    acb._check("acb_dit_sinusoid", acb.lib().acb_dit_sinusoid(tt.data_ptr(), 256, 10000, out.data_ptr(),
                                                               acb._stream(None)))
    got = out.cpu().numpy()
    a = np.float32(t) * np.float32(1000.0)
    b = np.float32(np.float32(t) - np.float32(t_r)) * np.float32(1000.0)
    assert np.abs(got[0] - O.timestep_embedding(a)).max() <= 1e-3
    assert np.abs(got[1] - O.timestep_embedding(b)).max() <= 1e-3
    if t == 1.0 and t_r == 1.0:
        assert np.abs(got[0, :4] - [0.562379, 0.789627, 0.439928, -0.023645]).max() <= 1e-3
        assert np.array_equal(got[1], np.concatenate([np.ones(128), np.zeros(128)]).astype(np.float32))
    assert acb.lib().acb_dit_sinusoid(None, 256, 10000, out.data_ptr(), acb._stream(None)) == 1


def test_dit_config4_width_matches_oracle(cuda, tmp_path):
    """Config 4 layer shapes (hidden 2048, FFN 6144, 16/8 heads, 1500 frames -> 750 tokens with
    the 128 sliding window, 512 condition rows) with 2 layers and 2 sequences."""
    import torch
    import synthetic
    cfg = dict(synthetic.ACESTEP_DIT_2B, n_layers=2)
    path, keep = _model(tmp_path, cfg, seed=7)
    dit = acb.DiT(path)
    rng = np.random.default_rng(11)
    N, T, enc_S = 2, 1500, 512
    x = rng.standard_normal((N, T, cfg["in_channels"])).astype(np.float32)
    enc = rng.standard_normal((N, enc_S, cfg["enc_hidden_size"])).astype(np.float32)
    got = dit.forward(torch.from_numpy(x).to(cuda), torch.from_numpy(enc).to(cuda), 0.75, 0.75).cpu().numpy()
    dit.close()
    ref = O.dit_from_gguf_tensors(cfg, keep).forward(x, enc, 0.75, 0.75)
    _check(got, ref, 0.9999, 1e-2, "config-4 width")


def test_dpm3m_solver_steps_match_oracle(cuda):
    """The DPM++ 3M solver (solver-dpm.h:14-50) over a whole 8-step schedule on N=2 x 750 x 64
    latents plus a ragged tail: every intermediate xt and the stored velocity history bit-identical
    to the oracle (Euler bootstrap, then second order, then third), the x0 of the last step through
    acb_dit_euler as for every solver."""
    import torch
    rng = np.random.default_rng(33)
    n = 2 * 750 * 64 + 37
    sched = [1.0, 0.955, 0.9, 0.833, 0.75, 0.643, 0.5, 0.3]
    x_ref = rng.standard_normal(n).astype(np.float32)
    xt = torch.from_numpy(x_ref.copy()).to(cuda)
    prev = torch.full((n,), float("nan"), device=cuda)  # unused until history says otherwise
    prev2 = torch.full((n,), float("nan"), device=cuda)
    p_ref = pp_ref = None
    for step, t in enumerate(sched):
        v = (rng.standard_normal(n) * 0.5).astype(np.float32)
        vd = torch.from_numpy(v).to(cuda)
        t_next = sched[step + 1] if step + 1 < len(sched) else 0.0
        tt = torch.tensor([t, t, t_next], dtype=torch.float32, device=cuda)
        if step == len(sched) - 1:
            out = torch.empty_like(xt)
            acb.dit_euler(xt, vd, tt, True, out=out)
            want = (x_ref - (v * np.float32(t)).astype(np.float32)).astype(np.float32)
            assert np.array_equal(out.cpu().numpy(), want)
            break
        acb.dit_dpm3m(xt, vd, prev, prev2, min(step, 2), tt)
        x_ref, p_ref, pp_ref = O.dpm3m_step(x_ref, v, p_ref, pp_ref, t, t_next)
        assert np.array_equal(xt.cpu().numpy(), x_ref), f"step {step}"
        assert np.array_equal(prev.cpu().numpy(), p_ref)
        if pp_ref is not None:
            assert np.array_equal(prev2.cpu().numpy(), pp_ref)
    with pytest.raises(acb.AcbError):  # a negative history is rejected before any launch
        acb.dit_dpm3m(xt, vd, prev, prev2, -1, tt)


def test_dit_generate_sde_device_noise_matches_oracle(cuda, tmp_path):
    """The SDE solver with no host noise source: the library draws the reference's Philox stream
    (seed_b + step + 1, bf16) inside each step; the oracle's generate gets the oracle's Philox
    (pinned to the reference's own dump) as its source. Same bars as every generate."""
    cfg = DIT_TINY
    path, keep = _model(tmp_path, cfg, seed=16)
    dit = acb.DiT(path)
    od = O.dit_from_gguf_tensors(cfg, keep)
    null = keep["null_condition_emb"][1].astype(np.float32)
    rng = np.random.default_rng(17)
    N, T, enc_S, Oc = 2, 64, 16, cfg["out_channels"]
    noise = np.stack([O.philox_randn(s, T * Oc).reshape(T, Oc) for s in (77, 78)])
    ctx = rng.standard_normal((N, T, cfg["in_channels"] - Oc)).astype(np.float32)
    enc = rng.standard_normal((N, enc_S, cfg["enc_hidden_size"])).astype(np.float32)
    sched = acb.turbo_schedule(4)
    seeds = [77, 2**35 + 3]
    x0, _ = dit.generate_ex(noise, ctx, enc, sched, guidance_scale=3.0, solver="sde", seeds=seeds)
    ref = O.dit_generate(od, noise, ctx, enc, null, sched, 3.0, solver="sde", seeds=seeds, randn=O.philox_randn)
    _check(x0, ref, 0.9999, 1e-2, "sde device noise")
    # the host source given the same stream lands on the same trajectory
    x1, _ = dit.generate_ex(noise, ctx, enc, sched, guidance_scale=3.0, solver="sde", seeds=seeds,
                            randn=O.philox_randn)
    _check(x1, x0, 0.9999, 1e-2, "sde host vs device noise")
    dit.close()


def test_sde_solver_steps_match_oracle(cuda):
    """The SDE ancestral solver (solver-sde.h:17-38) over a schedule, with bf16-rounded seeded
    normal noise as the reference draws it: every step bit-identical to the oracle."""
    import torch
    rng = np.random.default_rng(44)
    n = 2 * 750 * 64 + 5
    sched = [1.0, 0.9, 0.75, 0.5, 0.3]
    x_ref = rng.standard_normal(n).astype(np.float32)
    xt = torch.from_numpy(x_ref.copy()).to(cuda)
    for step in range(len(sched) - 1):
        v = (rng.standard_normal(n) * 0.5).astype(np.float32)
        z = O.round_bf16(rng.standard_normal(n).astype(np.float32))
        tt = torch.tensor([sched[step], sched[step], sched[step + 1]], dtype=torch.float32, device=cuda)
        acb.dit_sde(xt, torch.from_numpy(v).to(cuda), torch.from_numpy(z).to(cuda), tt)
        x_ref = O.sde_step(x_ref, v, z, sched[step], sched[step + 1])
        assert np.array_equal(xt.cpu().numpy(), x_ref), f"step {step}"
