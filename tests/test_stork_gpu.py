"""GPU: the STORK4 solver (acb_stork4_*, and the "stork4" solver of acb_dit_generate_ex) against the
oracle's restatement of solver_stork4_step (src/solvers/solver-stork.h:270-315).

The ROCK4 tables are data the caller supplies (the reference compiles them in); the tests use
seeded synthetic tables of the same shape (increasing degrees, finishing and recurrence
coefficients), which exercise the same arithmetic. Bars: every step's latent bit-identical to the
oracle (the solver is elementwise f32 / f64 arithmetic in the reference's order; only its
stability guards reduce, and they compare against thresholds), including the derivative orders
2 / 1 / 0, the halving of the sub step count on a non-finite pass and the Euler bootstrap; the
whole DiT generate with stork4 at the DiT bars (cosine >= 0.9999, max_rel <= 1e-2)."""
import os

import numpy as np
import pytest

import acb
import oracle as O
from helpers import assert_bitexact, cos_sim, max_rel

pytestmark = pytest.mark.gpu


def synth_tables(seed=0, blow_degree=None):
    """Tables shaped like ROCK4's: ms increasing, fpa [len][6], fpb [len][4], recf covering every
    degree's recurrence. blow_degree: that degree's recurrence coefficients overflow f32."""
    rng = np.random.default_rng(seed)
    ms = np.array([1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 12, 14, 16], dtype=np.int32)
    n = int(sum(2 * m - 1 for m in ms)) + 4
    recf = rng.uniform(0.05, 0.4, n)
    if blow_degree is not None:
        mr = int(sum(2 * m - 1 for m in ms[ms < blow_degree]))
        recf[mr:mr + 2 * (blow_degree - 2) + 3] = 1e19
    fpa = rng.uniform(-0.5, 0.5, (ms.size, 6))
    fpb = rng.uniform(0.0, 0.5, (ms.size, 4))
    return dict(ms=ms, fpa=fpa, fpb=fpb, recf=recf)


def _velocities(rng, n, k):
    base = rng.standard_normal(n).astype(np.float32)
    out = []
    for i in range(k):
        v = base + np.float32(0.05 * i) * rng.standard_normal(n).astype(np.float32)
        if i == 5:
            v = v * np.float32(0.1)  # a jump: the first-derivative guard drops to order 0
        out.append(v.astype(np.float32))
    return out


@pytest.mark.parametrize("substeps,blow", [(10, None), (16, None), (10, 10), (3, None)])
def test_stork4_steps_bitexact(cuda, substeps, blow):
    import torch
    rng = np.random.default_rng(substeps)
    n = 3 * 750 * 64 + 5
    tables = synth_tables(substeps, blow)
    sched = [1.0, 0.95, 0.9, 0.8, 0.7, 0.55, 0.4, 0.3, 0.2, 0.1]
    x = rng.standard_normal(n).astype(np.float32)
    vs = _velocities(rng, n, len(sched) - 1)
    dev = acb.Stork4(tables, n, substeps)
    ref = O.Stork4(tables, substeps)
    d_x = torch.from_numpy(x.copy()).cuda()
    for k in range(len(sched) - 1):
        d_v = torch.from_numpy(vs[k]).cuda()
        dev.step(d_x, d_v, sched[k], sched[k + 1])
        x = ref.step(x, vs[k], sched[k], sched[k + 1])
        got = d_x.cpu().numpy()
        assert np.all(np.isfinite(got))
        assert_bitexact(got, x, f"step {k}")
    dev.close()


def test_dit_generate_stork4_matches_oracle(cuda, tmp_path):
    import synthetic
    cfg = dict(n_layers=2, hidden_size=256, intermediate_size=512, n_heads=4, n_kv_heads=2, head_dim=128,
               in_channels=64, out_channels=32, patch_size=2, sliding_window=16, rope_theta=1000000.0,
               rms_norm_eps=1e-6, enc_hidden_size=256)
    keep = {}
    path = os.path.join(str(tmp_path), "dit.gguf")
    synthetic.write_dit_gguf(path, cfg, synthetic.Q8_0, seed=51, device="cuda", keep=keep)
    od = O.dit_from_gguf_tensors(cfg, keep)
    null = keep["null_condition_emb"][1].astype(np.float32)
    rng = np.random.default_rng(52)
    N, T, enc_S, Oc = 2, 64, 20, cfg["out_channels"]
    noise = rng.standard_normal((N, T, Oc)).astype(np.float32)
    ctx = rng.standard_normal((N, T, cfg["in_channels"] - Oc)).astype(np.float32)
    enc = rng.standard_normal((N, enc_S, cfg["enc_hidden_size"])).astype(np.float32)
    sched = acb.turbo_schedule(8)
    tables = synth_tables(7)
    dit = acb.DiT(path)
    with pytest.raises(acb.AcbError):  # no tables yet
        dit.generate_ex(noise, ctx, enc, sched, guidance_scale=3.0, solver="stork4")
    dit.set_stork4_tables(tables)
    got, _ = dit.generate_ex(noise, ctx, enc, sched, guidance_scale=3.0, solver="stork4", stork_substeps=10)
    ref = O.dit_generate(od, noise, ctx, enc, null, sched, 3.0, solver="stork4", stork_tables=tables,
                         stork_substeps=10)
    for b in range(N):
        c, e = cos_sim(got[b], ref[b]), max_rel(got[b], ref[b])
        assert c >= 0.9999 and e <= 1e-2, (b, c, e)
    dit.close()
