"""GPU: LM token sampling on the device (acb_sample_top_k_p) against the oracle's restatement of
sample_top_k_p (src/sampling.h:30-133), with the phase-2 targeted CFG + EOS/audio-code compaction
of src/pipeline-lm.cpp:474-497 in front.

Bars:
- greedy (temperature 0): the index is identical to the oracle's on every row (first maximum);
- sampling: the reference adds its probabilities one by one in f32 (a running sum whose rounding
  reaches V * 2^-24 of the total) and the device in a fixed parallel order, so an index may differ
  where the draw falls within that rounding of a boundary: the device's index must lie between
  the oracle's indices for u moved by that bound either way (and top_p moved by 1e-5), and on
  truncated rows (top_k / top_p) at least half the draws must match exactly;
- the device result is deterministic (two launches agree bit for bit).
The uniforms u are the canonical variates a std::mt19937 would give the reference's
uniform_real_distribution; here they are seeded numpy draws, including 0 and values close to 1.
"""
import numpy as np
import pytest

import acb
import oracle as O

pytestmark = pytest.mark.gpu

EOS, CODE_OFF, N_CODES = 151645, 151669, 64000  # TOKEN_IM_END, AUDIO_CODE_BASE, AUDIO_CODE_COUNT


def _accept(row, temp, top_p, top_k, u, got):
    """(accepted, exact): exact when the oracle returns the same index; accepted when the device's
    index lies between the oracle's indices for u -/+ d, d = V * 2^-24 (the bound of the rounding
    of the reference's one-by-one f32 running sum relative to its total; the index is monotone in
    u), with top_p also moved by 1e-5 for the nucleus boundary."""
    ref = O.sample_top_k_p(row, temp, top_p, top_k, u)
    if ref == got:
        return True, True
    d = row.size * 2.0 ** -24 + 1e-6
    umax = float(np.nextafter(np.float32(1), np.float32(0)))
    for pp in ((top_p, top_p - 1e-5, top_p + 1e-5) if 0 < top_p < 1 else (top_p,)):
        lo = O.sample_top_k_p(row, temp, pp, top_k, max(u - d, 0.0))
        hi = O.sample_top_k_p(row, temp, pp, top_k, min(u + d, umax))
        if hi < lo:  # u + d past the running sum's end: the reference falls back to index 0
            hi = row.size - 1
        if lo <= got <= hi:
            return True, False
    return False, False


@pytest.mark.parametrize("temp,top_p,top_k", [(0.0, 0.9, 0), (1.0, 1.0, 0), (0.85, 0.9, 0), (1.0, 0.95, 50),
                                              (1.2, 1.0, 200), (0.7, 0.5, 0)])
def test_sample_whole_rows_matches_oracle(cuda, temp, top_p, top_k):
    import torch
    rng = np.random.default_rng(int(temp * 100) + top_k)
    rows, V = 48, 70000
    x = (rng.standard_normal((rows, V)) * 2.5).astype(np.float32)
    x[:, 123] += 9.0  # a few dominant tokens, as a trained LM head gives
    x[:, 60000] += 8.5
    u = rng.random(rows).astype(np.float32)
    u[0], u[1] = 0.0, np.float32(0.99999994)
    d_x = torch.from_numpy(x).cuda()
    d_u = torch.from_numpy(u).cuda()
    got = acb.sample_top_k_p(d_x, temp, top_p, top_k, d_u).cpu().numpy()
    again = acb.sample_top_k_p(d_x, temp, top_p, top_k, d_u).cpu().numpy()
    assert np.array_equal(got, again)
    exact = 0
    for r in range(rows):
        ok, ex = _accept(x[r], temp, top_p, top_k, float(u[r]), int(got[r]))
        assert ok, (r, got[r], O.sample_top_k_p(x[r], temp, top_p, top_k, float(u[r])))
        exact += ex
    if temp <= 0:
        assert exact == rows
    elif top_k > 0 or 0 < top_p < 1:
        assert exact >= rows // 2, exact  # truncated rows: most draws land away from a boundary


def test_sample_cfg_compact_matches_oracle(cuda):
    import torch
    rng = np.random.default_rng(77)
    rows, V = 8, CODE_OFF + N_CODES
    lc = (rng.standard_normal((rows, V)) * 2.0).astype(np.float32)
    lu = (rng.standard_normal((rows, V)) * 2.0).astype(np.float32)
    u = rng.random(rows).astype(np.float32)
    d_lc, d_lu, d_u = (torch.from_numpy(a).cuda() for a in (lc, lu, u))
    for temp, top_p, top_k, cfg in ((0.85, 0.9, 0, 2.0), (1.0, 1.0, 0, 1.5), (0.0, 0.9, 0, 2.0)):
        got = acb.sample_top_k_p(d_lc, temp, top_p, top_k, d_u, uncond=d_lu, cfg_scale=cfg, col0=EOS,
                                 span_off=CODE_OFF, span_len=N_CODES).cpu().numpy()
        for r in range(rows):
            row = O.lm_compact_cfg(lc[r], lu[r], cfg, EOS, CODE_OFF, N_CODES)
            ok, _ = _accept(row, temp, top_p, top_k, float(u[r]), int(got[r]))
            assert ok, (temp, top_p, r, got[r])
    # without CFG: the compaction alone
    got = acb.sample_top_k_p(d_lc, 0.0, 1.0, 0, None, col0=EOS, span_off=CODE_OFF, span_len=N_CODES).cpu().numpy()
    for r in range(rows):
        assert got[r] == int(np.argmax(O.lm_compact_cfg(lc[r], None, 1.0, EOS, CODE_OFF, N_CODES)))


def test_sample_distribution(cuda):
    """Many draws from one row follow the kept tokens' softmax (a chi-square-like check)."""
    import torch
    rng = np.random.default_rng(5)
    V, n = 1000, 20000
    row = (rng.standard_normal(V) * 1.5).astype(np.float32)
    x = np.repeat(row[None, :], n, axis=0)
    u = rng.random(n).astype(np.float32)
    got = acb.sample_top_k_p(torch.from_numpy(x).cuda(), 1.0, 1.0, 20, torch.from_numpy(u).cuda()).cpu().numpy()
    top = np.argsort(-row)[:20]
    assert set(np.unique(got)) <= set(top.tolist())
    p = np.exp(row[top] - row[top].max())
    p /= p.sum()
    freq = np.array([(got == t).sum() for t in top]) / n
    assert np.abs(freq - p).max() < 0.02


def test_lm_forward_batch_sample_matches_host_sampling(cuda, tmp_path):
    """acb_qw3lm_forward_batch_sample (device CFG + compaction + sampling) against the reference's
    host path: the same step through acb_qw3lm_forward_batch on a second handle, its logits
    combined, compacted and sampled by the oracle (pipeline-lm.cpp:474-497)."""
    import os

    import lm_fixtures as F
    cfg = dict(F.TINY, vocab_size=1000)
    tensors = F.make_tensors(cfg, F.policy_all(O.Q8_0), seed=21, embed_std=0.5)
    path = os.path.join(str(tmp_path), "lm.gguf")
    F.write_gguf(path, cfg, tensors)
    n_active, eos, code_off, n_codes = 3, 7, 200, 700
    a = acb.QW3LM(path, max_seq_len=64, n_kv_sets=2 * n_active)
    b = acb.QW3LM(path, max_seq_len=64, n_kv_sets=2 * n_active)
    rng = np.random.default_rng(3)
    sets = np.arange(2 * n_active, dtype=np.int32)
    for m in (a, b):
        for s_ in sets:
            m.forward(np.array([1, 2, 3 + s_], np.int32), kv_set=int(s_))
    ids = rng.integers(0, 1000, 2 * n_active).astype(np.int32)
    ids[n_active:] = ids[:n_active]  # the uncond half feeds the same token, its own kv set
    exact = 0
    for step, (temp, top_p, top_k) in enumerate([(0.85, 0.9, 0), (1.0, 1.0, 0), (0.0, 0.9, 0), (1.0, 0.95, 40)]):
        u = rng.random(n_active).astype(np.float32)
        got = a.forward_batch_sample(ids, sets, n_active, True, 2.0, eos, code_off, n_codes, temp, top_p, top_k, u)
        lg = b.forward_batch(ids, sets)
        for i in range(n_active):
            row = O.lm_compact_cfg(lg[i], lg[n_active + i], 2.0, eos, code_off, n_codes)
            ok, ex = _accept(row, temp, top_p, top_k, float(u[i]), int(got[i]))
            assert ok, (step, i, got[i])
            exact += ex
        nxt = np.where(got == 0, eos, code_off + got - 1).astype(np.int32)
        ids = np.concatenate([nxt, nxt])
    assert exact >= 8
    assert a.kv_pos(0) == b.kv_pos(0)
    a.close()
    b.close()
