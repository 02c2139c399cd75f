"""GPU: the device Philox noise (src/philox.h) through the C ABI.

- acb_philox_bits: the integer Philox4x32-10 rounds bit for bit against the oracle (counters that
  cross the 2^32 boundary of the subsequence word, negative and 64-bit seeds);
- acb_philox_randn against the oracle (itself pinned bit for bit to the reference's own
  test-philox dump, tests/golden/philox_golden.npz) over the full 192000-value dump of nine seeds:
  the float tail is CUDA's logf / sinf against the host libm, so a value may land on the other
  side of a bf16 rounding boundary -- bar: at most 1 in 1000 values differ, each by one bf16 step;
  unrounded values within 4e-6 absolute;
- against the golden fixture directly, and against torch.randn on a CUDA generator in bf16 (the
  comparison the reference's own tests/test-philox.py makes; its bar: cosine > 0.9999);
- acb_dit_sde_philox equal bit for bit to acb_dit_sde fed with acb_philox_randn's noise."""
import os

import numpy as np
import pytest

import acb
import oracle as O

pytestmark = pytest.mark.gpu

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "philox_golden.npz"))


def _bf16_close(got, ref, what):
    gb, rb = got.view(np.uint32), ref.view(np.uint32)
    assert not (gb & 0xFFFF).any(), what  # bf16-representable
    diff = gb != rb
    assert diff.mean() <= 1e-3, (what, int(diff.sum()))
    steps = np.abs((gb[diff] >> 16).astype(np.int64) - (rb[diff] >> 16).astype(np.int64))
    assert (steps == 1).all(), (what, steps.max() if steps.size else 0)


@pytest.mark.parametrize("seed,first", [(42, 0), (-1, 7), (2**40 + 7, 2**32 - 100), (9223372036854775807, 123)])
def test_philox_bits_match_oracle(cuda, seed, first):
    n = 4096
    got = acb.philox_bits(seed, first, n).cpu().numpy().view(np.uint32)
    k = (seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF)
    for i in list(range(0, n, 97)) + [n - 1]:
        c = first + i
        ref = O.philox4x32_10([0, 0, c & 0xFFFFFFFF, c >> 32], k)
        assert np.array_equal(got[i], ref), (seed, c)


@pytest.mark.parametrize("i", range(len(GOLD["seeds"])))
def test_philox_randn_matches_oracle_and_reference_dump(cuda, i):
    seed, n = int(GOLD["seeds"][i]), int(GOLD["full_n"])
    got = acb.philox_randn(seed, n).cpu().numpy()
    _bf16_close(got, O.philox_randn(seed, n), f"oracle seed {seed}")
    ref_bits = GOLD["bf16_bits"][i].astype(np.uint32) << 16
    _bf16_close(got[:8192], ref_bits.view(np.float32), f"reference dump seed {seed}")


def test_philox_randn_unrounded_and_edges(cuda):
    import torch
    raw = acb.philox_randn(5, 100000, bf16_round=False).cpu().numpy()
    ref = O.philox_randn(5, 100000, bf16_round=False)
    assert np.abs(raw - ref).max() <= 4e-6
    assert acb.philox_randn(5, 0).numel() == 0
    odd = acb.philox_randn(5, 1237).cpu().numpy()  # a length that is no multiple of a block
    _bf16_close(odd, O.philox_randn(5, 1237), "ragged")
    out = torch.full((10,), 7.0, device=cuda)
    acb.philox_randn(5, 3, out=out)
    assert (out[3:] == 7.0).all()  # nothing written past n
    assert acb.lib().acb_philox_randn(1, None, 10, 1, acb._stream(None)) == 1
    assert acb.lib().acb_philox_bits(1, 0, 4, out.data_ptr() + 4, acb._stream(None)) == 1  # misaligned


def test_philox_randn_matches_torch_cuda_bf16(cuda):
    """The reference's own check (tests/test-philox.py): its stream against torch.randn in bf16 on a
    CUDA generator with the same seed, 192000 values."""
    import torch
    n = 64 * 25 * 120
    for seed in (42, 20260101):
        gen = torch.Generator(device=cuda).manual_seed(seed)
        want = torch.randn([n], generator=gen, device=cuda, dtype=torch.bfloat16).float().cpu().numpy()
        got = acb.philox_randn(seed, n).cpu().numpy()
        cos = float(np.dot(got, want) / (np.linalg.norm(got) * np.linalg.norm(want)))
        assert cos > 0.9999, (seed, cos)
        assert (got == want).mean() >= 0.999, (seed, (got != want).sum())


def test_sde_philox_step_equals_sde_with_device_noise(cuda):
    import torch
    rng = np.random.default_rng(8)
    n_tracks, n_per = 3, 750 * 64 + 3
    x = torch.from_numpy(rng.standard_normal(n_tracks * n_per).astype(np.float32)).to(cuda)
    v = torch.from_numpy(rng.standard_normal(n_tracks * n_per).astype(np.float32)).to(cuda)
    seeds = [11, -4, 2**33 + 1]
    tt = torch.tensor([0.9, 0.9, 0.75], dtype=torch.float32, device=cuda)
    noise = torch.cat([acb.philox_randn(s, n_per) for s in seeds])
    a = acb.dit_sde(x.clone(), v, noise, tt)
    b = acb.dit_sde_philox(x.clone(), v, torch.tensor(seeds, dtype=torch.int64, device=cuda), tt)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    # and the oracle step with the oracle's (reference) noise: equal where the noise is
    z = np.concatenate([O.philox_randn(s, n_per) for s in seeds])
    ref = O.sde_step(x.cpu().numpy(), v.cpu().numpy(), z, 0.9, 0.75)
    same = noise.cpu().numpy() == z
    assert same.mean() >= 0.999
    assert np.array_equal(b.cpu().numpy()[same], ref[same])
