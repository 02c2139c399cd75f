"""CPU: the oracle's Philox noise (src/philox.h) pinned bit for bit against the reference's own
generator: tests/golden/philox_golden.npz holds what the reference's tests/test-philox.cpp printed
(compiled from the reference checkout, tests/golden/make_golden.py) for nine seeds -- small,
negative, above 2^32, INT64_MIN and INT64_MAX -- as bf16 bits of the first 8192 values plus the
SHA-256 of the whole 192000-value dump (64 channels x 25 Hz x 120 s, the size the reference's
test-philox.py compares against torch.randn on CUDA).

Also properties of the layout that do not restate the formulas: value k comes from counter
{0, 0, k_lo, k_hi} alone (any window of the stream equals the same window of a longer run), the
unrounded stream rounds to the bf16 stream, and the values look like N(0, 1)."""
import hashlib
import os

import numpy as np
import pytest

import oracle as O

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "philox_golden.npz"))


def _bits(v):
    return (v.view(np.uint32) >> 16).astype(np.uint16)


@pytest.mark.parametrize("i", range(len(GOLD["seeds"])))
def test_oracle_philox_matches_reference_dump(i):
    seed = int(GOLD["seeds"][i])
    v = O.philox_randn(seed, int(GOLD["full_n"]))
    assert not (v.view(np.uint32) & 0xFFFF).any()  # every value bf16-representable
    assert np.array_equal(_bits(v[:8192]), GOLD["bf16_bits"][i]), seed
    assert hashlib.sha256(v.tobytes()).hexdigest() == str(GOLD["full_sha256"][i]), seed


def test_philox_value_depends_on_its_counter_only():
    long = O.philox_randn(7, 5000)
    assert np.array_equal(O.philox_randn(7, 1234), long[:1234])
    # element k is the first Box-Muller normal of counter {0, 0, k, 0}: recompute k = 4321 by hand
    w = O.philox4x32_10([0, 0, 4321, 0], (7, 0))
    u = np.float32(np.float32(w[0]) * np.float32(2.0 ** -32) + np.float32(2.0 ** -33))
    a = np.float32(np.float32(w[1]) * np.float32(2 * np.pi * 2.0 ** -32) + np.float32(np.pi * 2.0 ** -32))
    z = np.sqrt(-2.0 * np.log(np.float64(u))) * np.sin(np.float64(a))
    assert abs(float(long[4321]) - z) <= 2 ** -8 * max(abs(z), 1e-3)  # within bf16 rounding


def test_philox_rounds_and_keys_are_distinct():
    """Different counters, different key words: different outputs (no word of the state is dropped)."""
    outs = {tuple(O.philox4x32_10(c, k)) for c, k in [([0, 0, 0, 0], (0, 0)), ([1, 0, 0, 0], (0, 0)),
                                                      ([0, 1, 0, 0], (0, 0)), ([0, 0, 1, 0], (0, 0)),
                                                      ([0, 0, 0, 1], (0, 0)), ([0, 0, 0, 0], (1, 0)),
                                                      ([0, 0, 0, 0], (0, 1))]}
    assert len(outs) == 7


def test_philox_unrounded_rounds_to_bf16_stream():
    raw = O.philox_randn(99, 20000, bf16_round=False)
    r = O.philox_randn(99, 20000)
    u = raw.view(np.uint32)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).view(np.float32)
    assert np.array_equal(rounded, r)


def test_philox_looks_normal():
    v = O.philox_randn(2026, 192000).astype(np.float64)
    assert abs(v.mean()) < 0.01 and abs(v.std() - 1.0) < 0.01
    assert abs((np.abs(v) < 1.0).mean() - 0.6827) < 0.005
