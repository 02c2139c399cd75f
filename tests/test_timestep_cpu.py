"""CPU: pin the oracle's timestep sinusoid (dit_ggml_build_temb, src/dit-graph.h:81-117, over
ggml_timestep_embedding) against the values the reference itself printed on its CPU backend.

The reference's debug runs dump the first four channels of both sinusoids of the first DiT step
(tests/CPU-Q8_0.log:162-163, tests/CPU-Q4_K_M.log:82): at t = 1.0 and t_r = t they read
sinusoidal_t = 0.562379 0.789627 0.439928 -0.023645 (the embedding of t * 1000, i.e. cos(1000 f_j)
with f_j = exp(-ln(10000) j / 128)) and sinusoidal_r = 1 1 1 1 (the embedding of (t - t_r) * 1000
= 0). These numbers do not depend on any weight, so they pin the oracle's scale, frequency ladder
and cos-before-sin layout directly. The printed values have six decimals: the bar is 5e-7."""
import numpy as np

import oracle as O

LOG_SINUSOIDAL_T = np.array([0.562379, 0.789627, 0.439928, -0.023645])
LOG_SINUSOIDAL_R = np.array([1.0, 1.0, 1.0, 1.0])


def test_sinusoid_at_t1_matches_reference_cpu_log():
    e = np.asarray(O.timestep_embedding(np.float32(1.0) * np.float32(1000.0))).ravel()
    assert e.shape == (256,)
    assert np.abs(e[:4] - LOG_SINUSOIDAL_T).max() <= 5e-7, e[:4]


def test_sinusoid_at_zero_offset_matches_reference_cpu_log():
    e = np.asarray(O.timestep_embedding(np.float32(0.0))).ravel()
    assert np.abs(e[:4] - LOG_SINUSOIDAL_R).max() <= 5e-7
    # cos half all ones, sin half all zeros
    assert np.array_equal(e[:128], np.ones(128, np.float32)) and np.array_equal(e[128:], np.zeros(128, np.float32))


def test_sinusoid_layout_and_ladder():
    """cos in channels [0, half), sin in [half, dim), frequencies exp(-ln(P) j / half) (float64 check)."""
    t = 437.5
    e = np.asarray(O.timestep_embedding(np.float32(t))).ravel().astype(np.float64)
    f = np.exp(-np.log(10000.0) * np.arange(128) / 128)
    assert np.abs(e[:128] - np.cos(t * f)).max() <= 1e-4
    assert np.abs(e[128:] - np.sin(t * f)).max() <= 1e-4
    odd = np.asarray(O.timestep_embedding(np.float32(t), dim=257)).ravel()
    assert odd.shape == (257,) and odd[256] == 0.0
