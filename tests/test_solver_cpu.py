"""CPU: pin the oracle's DPM++ 3M step (src/solvers/solver-dpm.h:14-50) by properties that do not
restate its formula: the Adams-Bashforth weights of each order sum to one (a constant velocity
field moves xt exactly like Euler), third order integrates a velocity that is quadratic in t
exactly over uniform steps, second order a linear one, and the history moves down one slot per
step with the reference's bootstrap (Euler, then second, then third order). Also the oracle's DCW
step against a frame-by-frame restatement of the Haar pair (odd T included)."""
import numpy as np
import pytest

import oracle as O


def _run(v_of_t, ts, x0):
    x, p, pp = x0.astype(np.float32), None, None
    for a, b in zip(ts[:-1], ts[1:]):
        x, p, pp = O.dpm3m_step(x, v_of_t(a), p, pp, a, b)
    return x, p, pp


def test_dpm3m_constant_velocity_moves_like_euler():
    rng = np.random.default_rng(1)
    v = rng.standard_normal(1000).astype(np.float32)
    x0 = rng.standard_normal(1000).astype(np.float32)
    ts = np.linspace(1.0, 0.25, 7)
    x, _, _ = _run(lambda t: v, ts, x0)
    want = x0.astype(np.float64) - v.astype(np.float64) * (ts[0] - ts[-1])
    assert np.abs(x - want).max() <= 1e-5 * (np.abs(want).max() + 1)


def test_dpm3m_orders_are_exact_on_polynomials():
    # after the bootstrap, a step of order k integrates v(t) of degree k-1 exactly (uniform steps)
    h = 0.125
    ts = 1.0 - h * np.arange(6)
    a, b, c = 0.7, -1.3, 2.1
    quad = lambda t: np.array([a + b * t + c * t * t], dtype=np.float32)
    integral = lambda t0, t1: a * (t0 - t1) + b * (t0 ** 2 - t1 ** 2) / 2 + c * (t0 ** 3 - t1 ** 3) / 3
    x = np.zeros(1, np.float32)
    p = pp = None
    for i in range(5):
        t0, t1 = ts[i], ts[i + 1]
        xb = x.astype(np.float64)
        x, p, pp = O.dpm3m_step(x, quad(t0), p, pp, t0, t1)
        if i >= 2:  # third order from the third step on
            assert abs(float(x[0]) - (xb[0] - integral(t0, t1))) <= 2e-6
    lin = lambda t: np.array([a + b * t], dtype=np.float32)
    x1, p1, _ = O.dpm3m_step(np.zeros(1, np.float32), lin(ts[0]), None, None, ts[0], ts[1])
    x2, _, _ = O.dpm3m_step(x1, lin(ts[1]), p1, None, ts[1], ts[2])
    want = -(a * (ts[1] - ts[2]) + b * (ts[1] ** 2 - ts[2] ** 2) / 2)
    assert abs(float(x2[0] - x1[0]) - want) <= 1e-6


def test_dpm3m_history_shift():
    v0, v1, v2 = (np.full(3, k, np.float32) for k in (1.0, 2.0, 3.0))
    x = np.zeros(3, np.float32)
    x, p, pp = O.dpm3m_step(x, v0, None, None, 1.0, 0.5)
    assert pp is None and np.array_equal(p, v0) and np.array_equal(x, -0.5 * v0)
    x, p, pp = O.dpm3m_step(x, v1, p, pp, 0.5, 0.25)
    assert np.array_equal(p, v1) and np.array_equal(pp, v0)
    x, p, pp = O.dpm3m_step(x, v2, p, pp, 0.25, 0.125)
    assert np.array_equal(p, v2) and np.array_equal(pp, v1)


def test_sde_step_endpoints():
    # t_next = 0 gives the x0 prediction itself; t_next = 1 gives pure noise
    rng = np.random.default_rng(5)
    x, v, z = (rng.standard_normal(64).astype(np.float32) for _ in range(3))
    x0 = (x - (v * np.float32(0.7)).astype(np.float32)).astype(np.float32)
    assert np.array_equal(O.sde_step(x, v, z, 0.7, 0.0), x0)
    assert np.array_equal(O.sde_step(x, v, z, 0.7, 1.0), z)


@pytest.mark.parametrize("T", [6, 7])
def test_dcw_matches_loop_restatement(T):
    """The oracle's DCW (dit-sampler.h:613-666 with dwt-haar.h) against a frame-by-frame restatement
    of the Haar pair, including odd T (the last frame paired with zero and dropped on the way back)
    and the zero-scale early return."""
    f, r = np.float32, np.float32(0.70710678118654752440)
    rng = np.random.default_rng(T)
    xt = rng.standard_normal((2, T, 3)).astype(np.float32)
    v = rng.standard_normal((2, T, 3)).astype(np.float32)
    t_curr, t_next, sc, hs = 0.8, 0.6, 0.3, 0.2

    def fwd(x):
        Tl = (T + 1) // 2
        L = np.zeros((x.shape[0], Tl, x.shape[2]), np.float32)
        H = np.zeros_like(L)
        for j in range(Tl):
            a = x[:, 2 * j]
            if 2 * j + 1 < T:
                b = x[:, 2 * j + 1]
                L[:, j], H[:, j] = ((a + b) * r).astype(f), ((a - b) * r).astype(f)
            else:
                L[:, j], H[:, j] = (a * r).astype(f), (a * r).astype(f)
        return L, H

    def inv(L, H):
        out = np.zeros((L.shape[0], T, L.shape[2]), np.float32)
        for j in range(L.shape[1]):
            out[:, 2 * j] = ((L[:, j] + H[:, j]) * r).astype(f)
            if 2 * j + 1 < T:
                out[:, 2 * j + 1] = ((L[:, j] - H[:, j]) * r).astype(f)
        return out

    den = (xt - (v * f(t_next)).astype(f)).astype(f)
    xL, xH = fwd(xt)
    yL, yH = fwd(den)
    sl, sh, sdh = f(f(t_curr) * f(sc)), f((f(1) - f(t_curr)) * f(sc)), f((f(1) - f(t_curr)) * f(hs))
    want = {
        "low": inv((xL + (sl * (xL - yL)).astype(f)).astype(f), xH),
        "high": inv(xL, (xH + (sh * (xH - yH)).astype(f)).astype(f)),
        "double": inv((xL + (sl * (xL - yL)).astype(f)).astype(f), (xH + (sdh * (xH - yH)).astype(f)).astype(f)),
        "pix": (xt + (f(sc) * (xt - den).astype(f)).astype(f)).astype(f),
    }
    for mode, ref in want.items():
        got = O.dcw_step(xt, v, t_curr, t_next, sc, hs, mode)
        assert np.array_equal(got, ref), mode
    assert np.array_equal(O.dcw_step(xt, v, t_curr, t_next, sc, hs, "nonsense"), want["low"])
    assert O.dcw_step(xt, v, 1.0, t_next, sc, 0.0, "high") is xt  # (1 - t_curr) * scaler = 0: untouched
