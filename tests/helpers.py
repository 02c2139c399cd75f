"""Shared comparison helpers for the parity tests (tolerances are written at each call site)."""
import numpy as np


def cos_sim(a, b) -> float:
    a = np.asarray(a, dtype=np.float64).ravel()
    b = np.asarray(b, dtype=np.float64).ravel()
    na, nb = np.linalg.norm(a), np.linalg.norm(b)
    if na == 0 and nb == 0:
        return 1.0
    return float(a @ b / (na * nb))


def max_rel(a, ref) -> float:
    """max |a - ref| / max |ref| (the relative-error measure used for layer outputs)."""
    a = np.asarray(a, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    den = np.abs(ref).max()
    return float(np.abs(a - ref).max() / (den if den > 0 else 1.0))


def assert_bitexact(a, ref, what=""):
    a = np.ascontiguousarray(a)
    ref = np.ascontiguousarray(ref)
    assert a.shape == ref.shape, (what, a.shape, ref.shape)
    va = a.view(np.uint32 if a.dtype == np.float32 else np.uint16)
    vr = ref.view(np.uint32 if ref.dtype == np.float32 else np.uint16)
    bad = np.count_nonzero(va != vr)
    assert bad == 0, f"{what}: {bad} of {a.size} elements differ (max abs {np.abs(a.astype(np.float64) - ref).max()})"


def assert_nearly_exact(a, ref, rel_tol, min_exact_frac, what=""):
    """All elements within rel_tol (relative to max |ref|) and at least min_exact_frac identical."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    ref = np.ascontiguousarray(ref, dtype=np.float32)
    assert a.shape == ref.shape
    exact = np.count_nonzero(a.view(np.uint32) == ref.view(np.uint32)) / max(a.size, 1)
    r = max_rel(a, ref)
    assert r <= rel_tol and exact >= min_exact_frac, f"{what}: max_rel {r:.3g}, exact fraction {exact:.6f}"
