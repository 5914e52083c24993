"""Error metrics and the parity tolerance used by every numerical test.

Tolerance (fp16 operands, fp32 accumulation, against the fp32 oracle):
max-abs <= 1e-2 and rel-L2 <= 1e-3.
"""
import numpy as np

MAX_ABS = 1e-2
REL_L2 = 1e-3


def max_abs(a, b) -> float:
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64)))) if np.size(a) else 0.0


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.linalg.norm(b.ravel())
    return float(np.linalg.norm((a - b).ravel()) / (den if den > 0 else 1.0))


def assert_close(got, want, max_abs_tol=MAX_ABS, rel_tol=REL_L2, what=""):
    got = np.asarray(got)
    want = np.asarray(want)
    assert got.shape == want.shape, (what, got.shape, want.shape)
    assert np.all(np.isfinite(got)), f"{what}: non-finite output"
    ma, rl = max_abs(got, want), rel_l2(got, want)
    assert ma <= max_abs_tol and rl <= rel_tol, f"{what}: max_abs={ma:.3e} rel_l2={rl:.3e}"
    return ma, rl
