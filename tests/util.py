"""Comparison helpers shared by the tests."""
import numpy as np

F16 = np.float16


def max_rel_err(got, ref):
    """Normwise max relative error: max |got - ref| / max |ref| (the fp16
    tolerance measure used throughout; elementwise relative error is not
    meaningful near zero)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    denom = max(np.abs(ref).max(), 1e-30)
    return float(np.abs(got - ref).max() / denom)


def f16_ulps(got, ref):
    """Largest distance in fp16 units-in-the-last-place (same-sign values)."""
    a = np.asarray(got, F16).view(np.int16).astype(np.int64)
    b = np.asarray(ref, F16).view(np.int16).astype(np.int64)
    a = np.where(a < 0, -32768 - a, a)
    b = np.where(b < 0, -32768 - b, b)
    return int(np.abs(a - b).max())
