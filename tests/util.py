"""Shared parity metrics. Tolerance (fp16 KV, fp32 accumulate): max-abs <= 2e-3
and relative L2 <= 1e-3 against the CPU oracle."""
import numpy as np

MAX_ABS = 2e-3
REL_L2 = 1e-3


def errs(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    d = got - ref
    return float(np.max(np.abs(d))) if d.size else 0.0, \
        float(np.linalg.norm(d) / max(np.linalg.norm(ref), 1e-30))


def assert_parity(got, ref, max_abs=MAX_ABS, rel_l2=REL_L2, what=""):
    ma, rl = errs(got, ref)
    assert np.all(np.isfinite(got)), f"{what}: non-finite output"
    assert ma <= max_abs and rl <= rel_l2, f"{what}: max_abs={ma:.3e} rel_l2={rl:.3e}"
    return ma, rl
