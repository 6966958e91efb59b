"""Helpers shared by the GPU parity tests (tolerances are stated here once)."""
import numpy as np

# north-star tolerance for matmuls and logits: 1e-3 relative (fp32 accumulate)
REL_TOL = 1e-3


def rel_errors(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    d = got - ref
    norm = np.linalg.norm(d) / max(np.linalg.norm(ref), 1e-30)
    mx = np.abs(d).max() / max(np.abs(ref).max(), 1e-30)
    return norm, mx


def assert_close(got, ref, tol=REL_TOL, what=""):
    norm, mx = rel_errors(got, ref)
    assert norm <= tol and mx <= tol, f"{what}: normwise {norm:.3e}, max/max {mx:.3e} > {tol}"
