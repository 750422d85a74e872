"""Numerical acceptance shared by the parity tests.

Decoded weights, routed indices and alignment tables: bit-exact. Layer outputs: relative L2 error <= 2e-3 and
max |err| <= 1e-2 * max(1, rms(reference)) against the fp32-accumulated oracle (the BASELINE tolerance
"2e-3 relative / 1e-2 max-abs", with the max-abs bound scaled to the output's magnitude so that an fp16 output
whose values exceed 1 is not failed by its own last-place rounding)."""
import numpy as np

REL_TOL = 2e-3
ABS_TOL = 1e-2


def assert_close(out, ref, rel_tol=REL_TOL, abs_tol=ABS_TOL, what=""):
    out = np.asarray(out, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert out.shape == ref.shape, (what, out.shape, ref.shape)
    assert np.isfinite(out).all(), f"{what}: non-finite output"
    den = np.linalg.norm(ref)
    rel = np.linalg.norm(out - ref) / (den if den > 0 else 1.0)
    rms = float(np.sqrt(np.mean(ref ** 2))) if ref.size else 0.0
    mx = float(np.abs(out - ref).max()) if ref.size else 0.0
    assert rel <= rel_tol, f"{what}: relative error {rel:.3e} > {rel_tol}"
    assert mx <= abs_tol * max(1.0, rms), f"{what}: max abs error {mx:.3e} > {abs_tol} * max(1, rms={rms:.3g})"
    return rel, mx
