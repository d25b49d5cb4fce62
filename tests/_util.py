"""Shared helpers for the parity tests (tolerances are the decode spec's)."""
import numpy as np

# logits / hidden-state tolerance: max-abs 2e-2 and relative (to the
# reference's max magnitude) 1e-2 against the numpy fp32 oracle.
ABS_TOL = 2e-2
REL_TOL = 1e-2


def assert_close(got, ref, abs_tol=ABS_TOL, rel_tol=REL_TOL, what="value"):
    g = np.asarray(got, dtype=np.float32)
    r = np.asarray(ref, dtype=np.float32)
    assert g.shape == r.shape, f"{what}: shape {g.shape} != {r.shape}"
    assert np.all(np.isfinite(g)), f"{what}: non-finite output"
    err = float(np.max(np.abs(g - r))) if g.size else 0.0
    scale = float(np.max(np.abs(r))) if r.size else 0.0
    assert err <= abs_tol, f"{what}: max-abs error {err:.3e} > {abs_tol}"
    assert err <= rel_tol * max(scale, 1e-30) or err <= 1e-6, \
        f"{what}: relative error {err / max(scale, 1e-30):.3e} > {rel_tol}"
    return err


def f16_bits_equal(a, b):
    return np.array_equal(np.asarray(a, np.float16).view(np.uint16), np.asarray(b, np.float16).view(np.uint16))


def greedy_ids_match(gpu_ids, ref_ids, ref_logits_per_step, margin=ABS_TOL):
    """Greedy ids must match wherever the reference's top-2 margin exceeds the
    tolerance; after the first divergence the continuations are different
    sequences, so comparison stops there.  Returns the number of steps compared."""
    from oracle.mirror import top2_margin
    n = 0
    for i, (g, r) in enumerate(zip(gpu_ids, ref_ids)):
        if g != r:
            m = top2_margin(ref_logits_per_step[i])
            assert m <= margin, f"step {i}: gpu id {g} != oracle id {r} with top-2 margin {m:.3e}"
            return n
        n += 1
    return n
