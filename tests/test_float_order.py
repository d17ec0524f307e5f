"""The row kernels take a warp's max of |h| (or |act|) with one integer max over the float bit
patterns (redux.sync.max.u32).  That equals the float max when every value is non-negative and
not NaN, which holds for running maxima of absolute values that start at +0 (max.f32 and the
bf16 max return the number when one operand is NaN).  Checked here over every non-negative bf16
value, random float32 values, subnormals, +0 and +inf."""
import numpy as np


def _as_u32(v):
    return np.asarray(v, dtype=np.float32).view(np.uint32)


def test_integer_order_of_nonnegative_floats_is_the_float_order():
    rng = np.random.default_rng(7)
    bf16 = (np.arange(0, 0x7F81, dtype=np.uint32) << 16).view(np.float32)   # +0 .. +inf, no NaN
    rand = np.abs(rng.standard_normal(1 << 16).astype(np.float32)) * np.float32(10.0) ** rng.integers(-40, 38, 1 << 16)
    sub = (rng.integers(1, 1 << 23, 4096, dtype=np.uint32)).view(np.float32)   # subnormals
    vals = np.concatenate([bf16, rand.astype(np.float32), sub, np.float32([0.0, np.inf])])
    assert not np.isnan(vals).any() and (vals >= 0).all()
    order_f = np.argsort(vals, kind="stable")
    order_u = np.argsort(_as_u32(vals), kind="stable")
    np.testing.assert_array_equal(vals[order_f], vals[order_u])
    # per-"warp" maxima of 32 values agree bit for bit
    w = vals[: (vals.size // 32) * 32].reshape(-1, 32)
    np.testing.assert_array_equal(_as_u32(w.max(axis=1)), _as_u32(w).max(axis=1))


def test_running_abs_max_from_plus_zero_never_becomes_nan():
    x = np.float32([np.nan, -3.0, np.nan, 2.5, -np.inf, -0.0])
    m = np.float32(0.0)
    for v in x:
        m = np.fmax(m, np.abs(v))   # fmax returns the number when one operand is NaN, as max.f32 does
    assert m == np.inf and not np.isnan(m)
