"""The activation digits' integer X = rint(v / step) with a correctly rounded binary32 division (the reference's
arithmetic) equals rint(RN32(RN64(v) * RN64(1 / step))), the form the CUDA kernels use (umma_sm100.cuh,
digit_quotient: one double multiply per element instead of a float division). numpy's float32 division and
float64 multiply / float32 conversion are IEEE round-to-nearest, so this checks the identity itself on the CPU;
the GPU parity tests check the kernels that use it against the oracle."""
import numpy as np
import pytest

RANGE = np.float32(8355710.0)


def _x_division(v: np.ndarray, step: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore", under="ignore"):
        return np.rint(np.divide(v, step, dtype=np.float32)).astype(np.int64)


def _x_reciprocal(v: np.ndarray, step: np.ndarray) -> np.ndarray:
    r = 1.0 / step.astype(np.float64)
    with np.errstate(over="ignore", under="ignore"):
        return np.rint((v.astype(np.float64) * r).astype(np.float32)).astype(np.int64)


def _steps(rows: np.ndarray) -> np.ndarray:
    mx = np.abs(rows).max(axis=1, keepdims=True).astype(np.float32)
    return np.where(mx > 0, mx / RANGE, np.float32(1.0)).astype(np.float32)


@pytest.mark.parametrize("scale_exp", [-118, -60, -20, -3, 0, 7, 40, 100])
def test_reciprocal_digits_match_division_on_random_rows(scale_exp):
    rng = np.random.default_rng(1000 + scale_exp)
    rows = (rng.standard_normal((256, 1536)) * 2.0 ** scale_exp).astype(np.float32)
    # heavy-tailed rows too: a few large entries set the step, the rest span many binades
    rows[::4] *= np.exp2(rng.integers(-30, 1, rows[::4].shape)).astype(np.float32)
    step = _steps(rows)
    keep = step[:, 0] > 0  # max |v| / RANGE underflowing to zero leaves no finite digits on either path
    rows, step = rows[keep], step[keep]
    assert rows.shape[0] > 0
    np.testing.assert_array_equal(_x_reciprocal(rows, step), _x_division(rows, step))


def test_reciprocal_digits_match_division_on_arbitrary_float_pairs():
    """Uniformly random bit patterns for v and step (finite, step > 0, |v| <= RANGE * step), every binade."""
    rng = np.random.default_rng(7)
    n = 2_000_000
    step = rng.integers(1, 0x7F7FFFFF, n, dtype=np.uint32).view(np.float32)
    frac = rng.random(n).astype(np.float32) * np.where(rng.random(n) < 0.5, -1, 1).astype(np.float32)
    with np.errstate(over="ignore", under="ignore"):
        v = (frac * RANGE * step).astype(np.float32)
    ok = np.isfinite(v)
    v, step = v[ok], step[ok]
    np.testing.assert_array_equal(_x_reciprocal(v, step), _x_division(v, step))


def test_reciprocal_digits_at_rounding_ties_and_edges():
    """Quotients at and next to half-integers (rint ties), the extremes +-RANGE, zero, subnormal values and
    subnormal steps."""
    rng = np.random.default_rng(11)
    step = (rng.random(4096) * 2.0 ** rng.integers(-100, 100, 4096)).astype(np.float32)
    step = step[step > 0]
    half = (rng.integers(-8355710, 8355710, step.size) + 0.5).astype(np.float64)
    v = (half * step.astype(np.float64)).astype(np.float32)
    cases_v = [v, np.nextafter(v, np.float32(np.inf)), np.nextafter(v, np.float32(-np.inf)),
               (RANGE * step).astype(np.float32), (-RANGE * step).astype(np.float32), np.zeros_like(step)]
    for cv in cases_v:
        ok = np.isfinite(cv)
        np.testing.assert_array_equal(_x_reciprocal(cv[ok], step[ok]), _x_division(cv[ok], step[ok]))
    tiny = np.array([1.4e-45, 2.8e-45, 1e-40, 1.17e-38], dtype=np.float32)
    for s in tiny:
        sv = np.full(1000, s, np.float32)
        vv = (np.linspace(-1.0, 1.0, 1000) * float(s) * 8355710.0).astype(np.float32)
        ok = np.isfinite(vv)
        np.testing.assert_array_equal(_x_reciprocal(vv[ok], sv[ok]), _x_division(vv[ok], sv[ok]))
