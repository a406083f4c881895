"""The cost model's fit without a GPU (frc_costmodel_fit, the reference's
least squares of src/bench.c:163-191): exact lines are recovered, a
negative intercept refits through the origin, bad inputs are refused."""
import numpy as np

import fronk_b200 as fb


def test_fit_recovers_an_exact_line(built):
    nbytes = np.array([2_000_000, 4_000_000, 6_000_000, 8_000_000], np.uint64)
    t0, bw = 12_000.0, 5.0e12
    ns = t0 + 1e9 * nbytes.astype(np.float64) / bw
    rc, m = fb.costmodel_fit(ns, nbytes)
    assert rc == fb.OK and m.burst_max == 4
    assert abs(m.t0_ns - t0) < 1e-6 * t0 and abs(m.bw_eff - bw) < 1e-9 * bw
    assert list(m.ns)[:4] == list(ns) and list(m.bytes)[:4] == list(nbytes)


def test_fit_matches_numpy_least_squares_and_clamps_t0(built):
    rng = np.random.default_rng(3)
    x = np.array([1e6, 3e6, 5e6], np.float64)
    ns = 5000 + x * 2e-4 * (1 + 0.05 * rng.standard_normal(3))
    rc, m = fb.costmodel_fit(ns, x.astype(np.uint64))
    slope, icpt = np.polyfit(x, ns, 1)
    if icpt >= 0:
        assert rc == fb.OK and abs(m.t0_ns - icpt) < 1e-6 * max(1.0, abs(icpt))
        assert abs(m.bw_eff - 1e9 / slope) < 1e-9 * m.bw_eff
    # a line whose least-squares intercept is negative: through the origin instead
    ns2 = np.array([100.0, 500.0, 900.0])
    rc, m = fb.costmodel_fit(ns2, x.astype(np.uint64))
    assert rc == fb.OK and m.t0_ns == 0.0
    assert abs(m.bw_eff - 1e9 / (np.dot(x, ns2) / np.dot(x, x))) < 1e-9 * m.bw_eff


def test_fit_refuses_bad_inputs(built):
    x = np.array([1, 2, 3], np.uint64)
    assert fb.costmodel_fit([5.0], [1])[0] == fb.INVALID
    assert fb.costmodel_fit([1.0, -2.0, 3.0], x)[0] == fb.NUMERIC
    assert fb.costmodel_fit([3.0, 2.0, 1.0], x)[0] == fb.NUMERIC        # time falls with bytes
    assert fb.costmodel_fit([1.0, np.nan, 3.0], x)[0] == fb.NUMERIC
