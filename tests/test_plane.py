"""The in-box head plane's host rule without a GPU: x goes through fp16 the
way the reference head sends it (src/plane.c:258-262, src/wire.c:46-67):
round to nearest even, and a value with no finite fp16 form is refused."""
import numpy as np

import fronk_b200 as fb


def test_round_half_matches_ieee_fp16(built):
    rng = np.random.default_rng(11)
    x = np.concatenate([
        rng.normal(0, 1, 20000), rng.normal(0, 3000, 20000), rng.uniform(-1e-4, 1e-4, 20000),
        rng.uniform(-65519.9, 65519.9, 5000),
        [0.0, -0.0, 2.0 ** -24, 2.0 ** -25, 1.5 * 2.0 ** -25, 2.0 ** -14, 65504.0, 65519.0, -65519.99, 1e-30],
    ]).astype(np.float32)
    rc, y = fb.round_half(x)
    assert rc == fb.OK
    want = x.astype(np.float16).astype(np.float32)
    assert np.array_equal(y.view(np.uint32), want.view(np.uint32))


def test_round_half_refuses_values_without_a_finite_half(built):
    for bad in (65520.0, -65520.0, 1e6, np.inf, -np.inf, np.nan):
        rc, _ = fb.round_half(np.array([1.0, bad, 2.0], np.float32))
        assert rc == fb.INVALID, bad
