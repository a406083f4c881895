"""tcgen05 kind::i8 building block: the shared-memory descriptors, the
instruction descriptor and the tensor-memory read-back of frc_umma.cuh,
against an exact integer matrix product."""
import numpy as np
import pytest

import fronk_b200 as fb

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n,k", [(16, 32), (64, 256), (256, 256), (48, 96), (256, 32)])
def test_umma_i8_matches_integer_product(gpu, n, k):
    rng = np.random.default_rng(1000 * n + k)
    a = rng.integers(-127, 128, size=(128, k), dtype=np.int64)
    b = rng.integers(-127, 128, size=(n, k), dtype=np.int64)
    with fb.Context(0, 2048) as ctx:
        d = ctx.debug_umma(a.astype(np.int8), b.astype(np.int8))
    assert np.array_equal(d.astype(np.int64), a @ b.T)


def test_umma_i8_extremes(gpu):
    a = np.full((128, 256), -127, np.int8)
    b = np.full((64, 256), -127, np.int8)
    a[::2] = 127
    with fb.Context(0, 2048) as ctx:
        d = ctx.debug_umma(a, b)
    want = a.astype(np.int64) @ b.astype(np.int64).T
    assert np.array_equal(d.astype(np.int64), want)
