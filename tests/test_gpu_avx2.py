"""FRC_ACT_AVX2 on the GPU: the arithmetic of the reference's AVX2 backend
(backends/avx2.c).  Bit for bit against the oracle's restatement with the
same exp form (or_avx2_run, libm_expf=False) at several worker counts and
block load orders; against the AVX2 backend's own committed outputs
(tests/golden/native_ref.npz, one and four workers) bit for bit wherever the
C library's expf and the correctly rounded exp agree on the case, and within
1e-6 otherwise; NUMERIC for nonfinite scales with y untouched; refusals of
the forms it does not take."""
import numpy as np
import pytest

import fronk_b200 as fb
from oracle import OK, Q4_K, MXFP4
from tests.helpers import make_layers, request, rel_l2
from tests.test_golden import _load, _layers

pytestmark = pytest.mark.gpu
SEED = 0xA5A5


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("hidden", [2560, 2048])
def test_avx2_mode_matches_restatement_bitwise(gpu, oracle, hidden):
    g = fb.geometry(hidden)
    layer, blocks = 29, [2, 5, 13]
    cases = []
    for burst in (1, 3, 8, 16):
        for distinct in (True, False):
            for shared in (0.0, 0.5):
                cases.append(request(hidden, burst, SEED + burst * 13 + distinct, shared, distinct))
    experts = np.concatenate([c[0].ravel() for c in cases])
    layers = make_layers(g, SEED, blocks, experts, shared=True)
    m = oracle.model(hidden, Q4_K, MXFP4, layers)
    with fb.Context(0, hidden) as ctx:
        for b in blocks:
            assert ctx.load_layer(b, layer, layers[b]) == OK, ctx.last_error
        for workers in (1, 3, 8):
            ctx.set_avx2_workers(workers)
            for e, gt, x in cases:
                rc, y = ctx.run(layer, e, gt, x, fb.ACT_AVX2)
                assert rc == OK, ctx.last_error
                rc2, want = oracle.avx2_run(m, e, gt, x, workers=workers, libm_expf=False)
                assert rc2 == OK
                same = _bits(y) == _bits(want)
                assert same.all(), (workers, x.shape, int((~same).sum()))


@pytest.mark.parametrize("hidden", [2560, 2048])
def test_avx2_mode_against_backend_goldens(gpu, oracle, hidden):
    """The AVX2 backend's own outputs: equal bit for bit where its expf and
    the correctly rounded exp give the same case, within 1e-6 everywhere."""
    z = _load()
    g, layers, cases = _layers(z, hidden)
    layer = int(z["layer"])
    m = oracle.model(hidden, Q4_K, MXFP4, layers)
    exact = 0
    with fb.Context(0, hidden) as ctx:
        for b in sorted(layers):
            assert ctx.load_layer(b, layer, layers[b]) == OK, ctx.last_error
        for workers in (1, 4):
            ctx.set_avx2_workers(workers)
            for i, (e, gt, x, _, _) in enumerate(cases):
                want = z["d%d_c%d_y_avx2_w%d" % (hidden, i, workers)]
                rc, y = ctx.run(layer, e, gt, x, fb.ACT_AVX2)
                assert rc == OK, ctx.last_error
                for t in range(len(y)):
                    assert rel_l2(want[t], y[t]) <= 1e-6, (workers, i, t)
                _, libm = oracle.avx2_run(m, e, gt, x, workers=workers, libm_expf=True)
                _, cr = oracle.avx2_run(m, e, gt, x, workers=workers, libm_expf=False)
                if np.array_equal(_bits(libm), _bits(cr)):
                    assert np.array_equal(_bits(y), _bits(want)), (workers, i)
                    exact += 1
    assert exact >= 1


def test_avx2_mode_follows_load_order(gpu, oracle):
    hidden = 2048
    g = fb.geometry(hidden)
    layer, order = 6, [13, 2, 5]
    e, gt, x = request(hidden, 3, SEED + 21, 0.5)
    layers = make_layers(g, SEED, order, e, shared=True)
    with fb.Context(0, hidden) as ctx:
        for b in order:
            assert ctx.load_layer(b, layer, layers[b]) == OK, ctx.last_error
        ctx.set_avx2_workers(2)
        rc, y = ctx.run(layer, e, gt, x, fb.ACT_AVX2)
        _, want = oracle.avx2_run(oracle.model(hidden, Q4_K, MXFP4, layers), e, gt, x, workers=2,
                                  libm_expf=False, order=order)
        assert rc == OK and np.array_equal(_bits(y), _bits(want))
        ctx.unload(2)  # the remaining blocks are ascending again
        rc, y = ctx.run(layer, e, gt, x, fb.ACT_AVX2)
        rest = {13: layers[13], 5: layers[5]}
        _, want = oracle.avx2_run(oracle.model(hidden, Q4_K, MXFP4, rest), e, gt, x, workers=2, libm_expf=False)
        assert rc == OK and np.array_equal(_bits(y), _bits(want))


def test_avx2_mode_numeric_and_untouched(gpu, oracle):
    """A nonfinite Q8_0 scale of the shared expert (gate row or down row), a
    reserved MXFP4 exponent in a routed down row and a nonfinite Q4_K d are
    NUMERIC in the oracle and on the GPU; y stays untouched and the next
    clean call is exact."""
    hidden = 2048
    g = fb.geometry(hidden)
    layer = 4
    e, gt, x = request(hidden, 2, SEED + 7, 0.5)
    layers = make_layers(g, SEED, [1], e, shared=True)
    sb = fb.slice_bytes(g)
    rb = fb.row_bytes(Q4_K, hidden)
    eid = int(e[0, 0])
    corrupt = {
        "shared_down_scale": (512 * sb + 2 * (hidden * 34) + 5 * 34, (0x00, 0x7C)),
        "shared_gate_scale": (512 * sb + 3 * (hidden // 32 * 34) + 2 * 34, (0x00, 0x7C)),
        "routed_down_exp": (eid * sb + 2 * 32 * rb + 9 * 17, (255,)),
        "routed_gate_d": (eid * sb + 7 * rb + 144, (0x00, 0x7C)),
    }
    with fb.Context(0, hidden) as ctx:
        assert ctx.load_layer(1, layer, layers[1]) == OK, ctx.last_error
        for name, (off, val) in corrupt.items():
            arr = layers[1].copy()
            arr[off:off + len(val)] = val
            rc0, _ = oracle.avx2_run(oracle.model(hidden, Q4_K, MXFP4, {1: arr}), e, gt, x, libm_expf=False)
            assert rc0 == fb.NUMERIC, name
            assert ctx.refresh_layer(1, layer, arr) == OK, ctx.last_error
            out = np.full(x.shape, 7.25, np.float32)
            rc, _ = ctx.run(layer, e, gt, x, fb.ACT_AVX2, out=out)
            assert rc == fb.NUMERIC, (name, ctx.last_error)
            assert (out == 7.25).all(), name
        assert ctx.refresh_layer(1, layer, layers[1]) == OK
        rc, y = ctx.run(layer, e, gt, x, fb.ACT_AVX2)
        _, want = oracle.avx2_run(oracle.model(hidden, Q4_K, MXFP4, layers), e, gt, x, libm_expf=False)
        assert rc == OK and np.array_equal(_bits(y), _bits(want))


def test_avx2_mode_refusals(gpu):
    hidden = 2048
    e, gt, x = request(hidden, 1, SEED + 3, 0.0)
    with fb.Context(0, hidden, gate_type=fb.MXFP4) as ctx:   # not the reference's native layout
        ctx.load_layer(0, 0, np.zeros(fb.layer_bytes(fb.geometry(hidden, gate_type=fb.MXFP4)), np.uint8))
        rc, _ = ctx.run(0, e, gt, x, fb.ACT_AVX2)
        assert rc == fb.UNSUPPORTED
    g = fb.geometry(hidden)
    layers = make_layers(g, SEED, [0], e, shared=True)
    with fb.Context(0, hidden) as ctx:
        assert ctx.load_layer(0, 0, layers[0]) == OK
        rc, _ = ctx.run(0, e, gt, x, fb.ACT_AVX2, flags=fb.RUN_PEER)
        assert rc == fb.UNSUPPORTED
        with pytest.raises(fb.FrcError):
            ctx.set_avx2_workers(0)
        with pytest.raises(fb.FrcError):
            ctx.set_avx2_workers(33)
