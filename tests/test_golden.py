"""Parity against the committed golden outputs of the reference's own "ref"
and "ref-q8" backends and of its AVX2 backend with one and four workers
(tests/golden/native_ref.npz, written by tests/golden/make_golden.py from the
reference compiled from its sources).
These pin the native Q4_K + MXFP4 path where the reference itself is absent:
the oracle bit for bit on the CPU, the CUDA path on the GPU."""
import hashlib
import os

import numpy as np
import pytest

import fronk_b200 as fb
from oracle import OK, Q4_K, MXFP4
from tests.helpers import make_layers, rel_l2, conforms, BACKEND_TOL

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "native_ref.npz")
TOL = 1e-5          # fp32 mode vs "ref", Q8 mode vs "ref-q8": relative L2 per token


def _load():
    return np.load(GOLDEN)


def _cases(z, hidden):
    out = []
    for i in range(len(z["cases"])):
        k = "d%d_c%d_" % (hidden, i)
        out.append((z[k + "expert"], z[k + "gate"], z[k + "x"], z[k + "y_ref"], z[k + "y_ref_q8"]))
    return out


def _layers(z, hidden):
    g = fb.geometry(hidden)
    cases = _cases(z, hidden)
    experts = np.concatenate([c[0].ravel() for c in cases])
    layers = make_layers(g, int(z["seed"]), [int(b) for b in z["blocks"]], experts, shared=True)
    h = hashlib.sha256()
    for b in sorted(layers):
        h.update(np.ascontiguousarray(layers[b]).tobytes())
    assert h.hexdigest() == str(z["d%d_weights_sha256" % hidden]), "synthetic weights differ from the golden run"
    return g, layers, cases


@pytest.mark.parametrize("hidden", [2560, 2048])
def test_oracle_reproduces_reference_goldens(oracle, hidden):
    z = _load()
    _, layers, cases = _layers(z, hidden)
    m = oracle.model(hidden, Q4_K, MXFP4, layers)
    for e, gt, x, y_ref, y_q8 in cases:
        rc, y = oracle.ref_run(m, e, gt, x, 0)
        assert rc == OK and np.array_equal(y.view(np.uint32), y_ref.view(np.uint32))
        rc, y = oracle.ref_run(m, e, gt, x, 1)
        assert rc == OK and np.array_equal(y.view(np.uint32), y_q8.view(np.uint32))


@pytest.mark.parametrize("hidden", [2560, 2048])
def test_oracle_reproduces_avx2_goldens(oracle, hidden):
    """or_avx2_run with the C library's expf is the AVX2 backend bit for bit
    at its worker count."""
    z = _load()
    _, layers, cases = _layers(z, hidden)
    m = oracle.model(hidden, Q4_K, MXFP4, layers)
    for i, (e, gt, x, _, _) in enumerate(cases):
        for workers in (1, 4):
            rc, y = oracle.avx2_run(m, e, gt, x, workers=workers, libm_expf=True)
            want = z["d%d_c%d_y_avx2_w%d" % (hidden, i, workers)]
            assert rc == OK and np.array_equal(y.view(np.uint32), want.view(np.uint32)), (i, workers)


@pytest.mark.gpu
@pytest.mark.parametrize("hidden", [2560, 2048])
def test_cuda_matches_reference_goldens(gpu, oracle, hidden):
    z = _load()
    g, layers, cases = _layers(z, hidden)
    layer = int(z["layer"])
    with fb.Context(0, hidden) as ctx:
        for b, arr in layers.items():
            assert ctx.load_layer(b, layer, arr) == OK, ctx.last_error
        for e, gt, x, y_ref, y_q8 in cases:
            rc, y = ctx.run(layer, e, gt, x, fb.ACT_F32)
            assert rc == OK, ctx.last_error
            errs = [rel_l2(r, a) for r, a in zip(y_ref, y)]
            assert max(errs) <= TOL, errs
            rc, y = ctx.run(layer, e, gt, x, fb.ACT_Q8)
            assert rc == OK, ctx.last_error
            for t in range(len(y)):
                assert rel_l2(y_q8[t], y[t]) <= TOL, (t, rel_l2(y_q8[t], y[t]))
                assert conforms(oracle.compare(y_ref[t], y[t])[1], BACKEND_TOL)
