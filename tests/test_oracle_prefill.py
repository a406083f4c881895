"""The prefill arithmetic of the oracle (or_prefill_run): pinned through the
reference restatement (or_ref_run, itself bit-identical to the compiled
reference) and checked for the properties the GPU path relies on."""
import numpy as np
import pytest

import fronk_b200 as fb
from oracle import Oracle, MXFP4, Q8_0, OK, INVALID, NUMERIC
from tests.helpers import make_layers, request, BACKEND_TOL, conforms

SEED = 0x5EED


@pytest.fixture(scope="module")
def oracle():
    return Oracle()


def _model(oracle, down, blocks, e, hidden=2048):
    g = fb.geometry(hidden, gate_type=MXFP4, down_type=down)
    layers = make_layers(g, SEED, blocks, e, shared=False)
    return oracle.model(hidden, MXFP4, down, layers), layers, g


@pytest.mark.parametrize("down", [MXFP4, Q8_0])
@pytest.mark.parametrize("hidden", [2048, 2560])
def test_prefill_matches_ref_q8(oracle, down, hidden):
    """Against the reference's ref-q8 (or_ref_run q8, bit-identical to the
    compiled fr_ref_q8) on the same units: within 1e-5 per token (the exact
    block terms of the gate/up dots give the reference's own narrowed values,
    so the hidden slices round alike), and within the backend conformance
    limits of ref (src/backend.c:11-13)."""
    e, gt, x = request(hidden, 16, SEED + 5 + hidden)
    m, layers, _ = _model(oracle, down, [0, 3, 7], e, hidden)  # m points into layers: keep them alive
    rc, y, _, _ = oracle.prefill_run(m, e, gt, x)
    assert rc == OK
    rc, y_ref = oracle.ref_run(m, e, gt, x, 0)
    assert rc == OK
    rc, y_q8 = oracle.ref_run(m, e, gt, x, 1)
    assert rc == OK
    for t in range(16):
        assert conforms(oracle.compare(y_ref[t], y[t])[1], BACKEND_TOL)
        rel = oracle.compare(y_q8[t], y[t])[1][0]
        assert rel <= 1e-5, (t, rel)


def test_prefill_tokens_are_independent(oracle):
    """A token's result depends only on its own row: any subset of the burst
    gives the same bits (what lets full-size runs be checked on a sample)."""
    e, gt, x = request(2048, 24, SEED + 6)
    m, layers, _ = _model(oracle, MXFP4, [1, 2], e)
    rc, y, hq, hs = oracle.prefill_run(m, e, gt, x, want_hidden=True)
    assert rc == OK and hq.shape == (240, 2, 32) and hs.shape == (240, 2)
    sub = [3, 4, 17, 23]
    rc, ys, _, _ = oracle.prefill_run(m, e[sub], gt[sub], x[sub])
    assert rc == OK
    assert np.array_equal(ys.view(np.uint32), y[sub].view(np.uint32))


def test_prefill_rejects_shared_expert_and_bad_scales(oracle):
    e, gt, x = request(2048, 20, SEED + 7)
    m, layers, g = _model(oracle, MXFP4, [4], e)
    gs = gt.copy()
    gs[5, 10] = 0.25
    assert oracle.prefill_run(m, e, gs, x)[0] == INVALID
    # E8M0 exponent 255 in the first block of gate row 0 of a referenced slice
    layers[4][int(e[0, 0]) * fb.slice_bytes(g)] = 255
    assert oracle.prefill_run(m, e, gt, x)[0] == NUMERIC
