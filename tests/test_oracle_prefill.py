"""The prefill arithmetic of the oracle (or_prefill_run): pinned through the
reference restatement (or_ref_run, itself bit-identical to the compiled
reference) and checked for the properties the GPU path relies on."""
import numpy as np
import pytest

import fronk_b200 as fb
from oracle import Oracle, MXFP4, Q8_0, Q4_K, OK, INVALID, NUMERIC
from tests.helpers import make_layers, request, BACKEND_TOL, conforms

SEED = 0x5EED


@pytest.fixture(scope="module")
def oracle():
    return Oracle()


def _model(oracle, down, blocks, e, hidden=2048, gate=MXFP4):
    g = fb.geometry(hidden, gate_type=gate, down_type=down)
    layers = make_layers(g, SEED, blocks, e, shared=False)
    return oracle.model(hidden, gate, down, layers), layers, g


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


def test_prefill_rejects_bad_gates_and_scales(oracle):
    e, gt, x = request(2048, 20, SEED + 7)
    m, layers, g = _model(oracle, MXFP4, [4], e)
    gs = gt.copy()
    gs[5, 10] = -0.25  # a negative (shared) gate
    assert oracle.prefill_run(m, e, gs, x)[0] == INVALID
    # E8M0 exponent 255 in the first block of gate row 0 of a referenced slice
    layers[4][int(e[0, 0]) * fb.slice_bytes(g)] = 255
    assert oracle.prefill_run(m, e, gt, x)[0] == NUMERIC


@pytest.mark.parametrize("hidden", [2048, 2560])
def test_prefill_q4k_gate_up_matches_ref_q8(oracle, hidden):
    """The reference's own unit layout (Q4_K gate/up, MXFP4 down): the exact
    per-group terms (M*K1 + K3) * d * 2^E - (M*K2 + K4) * dmin * 2^E give
    y within 1e-5 of ref-q8 per token, and within the conformance limits of
    ref."""
    e, gt, x = request(hidden, 16, SEED + 9 + hidden)
    m, layers, _ = _model(oracle, MXFP4, [0, 4, 9], e, hidden, gate=Q4_K)
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


def test_prefill_q4k_nonfinite_super_block_scale_is_numeric(oracle):
    """A nonfinite d of any super-block of a referenced Q4_K row is NUMERIC,
    whatever the gate (the reference's rule for every referenced scale)."""
    e, gt, x = request(2048, 20, SEED + 12)
    g = fb.geometry(2048, gate_type=Q4_K, down_type=MXFP4)
    layers = make_layers(g, SEED, [2], e, shared=False)
    bad = layers[2].copy()
    # fp16 d = inf (0x7c00) of super-block 3 of up row 5 of a referenced slice
    off = int(e[4, 1]) * fb.slice_bytes(g) + (32 + 5) * fb.row_bytes(Q4_K, 2048) + 3 * 144
    bad[off:off + 2] = [0x00, 0x7c]
    m = oracle.model(2048, Q4_K, MXFP4, {2: bad})
    rc, _, _, _ = oracle.prefill_run(m, e, gt, x)
    assert rc == NUMERIC


@pytest.mark.parametrize("gate_type", [MXFP4, Q4_K])
def test_prefill_shared_expert_matches_ref_q8(oracle, gate_type):
    """The Q8_0 shared expert inside a burst (the reference's units always
    carry it): its pairs follow the routed ones, its Q8_0 block terms are
    exact integers times d * 2^E, and it is added after the token's routed
    experts; y within 1e-5 of ref-q8 per token."""
    e, gt, x = request(2048, 16, SEED + 33, shared_gate=0.4)
    gt[3, 10] = 0.0  # a token without the shared expert
    g = fb.geometry(2048, gate_type=gate_type, down_type=MXFP4)
    layers = make_layers(g, SEED, [0, 5, 11], e, shared=True)
    m = oracle.model(2048, gate_type, MXFP4, layers)
    rc, y, hq, hs = oracle.prefill_run(m, e, gt, x, want_hidden=True)
    assert rc == OK
    assert hq.shape[0] == 16 * 10 + 15
    rc, y_q8 = oracle.ref_run(m, e, gt, x, 1)
    assert rc == OK
    for t in range(16):
        assert oracle.compare(y_q8[t], y[t])[1][0] <= 1e-5, t
