"""CUDA path against the oracle, through the C ABI (frc_* in libfronk_b200.so).

Bar: bit-exact for activation quantization, block unpacking, integer block
dots and the hidden activations; output within relative L2 1e-5 per token of
the oracle port and of the reference's ref-q8 (or_ref_run q8, pinned to the
reference bit for bit).  fp32-activation mode
within 1e-5 of the reference's "ref" arithmetic (or_ref_run, pinned to the
reference bit for bit)."""
import numpy as np
import pytest

import fronk_b200 as fb
from oracle import Q4_K, MXFP4, Q8_0, OK, NUMERIC, INVALID, STATE
from tests.helpers import make_layers, request, rel_l2

pytestmark = pytest.mark.gpu
SEED = 0x5EED
TOL = 1e-5          # relative L2 per token (north star)


def _rows(type_, n, count, rng):
    rb = fb.row_bytes(type_, n)
    rows = rng.integers(0, 256, (count, rb)).astype(np.uint8)
    if type_ == Q4_K:
        for r in rows:
            r[1::144] &= 0x3b   # finite fp16 d and dmin (exponent < 31)
            r[3::144] &= 0x3b
    elif type_ == MXFP4:
        rows[:, ::17] = rng.integers(0, 255, (count, n // 32))
    else:
        rows[:, 1::34] &= 0x3b
    return rows


@pytest.mark.parametrize("type_", [Q4_K, MXFP4, Q8_0])
def test_decode_bit_exact(gpu, oracle, type_):
    rng = np.random.default_rng(type_)
    n = 2560
    rows = _rows(type_, n, 24, rng)
    if type_ == MXFP4:
        rows[0, ::17] = 0          # E8M0 zero exponent: 2^-127 subnormal
        rows[1, 0] = 255           # reserved exponent: nonfinite
    with fb.Context(0, 2048) as ctx:
        w = ctx.debug_decode(type_, rows, n, rows.shape[0])
    for i, r in enumerate(rows):
        rc, ref = oracle.decode_row(r, type_, n)
        fin = np.isfinite(ref)
        assert np.array_equal(np.isfinite(w[i]), fin)
        assert np.array_equal(w[i][fin].view(np.uint32), ref[fin].view(np.uint32)), i


def test_activation_quantization_bit_exact(gpu, oracle):
    rng = np.random.default_rng(1)
    d = 2048
    x = np.zeros((6, d), np.float32)
    for t in range(6):
        x[t] = rng.standard_normal(d) * 10.0 ** rng.integers(-20, 20)
    x[0, :64] = np.round(x[0, :64]) + 0.5          # ties
    x[1, :64] = 0                                   # zero group
    x[1, 64] = np.finfo(np.float32).max             # FLT_MAX group
    x[2, 128] = np.float32(2 ** -149)               # scale underflows
    x[3, 192] = np.float32(2 ** -125)               # reciprocal overflows
    with fb.Context(0, d) as ctx:
        q, s, deq = ctx.debug_quantize(x)
    for t in range(6):
        rc, qr, sr = oracle.q8_quantize(x[t])
        rc2, dr = oracle.q8_activation(x[t])
        assert rc == OK and rc2 == OK
        assert np.array_equal(q[t], qr)
        assert np.array_equal(s[t].view(np.uint32), sr.view(np.uint32))
        assert np.array_equal(deq[t].view(np.uint32), dr.view(np.uint32))


CONFIGS = [(2048, Q4_K, MXFP4), (2560, Q4_K, MXFP4), (2048, MXFP4, Q8_0), (2048, Q8_0, MXFP4)]


def _setup(ctx, g, blocks, experts, layer):
    layers = make_layers(g, SEED, blocks, experts, shared=True)
    for b, arr in layers.items():
        assert ctx.load_layer(b, layer, arr) == OK, ctx.last_error
    return layers


@pytest.mark.parametrize("hidden,gt,dt", CONFIGS)
def test_layer_q8_matches_oracle(gpu, oracle, hidden, gt, dt):
    g = fb.geometry(hidden, 48, gt, dt)
    blocks, layer = [0, 3, 7, 12, 19], 30
    cases = [request(hidden, t, SEED + 13 * t + int(sh * 4), sh, True) for t in (1, 2, 5, 16) for sh in (0.0, 0.5)]
    cases.append(request(hidden, 8, SEED + 1, 0.25, False))      # reused experts
    experts = np.concatenate([c[0].ravel() for c in cases])
    with fb.Context(0, hidden, 48, gt, dt) as ctx:
        layers = _setup(ctx, g, blocks, experts, layer)
        m = oracle.model(hidden, gt, dt, layers)
        for e, gate, x in cases:
            rc, y = ctx.run(layer, e, gate, x, fb.ACT_Q8)
            assert rc == OK, ctx.last_error
            h = ctx.debug_hidden()
            rc, y_ref, h_ref = oracle.port_run(m, e, gate, x, want_hidden=True)
            assert rc == OK
            assert np.array_equal(h.view(np.uint32), h_ref.view(np.uint32)), "hidden activations"
            errs = [rel_l2(r, a) for r, a in zip(y_ref, y)]
            assert max(errs) <= TOL, errs
            rc, y_q8 = oracle.ref_run(m, e, gate, x, 1)   # the reference's ref-q8, bit for bit
            assert rc == OK
            errs = [rel_l2(r, a) for r, a in zip(y_q8, y)]
            assert max(errs) <= TOL, ("vs ref-q8", errs)


def test_layer_q8_all_twenty_slices(gpu, oracle):
    hidden = 2048
    g = fb.geometry(hidden)
    e, gate, x = request(hidden, 4, SEED + 77, 0.0)
    with fb.Context(0, hidden) as ctx:
        layers = _setup(ctx, g, list(range(20)), e, 0)
        rc, y = ctx.run(0, e, gate, x, fb.ACT_Q8)
        assert rc == OK, ctx.last_error
        rc, y_ref, _ = oracle.port_run(oracle.model(hidden, Q4_K, MXFP4, layers), e, gate, x)
        assert max(rel_l2(r, a) for r, a in zip(y_ref, y)) <= TOL


def test_grid_sizes_alternate_on_one_context(gpu, oracle):
    """16 tokens launch one CTA an SM, one token two: alternating them on one
    context, an odd number of each in a row, keeps the grid barrier whole
    and the results right."""
    hidden = 2048
    g = fb.geometry(hidden)
    cases = [request(hidden, t, SEED + 500 + i, 0.0) for i, t in enumerate((16, 1, 1, 16, 16, 1, 16, 1))]
    experts = np.concatenate([c[0].ravel() for c in cases])
    with fb.Context(0, hidden) as ctx:
        layers = _setup(ctx, g, list(range(20)), experts, 2)
        m = oracle.model(hidden, Q4_K, MXFP4, layers)
        for e, gate, x in cases:
            rc, y = ctx.run(2, e, gate, x, fb.ACT_Q8)
            assert rc == OK, ctx.last_error
            rc, y_ref, _ = oracle.port_run(m, e, gate, x)
            assert rc == OK
            assert max(rel_l2(r, a) for r, a in zip(y_ref, y)) <= TOL


@pytest.mark.parametrize("hidden,gt,dt", CONFIGS)
def test_layer_f32_matches_reference_arithmetic(gpu, oracle, hidden, gt, dt):
    g = fb.geometry(hidden, 48, gt, dt)
    blocks, layer = [1, 4, 18], 2
    cases = [request(hidden, t, SEED + 5 * t, sh, True) for t in (1, 3, 8) for sh in (0.0, 0.5)]
    experts = np.concatenate([c[0].ravel() for c in cases])
    with fb.Context(0, hidden, 48, gt, dt) as ctx:
        layers = _setup(ctx, g, blocks, experts, layer)
        m = oracle.model(hidden, gt, dt, layers)
        for e, gate, x in cases:
            rc, y = ctx.run(layer, e, gate, x, fb.ACT_F32)
            assert rc == OK, ctx.last_error
            rc, y_ref = oracle.ref_run(m, e, gate, x, 0)
            assert rc == OK
            errs = [rel_l2(r, a) for r, a in zip(y_ref, y)]
            assert max(errs) <= TOL, errs


def test_burst_equals_single_tokens_and_repeats(gpu):
    hidden = 2048
    g = fb.geometry(hidden)
    e, gate, x = request(hidden, 8, SEED + 3, 0.5)
    with fb.Context(0, hidden) as ctx:
        _setup(ctx, g, [2, 6, 11], e, 9)
        for act in (fb.ACT_Q8, fb.ACT_F32):
            rc, y = ctx.run(9, e, gate, x, act)
            assert rc == OK
            rc, y2 = ctx.run(9, e, gate, x, act)
            assert np.array_equal(y.view(np.uint32), y2.view(np.uint32)), "repeat"
            for t in range(8):
                rc, yt = ctx.run(9, e[t:t + 1], gate[t:t + 1], x[t:t + 1], act)
                assert rc == OK
                assert np.array_equal(yt[0].view(np.uint32), y[t].view(np.uint32)), (act, t)


def test_sharded_blocks_sum_to_whole(gpu):
    hidden = 2048
    g = fb.geometry(hidden)
    e, gate, x = request(hidden, 3, SEED + 4, 0.0)
    layers = make_layers(g, SEED, list(range(8)), e, shared=False)
    parts = []
    for shard in ([0, 1, 2], [3, 4, 5, 6, 7]):
        with fb.Context(0, hidden) as ctx:
            for b in shard:
                assert ctx.load_layer(b, 1, layers[b]) == OK
            rc, y = ctx.run(1, e, gate, x, fb.ACT_F32)
            assert rc == OK
            parts.append(y)
    with fb.Context(0, hidden) as ctx:
        for b in range(8):
            assert ctx.load_layer(b, 1, layers[b]) == OK
        rc, whole = ctx.run(1, e, gate, x, fb.ACT_F32)
    assert max(rel_l2(w, s) for w, s in zip(whole, parts[0] + parts[1])) <= 1e-6


def test_failures_leave_output_untouched(gpu):
    hidden = 2048
    g = fb.geometry(hidden)
    e, gate, x = request(hidden, 2, SEED + 8, 0.5)
    with fb.Context(0, hidden) as ctx:
        sentinel = np.full((2, hidden), 7.0, np.float32)
        rc, y = ctx.run(0, e, gate, x, fb.ACT_Q8, out=sentinel.copy())
        assert rc == STATE and np.array_equal(y, sentinel), "nothing loaded"
        layers = make_layers(g, SEED, [4], e, shared=True)
        arr = layers[4]
        assert ctx.load_layer(4, 0, arr) == OK
        assert ctx.load_layer(4, 0, arr) == STATE
        rc, y = ctx.run(1, e, gate, x, fb.ACT_Q8, out=sentinel.copy())
        assert rc == STATE and np.array_equal(y, sentinel), "layer not loaded"
        for bad_e, bad_g, bad_x, code in (
                (np.where(np.arange(10) == 3, 512, e), gate, x, INVALID),              # id out of range
                (np.concatenate([e[:, :1], e[:, :9]], 1), gate, x, INVALID),            # duplicate id
                (e, np.where(np.arange(11) == 2, -1.0, gate).astype(np.float32), x, INVALID),
                (e, np.where(np.arange(11) == 2, np.nan, gate).astype(np.float32), x, NUMERIC),
                (e, gate, np.where(np.arange(hidden) == 5, np.inf, x).astype(np.float32), NUMERIC),
                (e, gate, np.full_like(x, np.finfo(np.float32).max), NUMERIC)):
            for act in (fb.ACT_Q8, fb.ACT_F32):
                rc, y = ctx.run(0, bad_e, bad_g, bad_x, act, out=sentinel.copy())
                assert rc == code and np.array_equal(y, sentinel), (code, act)
    sb = fb.slice_bytes(g)
    for offset, value in ((int(e[0, 0]) * sb + 1, 0x7C),                                # Q4_K d = inf
                          (int(e[0, 0]) * sb + 2 * 32 * fb.row_bytes(Q4_K, hidden), 255),  # MXFP4 e = 255
                          (512 * sb + 1, 0x7C)):                                          # shared Q8_0 d
        bad = make_layers(g, SEED, [4], e, shared=True)[4]
        bad[offset] = value
        with fb.Context(0, hidden) as ctx:
            assert ctx.load_layer(4, 0, bad) == OK
            for act in (fb.ACT_Q8, fb.ACT_F32):
                rc, y = ctx.run(0, e, gate, x, act, out=sentinel.copy())
                assert rc == NUMERIC and np.array_equal(y, sentinel), (offset, act)


@pytest.mark.parametrize("tokens", [1, 3])
def test_host_pass_equals_layer_by_layer_runs(gpu, tokens):
    """frc_host_pass (the C layer loop over frc_run) against the same chain
    driven call by call from Python: identical residual stream."""
    hidden, layers = 2048, 3
    g = fb.geometry(hidden)
    routes = [request(hidden, tokens, SEED + 300 + l, 0.3 if l == 1 else 0.0) for l in range(layers)]
    experts = np.concatenate([r[0].ravel() for r in routes])
    with fb.Context(0, hidden) as ctx:
        lay = make_layers(g, SEED, [2, 9], experts, shared=True)
        for l in range(layers):
            for b, arr in lay.items():
                assert ctx.load_layer(b, l, arr) == OK, ctx.last_error
        h0 = routes[0][2].astype(np.float32)
        h = h0.copy()
        for l in range(layers):
            ss = np.sum(h.astype(np.float64) ** 2, axis=1, keepdims=True)
            inv = (1.0 / np.sqrt(ss / hidden + 1e-6)).astype(np.float32)
            x = (h * inv).astype(np.float32)
            rc, y = ctx.run(l, routes[l][0], routes[l][1], x, fb.ACT_Q8)
            assert rc == OK, ctx.last_error
            h = (h + y).astype(np.float32)
        hp = h0.copy() if tokens > 1 else h0[0].copy()
        ctx.host_pass(0, np.stack([r[0] for r in routes]) if tokens > 1 else np.concatenate([r[0] for r in routes]),
                      np.stack([r[1] for r in routes]) if tokens > 1 else np.concatenate([r[1] for r in routes]), hp)
        assert np.array_equal(hp.reshape(h.shape).view(np.uint32), h.view(np.uint32))
