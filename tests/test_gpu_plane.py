"""The in-box head plane on the GPU (frc_plane_*): the sum of every
participant's part of the fp16-rounded request, in participant order, the
parts of participants after the first (remote nodes in the reference)
rounded through fp16 as the reference sends them; a deadline leaves the late
parts out and reports them, and their device status is kept apart; an x
without a finite fp16 form runs nothing.  Two contexts on one device stand in for two GPUs
(each context has its own stream and scratch)."""
import numpy as np
import pytest

import fronk_b200 as fb
from tests.helpers import make_layers, request

pytestmark = pytest.mark.gpu
SEED = 0x5EED


def _contexts(hidden, shares, e, layer):
    g = fb.geometry(hidden)
    ctxs = []
    for blocks in shares:
        c = fb.Context(0, hidden)
        for b, arr in make_layers(g, SEED, blocks, e, shared=True).items():
            assert c.load_layer(b, layer, arr) == fb.OK, c.last_error
        ctxs.append(c)
    return ctxs


def test_plane_sums_parts_in_order(gpu):
    hidden, layer = 2048, 4
    e, gate, x = request(hidden, 3, SEED + 950, 0.4)
    ctxs = _contexts(hidden, [[0, 3, 11], [7, 19]], e, layer)
    try:
        rc, xr = fb.round_half(x)
        assert rc == fb.OK
        parts = []
        for c in ctxs:
            rc, part = c.run(layer, e, gate, xr, fb.ACT_Q8)
            assert rc == fb.OK, c.last_error
            parts.append(part)
        rc, remote = fb.round_half(parts[1])   # participant 1's part crosses the wire as fp16
        assert rc == fb.OK
        want = (np.float32(0) + parts[0]) + remote
        with fb.Plane(ctxs) as plane:
            for _ in range(2):
                rc, y, missing = plane.run(layer, e, gate, x)
                assert rc == fb.OK and missing == 0
                assert np.array_equal(y.view(np.uint32), want.view(np.uint32))
            # a deadline that passes at once: the late parts are left out and reported
            rc, y, missing = plane.run(layer, e, gate, x, deadline_ns=1)
            assert rc == fb.OK
            expect = np.zeros_like(want)
            for i, part in enumerate((parts[0], remote)):
                if not missing >> i & 1:
                    expect = expect + part
            assert np.array_equal(y.view(np.uint32), expect.view(np.uint32))
            # the next call waits for the late parts, then is whole again; the
            # late parts' own status is kept apart (no device error here)
            rc, y, missing = plane.run(layer, e, gate, x)
            assert rc == fb.OK and missing == 0
            assert np.array_equal(y.view(np.uint32), want.view(np.uint32))
            assert [plane.late_status(i) for i in range(2)] == [fb.OK, fb.OK]
            # no finite fp16 form: nothing runs, y untouched
            bad = x.copy()
            bad[1, 5] = 70000.0
            out = np.full_like(want, 7.0)
            rc, y, _ = plane.run(layer, e, gate, bad, out=out)
            assert rc == fb.INVALID and np.all(out == 7.0)
    finally:
        for c in ctxs:
            c.close()
