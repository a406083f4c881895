"""frc_costmodel_measure on the GPU: the cost model a planner weighs this
backend with, measured on the loaded blocks (bytes = blocks x (10 x burst x
slice + shared slice), src/bench.c:157-160)."""
import numpy as np
import pytest

import fronk_b200 as fb
from tests.helpers import make_layers

pytestmark = pytest.mark.gpu
SEED = 0x5EED


def test_costmodel_measure(gpu):
    hidden, blocks = 2048, [1, 6, 13]
    g = fb.geometry(hidden)
    with fb.Context(0, hidden) as ctx:
        assert ctx.costmodel()[0] == fb.STATE                       # nothing loaded
        for b, arr in make_layers(g, SEED, blocks, np.arange(512), shared=True).items():
            assert ctx.load_layer(b, 0, arr) == fb.OK, ctx.last_error
        rc, m = ctx.costmodel(layer=0, burst_max=4, samples=5)
        assert rc == fb.OK, ctx.last_error
        sb, hb = fb.slice_bytes(g), fb.shared_bytes(g)
        assert [m.bytes[b] for b in range(4)] == [len(blocks) * (10 * (b + 1) * sb + hb) for b in range(4)]
        assert m.burst_max == 4 and m.t0_ns >= 0 and np.isfinite(m.bw_eff) and m.bw_eff > 0
        assert all(np.isfinite(m.ns[b]) and m.ns[b] > 0 for b in range(4))
        print("cost model: t0 %.1f us, bw_eff %.1f GB/s, ns %s" % (m.t0_ns / 1e3, m.bw_eff / 1e9, list(m.ns)[:4]))
        # the fp32-activation mode is measured in its own arithmetic (the cuda-f32 table's fit)
        rc, m32 = ctx.costmodel(layer=0, burst_max=2, samples=3, act=fb.ACT_F32)
        assert rc == fb.OK and m32.burst_max == 2 and all(m32.ns[b] > 0 for b in range(2))
        assert ctx.costmodel(layer=0, burst_max=2, samples=3, act=7)[0] == fb.INVALID
