"""frc_units_open on the GPU: a unit directory (unit-BB.bin + unit-BB.sha256)
loads the same weights as frc_load_unit of the same bytes, bit for bit in
the outputs, and a digest mismatch or an occupied block loads nothing."""
import hashlib

import numpy as np
import pytest

import fronk_b200 as fb
from tests.helpers import make_layers, request

pytestmark = pytest.mark.gpu
SEED = 0x5EED


def test_units_open_equals_load_unit(gpu, tmp_path):
    hidden, blocks = 2048, [2, 7]
    g = fb.geometry(hidden, 1)
    e, gate, x = request(hidden, 3, SEED + 900, 0.0)
    layers = make_layers(g, SEED, blocks, e, shared=False)   # one layer: a layer is the whole unit
    for b, arr in layers.items():
        assert arr.nbytes == fb.unit_bytes(g)
        (tmp_path / ("unit-%02u.bin" % b)).write_bytes(arr.tobytes())
        (tmp_path / ("unit-%02u.sha256" % b)).write_bytes(hashlib.sha256(arr.tobytes()).hexdigest().encode() + b"\n")
    mask = sum(1 << b for b in blocks)
    with fb.Context(0, hidden, 1) as ctx:
        assert ctx.units_open(str(tmp_path), mask) == fb.OK, ctx.last_error
        assert ctx.loaded_mask() == mask
        rc, y = ctx.run(0, e, gate, x, fb.ACT_Q8)
        assert rc == fb.OK, ctx.last_error
        assert ctx.units_open(str(tmp_path), 1 << 2) == fb.STATE   # occupied block
        assert ctx.loaded_mask() == mask
    with fb.Context(0, hidden, 1) as ctx:
        for b, arr in layers.items():
            assert ctx.load_unit(b, arr) == fb.OK
        rc, y2 = ctx.run(0, e, gate, x, fb.ACT_Q8)
        assert rc == fb.OK
    assert np.array_equal(y.view(np.uint32), y2.view(np.uint32))


def test_units_open_mismatch_loads_nothing(gpu, tmp_path):
    hidden = 2048
    g = fb.geometry(hidden, 1)
    e, _, _ = request(hidden, 1, SEED + 901, 0.0)
    arr = make_layers(g, SEED, [4, 9], e, shared=False)
    for b, a in arr.items():
        (tmp_path / ("unit-%02u.bin" % b)).write_bytes(a.tobytes())
        digest = hashlib.sha256(a.tobytes()).hexdigest()
        if b == 9:
            digest = ("0" if digest[0] != "0" else "1") + digest[1:]
        (tmp_path / ("unit-%02u.sha256" % b)).write_bytes(digest.encode() + b"\n")
    with fb.Context(0, hidden, 1) as ctx:
        rc = ctx.units_open(str(tmp_path), (1 << 4) | (1 << 9))
        assert rc == fb.MISMATCH and "SHA-256" in ctx.last_error
        assert ctx.loaded_mask() == 0                               # block 4 was unloaded again
        assert ctx.units_open(str(tmp_path), 1 << 4) == fb.OK
        assert ctx.loaded_mask() == 1 << 4
