"""Pins or_avx2_run, the CPU restatement of the reference's AVX2 backend
(backends/avx2.c: int8 activations per 256 with int16 sums per 32, its fp32
lane order, jobs dealt round robin to the workers), to the unmodified backend
compiled here from its own sources: bit for bit at the same worker count
(fr_avx2_set_tuning + fr_avx2_configure fix it), d = 2560 and the d = 2048
mirror build.  With the correctly rounded exp of the CUDA mode instead of the
C library's expf the outputs stay within 1e-6.  Skipped where the reference
was not compiled (the GPU host has only the prebuilt libraries)."""
import numpy as np
import pytest

import fronk_b200 as fb
from oracle import OK, Q4_K, MXFP4, Reference, reference_available
from tests.helpers import SparseUnit, make_layers, request

SEED = 0xA5A5
needs_ref = pytest.mark.skipif(not reference_available(2560) or not reference_available(2048),
                               reason="reference not compiled here")


def _configure(ref, blocks, workers):
    assert ref.configure_avx2(blocks, workers) == OK


@needs_ref
@pytest.mark.parametrize("hidden", [2560, 2048])
def test_avx2_restatement_matches_backend_bitwise(oracle, hidden):
    ref = Reference(hidden)
    g = fb.geometry(hidden)
    layer, blocks = 29, [2, 5, 13]
    cases = []
    for burst in (1, 3, 8):
        for distinct in (True, False):
            for shared in (0.0, 0.5):
                cases.append(request(hidden, burst, SEED + burst * 13 + distinct, shared, distinct))
    experts = np.concatenate([c[0].ravel() for c in cases])
    layers = make_layers(g, SEED, blocks, experts, shared=True)
    lb = fb.layer_bytes(g)
    units = {}
    for b, arr in layers.items():
        u = SparseUnit(ref.unit_bytes())
        u.write(layer * lb, arr)
        units[b] = u
    m = oracle.model(hidden, Q4_K, MXFP4, layers)
    be = ref.backend("avx2")
    try:
        for workers in (1, 3):
            _configure(ref, len(blocks), workers)
            for b in blocks:  # ascending: the backend's job order follows load order
                assert be.load(b, units[b].addr, ref.unit_bytes()) == OK
            try:
                for (e, gt, x) in cases:
                    rc, y_ref = ref.run(be, ref.request(layer, e, gt, x))
                    rc2, y = oracle.avx2_run(m, e, gt, x, workers=workers, libm_expf=True)
                    assert rc == OK and rc2 == OK
                    assert np.array_equal(y.view(np.uint32), y_ref.view(np.uint32)), (workers, x.shape)
                    # the CUDA mode's exp: equal but for the C library's rare
                    # last-bit expf roundings
                    rc3, y_cr = oracle.avx2_run(m, e, gt, x, workers=workers, libm_expf=False)
                    assert rc3 == OK
                    for t in range(x.shape[0]):
                        assert oracle.compare(y_ref[t], y_cr[t])[1][0] <= 1e-6
            finally:
                for b in blocks:
                    be.unload(b)
    finally:
        for u in units.values():
            u.close()


@needs_ref
def test_avx2_restatement_worker_sweep(oracle):
    """Seeded sweep of worker counts (up to 16), bursts and shared gates at
    d = 2048: the restatement equals the compiled backend bit for bit in
    every case, at the worker count the backend's engine actually runs
    (fr_avx2_configure leaves the host one logical CPU)."""
    hidden = 2048
    ref = Reference(hidden)
    g = fb.geometry(hidden)
    layer, blocks = 17, [0, 4, 9, 19]
    rng = np.random.default_rng(SEED)
    cases = [(int(rng.integers(1, 9)), float(rng.choice([0.0, 0.3])), bool(rng.integers(0, 2)), int(seed))
             for seed in rng.integers(1, 1 << 30, size=8)]
    reqs = [request(hidden, t, s, sh, distinct) for t, sh, distinct, s in cases]
    experts = np.concatenate([r[0].ravel() for r in reqs])
    layers = make_layers(g, SEED + 1, blocks, experts, shared=True)
    units = {}
    for b, arr in layers.items():
        u = SparseUnit(ref.unit_bytes())
        u.write(layer * fb.layer_bytes(g), arr)
        units[b] = u
    m = oracle.model(hidden, Q4_K, MXFP4, layers)
    be = ref.backend("avx2")
    try:
        for workers in (2, 4, 5, 7, 8, 16):
            _configure(ref, len(blocks), workers)
            for b in blocks:
                assert be.load(b, units[b].addr, ref.unit_bytes()) == OK
            engine = ref.avx2_engine_workers()
            assert 1 <= engine <= workers
            try:
                for e, gt, x in reqs:
                    rc, y_ref = ref.run(be, ref.request(layer, e, gt, x))
                    rc2, y = oracle.avx2_run(m, e, gt, x, workers=engine, libm_expf=True)
                    assert rc == rc2 == OK
                    assert np.array_equal(y.view(np.uint32), y_ref.view(np.uint32)), (workers, engine, x.shape)
            finally:
                for b in blocks:
                    be.unload(b)
    finally:
        for u in units.values():
            u.close()


@needs_ref
def test_avx2_restatement_follows_load_order(oracle):
    """The backend deals jobs over its blocks in load order; after an unload
    the remaining blocks are ascending again (backends/avx2.c:602-613)."""
    hidden = 2048
    ref = Reference(hidden)
    g = fb.geometry(hidden)
    layer, order = 6, [13, 2, 5]
    e, gt, x = request(hidden, 3, SEED + 21, 0.5)
    layers = make_layers(g, SEED, order, e, shared=True)
    units = {}
    for b, arr in layers.items():
        u = SparseUnit(ref.unit_bytes())
        u.write(layer * fb.layer_bytes(g), arr)
        units[b] = u
    be = ref.backend("avx2")
    try:
        _configure(ref, len(order), 2)
        for b in order:
            assert be.load(b, units[b].addr, ref.unit_bytes()) == OK
        rc, y_ref = ref.run(be, ref.request(layer, e, gt, x))
        m = oracle.model(hidden, Q4_K, MXFP4, layers)
        rc2, y = oracle.avx2_run(m, e, gt, x, workers=2, order=order)
        _, y_asc = oracle.avx2_run(m, e, gt, x, workers=2)
        assert rc == rc2 == OK and np.array_equal(y.view(np.uint32), y_ref.view(np.uint32))
        assert not np.array_equal(y_asc.view(np.uint32), y_ref.view(np.uint32))  # the order is visible
        be.unload(2)
        rest = {13: layers[13], 5: layers[5]}
        rc, y_ref = ref.run(be, ref.request(layer, e, gt, x))
        rc2, y = oracle.avx2_run(oracle.model(hidden, Q4_K, MXFP4, rest), e, gt, x, workers=2)
        assert rc == rc2 == OK and np.array_equal(y.view(np.uint32), y_ref.view(np.uint32))
    finally:
        for b in (13, 5):
            be.unload(b)
        for u in units.values():
            u.close()


@needs_ref
def test_avx2_restatement_numeric_cases(oracle):
    """A nonfinite Q8_0 scale of the shared expert and a reserved MXFP4
    exponent in a routed down row are NUMERIC in both."""
    hidden = 2048
    ref = Reference(hidden)
    g = fb.geometry(hidden)
    layer, blocks = 4, [1]
    e, gt, x = request(hidden, 2, SEED + 7, 0.5)
    layers = make_layers(g, SEED, blocks, e, shared=True)
    sb = fb.slice_bytes(g)
    for corrupt in ("shared_down_scale", "routed_down_exp"):
        arr = layers[1].copy()
        if corrupt == "shared_down_scale":
            off = 512 * sb + 2 * (hidden * 34) + 5 * 34   # shared down row 5, fp16 scale
            arr[off:off + 2] = (0x00, 0x7C)                # +inf
        else:
            eid = int(e[0, 0])
            off = eid * sb + 2 * 32 * fb.row_bytes(Q4_K, hidden) + 9 * 17  # routed down row 9
            arr[off] = 255
        u = SparseUnit(ref.unit_bytes())
        u.write(layer * fb.layer_bytes(g), arr)
        be = ref.backend("avx2")
        _configure(ref, 1, 2)
        try:
            assert be.load(1, u.addr, ref.unit_bytes()) == OK
            rc, _ = ref.run(be, ref.request(layer, e, gt, x))
            be.unload(1)
            m = oracle.model(hidden, Q4_K, MXFP4, {1: arr})
            rc2, _ = oracle.avx2_run(m, e, gt, x, workers=2)
            assert rc == rc2 == -3, (corrupt, rc, rc2)
        finally:
            u.close()
