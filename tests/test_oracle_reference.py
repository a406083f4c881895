"""Pins the oracle to the unmodified reference, compiled here from its own
sources: or_ref_run must equal fr_ref / fr_ref_q8 bit for bit (d = 2560 and the
d = 2048 mirror build), and must reproduce the reference's committed golden
vectors (tests/vectors/*.txt, legacy Q4_0 layout).  Skipped where the
reference was not compiled (the GPU host has only the prebuilt libraries)."""
import ctypes
import os

import numpy as np
import pytest

import fronk_b200 as fb
from oracle import OK, Q4_K, MXFP4, Q8_0, Reference, reference_available
from tests.helpers import SparseUnit, make_layers, request, conforms, BACKEND_TOL

# the reference's source tree: FRONK_REFERENCE, else a checkout beside this repository
REF_TREE = os.environ.get("FRONK_REFERENCE") or os.path.normpath(
    os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "..", "reference"))
needs_ref = pytest.mark.skipif(not reference_available(2560) or not reference_available(2048),
                               reason="reference not compiled here")

SEED = 0x5EED


def _units(ref, g, layer, blocks, experts):
    """Sparse full-size units holding the given experts (and the shared one)."""
    layers = make_layers(g, SEED, blocks, experts, shared=True)
    lb = fb.layer_bytes(g)
    units = {}
    for b, arr in layers.items():
        u = SparseUnit(ref.unit_bytes())
        u.write(layer * lb, arr)
        units[b] = u
    return units, layers


@needs_ref
@pytest.mark.parametrize("hidden", [2560, 2048])
def test_ref_run_matches_reference_bitwise(oracle, hidden):
    ref = Reference(hidden)
    g = fb.geometry(hidden)
    layer, blocks = 47, [0, 7, 19]
    cases = []
    for burst in (1, 3, 8):
        for distinct in (True, False):
            for shared in (0.0, 0.5):
                cases.append(request(hidden, burst, SEED + burst * 7 + distinct, shared, distinct))
    experts = np.concatenate([c[0].ravel() for c in cases])
    units, layers = _units(ref, g, layer, blocks, experts)
    backs = {name: ref.backend(name) for name in ("ref", "ref-q8")}
    for name, be in backs.items():
        for b, u in units.items():
            assert be.load(b, u.addr, ref.unit_bytes()) == OK
    m = oracle.model(hidden, Q4_K, MXFP4, layers)
    try:
        for (e, gt, x) in cases:
            req = ref.request(layer, e, gt, x)
            for name, q8 in (("ref", 0), ("ref-q8", 1)):
                rc, y_ref = ref.run(backs[name], req)
                rc2, y = oracle.ref_run(m, e, gt, x, q8)
                assert rc == OK and rc2 == OK
                assert np.array_equal(y.view(np.uint32), y_ref.view(np.uint32)), (name, x.shape)
    finally:
        for be in backs.values():
            for b in units:
                be.unload(b)
        for u in units.values():
            u.close()


@needs_ref
def test_port_matches_ref_q8(oracle):
    """The GPU's Q8 arithmetic (integer block dots of v and of the dequantized
    values' rounding residuals, exact block terms summed in double) gives the
    reference's own narrowed gate/up values, so it stays within 1e-5 of the
    compiled ref-q8, and within the frozen backend tolerance of ref
    (src/backend.c:11-13)."""
    hidden = 2560
    ref = Reference(hidden)
    g = fb.geometry(hidden)
    layer, blocks = 3, [1, 2, 5, 11]
    e, gt, x = request(hidden, 8, SEED + 99, 0.5)
    units, layers = _units(ref, g, layer, blocks, e)
    m = oracle.model(hidden, Q4_K, MXFP4, layers)
    backs = {name: ref.backend(name) for name in ("ref", "ref-q8")}
    try:
        for be in backs.values():
            for b, u in units.items():
                assert be.load(b, u.addr, ref.unit_bytes()) == OK
        req = ref.request(layer, e, gt, x)
        _, y_ref = ref.run(backs["ref"], req)
        _, y_q8 = ref.run(backs["ref-q8"], req)
        rc, y, _ = oracle.port_run(m, e, gt, x)
        assert rc == OK
        for t in range(8):
            assert conforms(oracle.compare(y_ref[t], y[t])[1], BACKEND_TOL)
            rel = oracle.compare(y_q8[t], y[t])[1][0]
            assert rel <= 1e-5, (t, rel)
    finally:
        for be in backs.values():
            for b in units:
                be.unload(b)
        for u in units.values():
            u.close()


class _Vector(ctypes.Structure):
    pass


@needs_ref
def test_legacy_golden_vectors(oracle):
    """The reference's own golden corpus (tests/vectors, README: ref at 1e-6)
    reproduced by the oracle's legacy Q4_0 path."""
    vec_dir = os.path.join(REF_TREE, "tests", "vectors")
    if not os.path.isdir(vec_dir):
        pytest.skip("reference vectors not present")
    ref = Reference(2560)

    class Vector(ctypes.Structure):
        _fields_ = [("name", ctypes.c_char_p), ("mask", ctypes.c_uint32), ("req", ref.Req),
                    ("data", ctypes.c_void_p * 20), ("digest", ctypes.c_char * 65)]

    ref.L.fr_vector_open.argtypes = [ctypes.c_uint, ctypes.c_void_p]
    ref.L.fr_vector_close.argtypes = [ctypes.c_void_p]
    legacy_layer = oracle.L.or_legacy_layer_bytes(2560)
    for index in range(8):
        v = Vector()
        assert ref.L.fr_vector_open(index, ctypes.byref(v)) == OK
        try:
            name = v.name.decode()
            with open(os.path.join(vec_dir, name + ".txt")) as f:
                head = f.readline().split()
                golden = np.array([float.fromhex(t) for t in f.read().split()], np.float32)
            burst, layer = v.req.burst, v.req.layer
            assert int(head[3]) == burst and golden.size == burst * 2560
            golden = golden.reshape(burst, 2560)
            m = oracle.model(2560, 0, 0, {}, legacy=1)
            for b in range(20):
                if v.data[b]:
                    m.layer[b] = v.data[b] + layer * legacy_layer
            e = np.ctypeslib.as_array(v.req.expert)[:burst]
            gt = np.ctypeslib.as_array(v.req.gate)[:burst]
            x = np.ctypeslib.as_array(v.req.x)[:burst]
            rc, y = oracle.ref_run(m, e, gt, x, 0)
            assert rc == OK
            # the golden text holds exact fp32 values printed with %a
            assert np.array_equal(y.view(np.uint32), golden.view(np.uint32)), name
        finally:
            ref.L.fr_vector_close(ctypes.byref(v))


def _scaled_groups(x, rng):
    """Spreads the 64-groups of x over many binades (subnormal to 1e30
    scales), so the dequantization residuals take every width."""
    x = x.copy()
    for t in range(x.shape[0]):
        for p in range(x.shape[1] // 64):
            x[t, 64 * p:64 * p + 64] *= np.float32(10.0 ** rng.integers(-40, 8))
    return x


@pytest.mark.parametrize("hidden,gt,dt", [(2048, Q4_K, MXFP4), (2560, Q4_K, MXFP4), (2048, MXFP4, Q8_0),
                                          (2048, Q8_0, MXFP4)])
def test_port_matches_ref_q8_oracle(oracle, hidden, gt, dt):
    """Runs without the compiled reference: or_ref_run (q8=1) is ref-q8 bit for
    bit (test_ref_run_matches_reference_bitwise), and the GPU arithmetic
    restated by or_port_run stays within 1e-5 of it per token, shared expert
    and reused experts included, also with activation groups spread from
    subnormal to large scales."""
    g = fb.geometry(hidden, 48, gt, dt)
    rng = np.random.default_rng(hidden + gt)
    cases = [request(hidden, t, SEED + 31 * t + int(4 * sh), sh, True) for t in (1, 3, 8) for sh in (0.0, 0.5)]
    cases.append(request(hidden, 16, SEED + 5, 0.25, False))
    e16, g16, x16 = request(hidden, 4, SEED + 6, 0.5)
    cases.append((e16, g16, _scaled_groups(x16, rng)))
    experts = np.concatenate([c[0].ravel() for c in cases])
    layers = make_layers(g, SEED + 1, [0, 5, 13], experts, shared=True)
    m = oracle.model(hidden, gt, dt, layers)
    for e, gate, x in cases:
        rc, y_q8 = oracle.ref_run(m, e, gate, x, 1)
        rc2, y, _ = oracle.port_run(m, e, gate, x)
        assert rc == OK and rc2 == OK
        for t in range(x.shape[0]):
            rel = oracle.compare(y_q8[t], y[t])[1][0]
            assert rel <= 1e-5, (t, rel)
