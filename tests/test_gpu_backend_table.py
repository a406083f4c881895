"""The drop-in plugin tables fr_cuda ("cuda", Q8 activations), fr_cuda_f32
("cuda-f32") and fr_cuda_avx2 ("cuda-avx2", the AVX2 backend's arithmetic,
against fr_avx2 at the same worker count) driven through their function
pointers, as the reference's
registry and node call a backend (src/backend.h:52-67), with the reference
compiled from its own sources loaded into the same process
(oracle/_ref/libfronk_ref.so, RTLD_GLOBAL): probe; load of full-size sparse
units (d = 2560, FR_NATIVE_BLOCK_BYTES each); run against the reference's
fr_ref / fr_ref_q8 on the same requests; the untouched-output rule on a bad
request; unload; and self_test, which runs the reference's own conformance
check fr_native_self_test (src/native.c:66-135; backends/user-template.c:96-98)
on the table."""
import ctypes

import numpy as np
import pytest

import fronk_b200 as fb
from oracle import OK, INVALID, STATE, Reference, reference_available
from tests.helpers import SparseUnit, make_layers, request, rel_l2

pytestmark = pytest.mark.gpu
SEED = 0x5EED
TOL = 1e-5
needs_ref = pytest.mark.skipif(not reference_available(2560), reason="reference library not built")


def _table(ref, name):
    return ref.Backend.in_dll(fb.library(), name)


@needs_ref
@pytest.mark.parametrize("name,ref_name", [("fr_cuda", "ref-q8"), ("fr_cuda_f32", "ref"), ("fr_cuda_avx2", "avx2")])
def test_table_against_reference(gpu, name, ref_name):
    ref = Reference(2560)
    be, rb = _table(ref, name), ref.backend(ref_name)
    if name == "fr_cuda_avx2":  # both at two workers: the same job dealing and summation order
        assert ref.configure_avx2(2, 2) == OK
        assert fb.library().fr_cuda_avx2_workers(2) == OK
    hw = ref.Hw()
    assert be.probe(ctypes.byref(hw)) == OK
    assert b"B200" in hw.gpu or b"sm_100" in hw.gpu, hw.gpu
    g = fb.geometry(2560)
    layer, blocks = 11, [2, 17]
    cases = [request(2560, t, SEED + 40 + t, sh, True) for t in (1, 3, 8) for sh in (0.0, 0.5)]
    experts = np.concatenate([c[0].ravel() for c in cases])
    layers = make_layers(g, SEED, blocks, experts, shared=True)
    units = {}
    try:
        for b, arr in layers.items():
            u = SparseUnit(ref.unit_bytes())
            u.write(layer * fb.layer_bytes(g), arr)
            units[b] = u
            assert be.load(b, u.addr, ref.unit_bytes()) == OK
            assert be.load(b, u.addr, ref.unit_bytes()) == STATE          # occupied slot
            assert rb.load(b, u.addr, ref.unit_bytes()) == OK
        for e, gate, x in cases:
            req = ref.request(layer, e, gate, x)
            rc, y_ref = ref.run(rb, req)
            rc2, y = ref.run(be, req)
            assert rc == OK and rc2 == OK
            errs = [rel_l2(r, a) for r, a in zip(y_ref, y)]
            assert max(errs) <= TOL, (name, errs)
        # a request the reference rejects leaves the output byte-identical
        e, gate, x = cases[2]
        bad = ref.request(layer, np.where(np.arange(10) == 4, 512, e).astype(np.uint16), gate, x)
        part = ref.Part()
        ctypes.memset(ctypes.addressof(part), 0x5A, ctypes.sizeof(part))
        before = bytes(memoryview(part))
        assert be.run(ctypes.byref(bad), ctypes.byref(part)) == INVALID
        assert bytes(memoryview(part)) == before
        assert be.self_test(None) == STATE                                # blocks loaded
    finally:
        for b in units:
            be.unload(b)
            rb.unload(b)
        for u in units.values():
            u.close()
    assert be.unload(blocks[0]) == STATE                                   # empty slot
    # the reference's own conformance check on the table (loads block 19 of
    # a fixture unit, bursts 1-8 distinct and reused, the shared expert, and
    # three corrupted scales that must fail with the output untouched)
    assert be.self_test(None) == OK
