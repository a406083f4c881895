"""Generates tests/golden/native_ref.npz: outputs of the reference's own
"ref" and "ref-q8" backends (backends/ref.c) and of its AVX2 backend
(backends/avx2.c) with one and with four workers, all compiled from the
reference's sources into oracle/_ref by oracle/build.py, on seeded
native-format units.

The reference commits golden vectors only for its legacy Q4_0 layout
(tests/vectors); these fixtures pin the native Q4_K + MXFP4 path at the
reference geometry (d = 2560) and at the d = 2048 mirror build, so that
parity is checked against the reference where the reference is not present
(the GPU host).  The weights are not stored: they are regenerated from the
seeds by the library's own encoders (frc_synth_slice, via
tests/helpers.make_layers) and checked against the stored sha256.

Run from the repository root, where the reference has been compiled:
    python tests/golden/make_golden.py
"""
import hashlib
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import fronk_b200 as fb  # noqa: E402
from oracle import OK, Reference  # noqa: E402
from tests.helpers import SparseUnit, make_layers, request  # noqa: E402

SEED = 0x5EED
LAYER = 11
BLOCKS = [0, 7, 19]
CASES = [(1, 0.0), (2, 0.5), (3, 0.25)]  # (tokens, shared-expert gate)
OUT = os.path.join(ROOT, "tests", "golden", "native_ref.npz")


def weights_digest(layers):
    h = hashlib.sha256()
    for b in sorted(layers):
        h.update(np.ascontiguousarray(layers[b]).tobytes())
    return h.hexdigest()


def cases_for(hidden):
    return [request(hidden, t, SEED + 31 * t + hidden, sh, True) for t, sh in CASES]


def generate(hidden):
    ref = Reference(hidden)
    g = fb.geometry(hidden)
    cases = cases_for(hidden)
    experts = np.concatenate([c[0].ravel() for c in cases])
    layers = make_layers(g, SEED, BLOCKS, experts, shared=True)
    lb = fb.layer_bytes(g)
    units = {}
    for b, arr in layers.items():
        u = SparseUnit(ref.unit_bytes())
        u.write(LAYER * lb, arr)
        units[b] = u
    backs = {name: ref.backend(name) for name in ("ref", "ref-q8")}
    out = {}
    try:
        for be in backs.values():
            for b, u in units.items():
                assert be.load(b, u.addr, ref.unit_bytes()) == OK
        for i, (e, gt, x) in enumerate(cases):
            req = ref.request(LAYER, e, gt, x)
            for name, key in (("ref", "y_ref"), ("ref-q8", "y_ref_q8")):
                rc, y = ref.run(backs[name], req)
                assert rc == OK, (name, rc)
                out["d%d_c%d_%s" % (hidden, i, key)] = y
            out["d%d_c%d_expert" % (hidden, i)] = e
            out["d%d_c%d_gate" % (hidden, i)] = gt
            out["d%d_c%d_x" % (hidden, i)] = x
    finally:
        for be in backs.values():
            for b in units:
                be.unload(b)
    avx2 = ref.backend("avx2")
    try:
        for workers in (1, 4):
            assert ref.configure_avx2(len(BLOCKS), workers) == OK
            for b in BLOCKS:  # ascending: the backend's job order follows load order
                assert avx2.load(b, units[b].addr, ref.unit_bytes()) == OK
            # fr_avx2_configure leaves the host one logical CPU: the engine
            # must run the worker count the fixture is named for
            assert ref.avx2_engine_workers() == workers, "host too small for %d AVX2 workers" % workers
            try:
                for i, (e, gt, x) in enumerate(cases):
                    rc, y = ref.run(avx2, ref.request(LAYER, e, gt, x))
                    assert rc == OK, ("avx2", workers, rc)
                    out["d%d_c%d_y_avx2_w%d" % (hidden, i, workers)] = y
            finally:
                for b in BLOCKS:
                    avx2.unload(b)
    finally:
        for u in units.values():
            u.close()
    out["d%d_weights_sha256" % hidden] = np.array(weights_digest(layers))
    return out


def main():
    data = {"layer": np.array(LAYER), "blocks": np.array(BLOCKS), "seed": np.array(SEED),
            "cases": np.array(CASES)}
    for hidden in (2560, 2048):
        data.update(generate(hidden))
    np.savez_compressed(OUT, **data)
    print("wrote", OUT, os.path.getsize(OUT), "bytes")


if __name__ == "__main__":
    main()
