"""Fixture builders shared by the tests: sparse layers and sparse reference units."""
import ctypes
import mmap

import numpy as np

import fronk_b200 as fb


def layer_keys(block, expert):
    return block * 1024 + expert


def make_layers(g, seed, blocks, experts, shared=True):
    """{block: uint8 array of one layer (reference layout)} with the given
    experts' slices (and the shared slice) filled; the rest stays zero."""
    lb, sb, hb = fb.layer_bytes(g), fb.slice_bytes(g), fb.shared_bytes(g)
    out = {}
    for b in blocks:
        arr = np.zeros(lb, np.uint8)
        for e in sorted(set(int(v) for v in np.asarray(experts).ravel())):
            arr[e * sb:(e + 1) * sb] = fb.synth_slice(g, seed, layer_keys(b, e))
        if shared:
            arr[512 * sb:512 * sb + hb] = fb.synth_shared(g, seed, layer_keys(b, 512))
        out[b] = arr
    return out


def request(hidden, tokens, seed, shared_gate=0.0, distinct=True):
    e, gt, x = fb.synth_request(hidden, tokens, seed)
    if not distinct and tokens > 1:
        e[1:] = e[0]          # every token uses the same ten experts
    gt[:, 10] = shared_gate
    return e, gt, x


class SparseUnit:
    """A full-size anonymous mapping (the reference's unit size); only the
    written pages are materialized (as src/native.c:66-75 does)."""

    def __init__(self, nbytes):
        self.mm = mmap.mmap(-1, nbytes, flags=mmap.MAP_PRIVATE | mmap.MAP_ANONYMOUS)
        self.nbytes = nbytes
        self.addr = ctypes.addressof(ctypes.c_char.from_buffer(self.mm))

    def write(self, offset, arr):
        self.mm[offset:offset + arr.nbytes] = arr.tobytes()

    def array(self):
        return np.frombuffer(self.mm, np.uint8)

    def close(self):
        try:
            self.mm.close()
        except BufferError:
            pass


def rel_l2(ref, act):
    ref = np.asarray(ref, np.float64)
    act = np.asarray(act, np.float64)
    den = np.sqrt((ref ** 2).sum())
    return float(np.sqrt(((act - ref) ** 2).sum()) / den) if den else float(np.abs(act).max())


def per_token_rel_l2(ref, act):
    return [rel_l2(r, a) for r, a in zip(ref, act)]


# The frozen backend conformance limits of src/backend.c:11-13.
BACKEND_TOL = (0.025, 0.030, 0.9998)
REFERENCE_TOL = (1e-6, 1e-6, 0.999999999999)


def conforms(metrics, tol):
    r, m, c = metrics
    return np.isfinite(r) and np.isfinite(m) and r <= tol[0] and m <= tol[1] and c >= tol[2]
