"""fronk_b200 - B200-native backend for Fronk's expert neuron-slice compute.

Python mirror of the C ABI in include/fronk_b200.h (ctypes).  The compute is
the in-tree CUDA library libfronk_b200.so; there is no CPU fallback: every
entry point raises when the library or an sm_100 device is missing.
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
# FRONK_B200_LIB selects another build (e.g. libfronk_b200_phases.so).
LIB_PATH = os.environ.get("FRONK_B200_LIB") or os.path.join(HERE, "libfronk_b200.so")

# src/backend.h:17-18
OK, INVALID, STATE, NUMERIC, IO, UNSUPPORTED, MISMATCH = 0, -1, -2, -3, -4, -5, -6
# src/native.h:8
Q8_0, Q4_K, MXFP4 = 8, 12, 39
ACT_F32, ACT_Q8, ACT_AVX2 = 0, 1, 2
RUN_RMSNORM = 1
RUN_OVERLAP = 2
RUN_PEER = 4
RUN_X_BF16 = 8
PEER_HANDLE_BYTES = 64
MAX_BLOCKS, ROUTED, SHARED, TOPK, ACTIVE, NEURONS, MAX_TOKENS = 20, 512, 512, 10, 11, 32, 16
MAX_PREFILL_TOKENS = 512
LAYERS = 48

_CODES = {OK: "OK", INVALID: "INVALID", STATE: "STATE", NUMERIC: "NUMERIC", IO: "IO",
          UNSUPPORTED: "UNSUPPORTED", MISMATCH: "MISMATCH"}


class FrcError(RuntimeError):
    def __init__(self, code, where, detail=""):
        self.code = code
        super().__init__("%s: %s (%d)%s" % (where, _CODES.get(code, "?"), code, ": " + detail if detail else ""))


class Geometry(ctypes.Structure):
    _fields_ = [("hidden", ctypes.c_uint32), ("layers", ctypes.c_uint32),
                ("gate_type", ctypes.c_uint32), ("down_type", ctypes.c_uint32)]

    def __repr__(self):
        return "Geometry(d=%d, layers=%d, gate=%d, down=%d)" % (self.hidden, self.layers, self.gate_type, self.down_type)


REFERENCE_GEOMETRY = (2560, LAYERS, Q4_K, MXFP4)   # src/model.h:16, src/native.h:1-3
BENCH_GEOMETRY = (2048, LAYERS, Q4_K, MXFP4)       # BASELINE configs[0] (down in MXFP4)

_lib = None
_vp, _u32, _u64, _sz, _int = ctypes.c_void_p, ctypes.c_uint, ctypes.c_uint64, ctypes.c_size_t, ctypes.c_int

_SIGS = {
    "frc_row_bytes": (_sz, [_u32, _u32]),
    "frc_slice_bytes": (_sz, [_vp]),
    "frc_shared_bytes": (_sz, [_vp]),
    "frc_layer_bytes": (_sz, [_vp]),
    "frc_unit_bytes": (_u64, [_vp]),
    "frc_slice_offset": (_u64, [_vp, _u32, _u32]),
    "frc_geometry_check": (_int, [_vp]),
    "frc_open": (_int, [_int, _vp, _vp]),
    "frc_close": (_int, [_vp]),
    "frc_load_unit": (_int, [_vp, _int, _vp, _sz]),
    "frc_load_layer": (_int, [_vp, _int, _u32, _vp, _sz]),
    "frc_refresh_layer": (_int, [_vp, _int, _u32, _vp, _sz]),
    "frc_probe_device": (_int, [_int, ctypes.c_char_p, _sz, _vp, _vp]),
    "frc_set_wait_limit": (_int, [_vp, _u64]),
    "frc_set_avx2_workers": (_int, [_vp, ctypes.c_uint]),
    "frc_avx2_timing": (_int, [_vp, _int]),
    "frc_avx2_times": (_int, [_vp, _vp]),
    "frc_debug_barrier_extra": (_int, [_vp, _u32]),
    "frc_debug_layer_variant": (_int, [_vp, _int]),
    "frc_unload_unit": (_int, [_vp, _int]),
    "frc_loaded_mask": (_int, [_vp, _vp]),
    "frc_units_open": (_int, [_vp, ctypes.c_char_p, _u32, _int]),
    "frc_unit_verify": (_int, [ctypes.c_char_p, _u32, _u64, _int]),
    "frc_sha256": (_int, [_vp, _sz, _vp]),
    "frc_plane_open": (_int, [_vp, _u32, _vp]),
    "frc_plane_run": (_int, [_vp, _u32, _u32, _vp, _vp, _vp, _u64, _vp, _vp]),
    "frc_plane_close": (_int, [_vp]),
    "frc_plane_late_status": (_int, [_vp, _u32, _vp]),
    "frc_round_half": (_int, [_vp, _sz, _vp]),
    "frc_costmodel_fit": (_int, [_vp, _vp, _u32, _vp]),
    "frc_costmodel_measure": (_int, [_vp, _vp, _u32, _u32, _u32, _int, _vp]),
    "frc_run": (_int, [_vp, _u32, _u32, _vp, _vp, _vp, _vp, _int]),
    "frc_run_device": (_int, [_vp, _u32, _u32, _vp, _vp, _vp, _vp, _vp, _vp, _int, _u32, _vp]),
    "frc_run_device_fixed": (_int, [_vp, _u32, _u32, _vp, _vp, _vp, _vp, _vp, _vp, _int, _u32, _vp]),
    "frc_host_pass": (_int, [_vp, _u32, _u32, _u32, _vp, _vp, _vp, _u32, _int]),
    "frc_host_pass_flags": (_int, [_vp, _u32, _u32, _u32, _vp, _vp, _vp, _u32, _int, _u32]),
    "frc_run_flags": (_int, [_vp, _u32, _u32, _vp, _vp, _vp, _vp, _int, _u32]),
    "frc_peer_export": (_int, [_vp, _u32, _vp]),
    "frc_peer_attach": (_int, [_vp, _u32, _u32, _vp]),
    "frc_peer_detach": (_int, [_vp]),
    "frc_status": (_int, [_vp, _vp]),
    "frc_launch_count": (_u64, [_vp]),
    "frc_strerror": (ctypes.c_char_p, [_int]),
    "frc_last_error": (ctypes.c_char_p, [_vp]),
    "frc_rand64": (_u64, [_u64, _u64]),
    "frc_normal": (ctypes.c_float, [_u64, _u64]),
    "frc_encode_row": (_int, [_u32, _vp, _u32, _vp]),
    "frc_synth_slice": (_int, [_vp, _u64, _u64, _vp]),
    "frc_synth_shared": (_int, [_vp, _u64, _u64, _vp]),
    "frc_synth_request_zipf": (_int, [_u32, _u32, _u64, ctypes.c_double, _vp, _vp, _vp]),
    "frc_synth_request": (_int, [_u32, _u32, _u64, _vp, _vp, _vp]),
    "frc_pool_load": (_int, [_vp, _vp, _u32, _vp]),
    "frc_fill_layer": (_int, [_vp, _int, _u32, _u64]),
    "frc_pool_pick": (_u32, [_u64, _u32, _u32, _u32, _u32]),
    "frc_debug_decode": (_int, [_vp, _u32, _vp, _u32, _u32, _vp]),
    "frc_debug_quantize": (_int, [_vp, _u32, _vp, _vp, _vp, _vp]),
    "frc_debug_hidden": (_int, [_vp, _vp, _sz, _vp]),
    "frc_debug_umma": (_int, [_vp, _u32, _u32, _vp, _vp, _vp]),
    "frc_debug_prefill_hidden": (_int, [_vp, _vp, _vp, _sz, _vp]),
    "frc_prefill_timing": (_int, [_vp, _int]),
    "frc_prefill_times": (_int, [_vp, _vp]),
    "frc_debug_phases": (_int, [_vp, _vp, _sz, _vp]),
}
EXPORTS = sorted(_SIGS) + ["fr_cuda", "fr_cuda_f32", "fr_cuda_avx2", "fr_cuda_select_device", "fr_cuda_close",
                          "fr_cuda_avx2_workers"]


def library():
    """The loaded libfronk_b200.so.  Raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FrcError(UNSUPPORTED, "library", "%s missing: run fronk_b200/build.py" % LIB_PATH)
        lib = ctypes.CDLL(LIB_PATH, mode=ctypes.RTLD_GLOBAL)
        for name, (res, args) in _SIGS.items():
            f = getattr(lib, name)
            f.restype, f.argtypes = res, args
        _lib = lib
    return _lib


def _ptr(a):
    return None if a is None else ctypes.c_void_p(a.ctypes.data)


def geometry(hidden=2048, layers=LAYERS, gate_type=Q4_K, down_type=MXFP4):
    g = Geometry(hidden, layers, gate_type, down_type)
    rc = library().frc_geometry_check(ctypes.byref(g))
    if rc:
        raise FrcError(rc, "geometry", repr(g))
    return g


def row_bytes(type_, n):
    return library().frc_row_bytes(type_, n)


def slice_bytes(g):
    return library().frc_slice_bytes(ctypes.byref(g))


def shared_bytes(g):
    return library().frc_shared_bytes(ctypes.byref(g))


def layer_bytes(g):
    return library().frc_layer_bytes(ctypes.byref(g))


def unit_bytes(g):
    return library().frc_unit_bytes(ctypes.byref(g))


def sha256(data):
    """SHA-256 (FIPS 180-4) of a bytes-like object, by the library's frc_sha256."""
    buf = np.frombuffer(bytes(data), np.uint8)
    out = np.zeros(32, np.uint8)
    rc = library().frc_sha256(_ptr(buf) if buf.size else None, buf.size, _ptr(out))
    if rc:
        raise FrcError(rc, "sha256", "")
    return out.tobytes()


class CostModel(ctypes.Structure):
    """frc_costmodel (the fields and meaning of the reference's fr_costmodel)."""
    _fields_ = [("burst_max", ctypes.c_uint), ("t0_ns", ctypes.c_double), ("bw_eff", ctypes.c_double),
                ("ns", ctypes.c_double * 8), ("bytes", ctypes.c_uint64 * 8)]


def costmodel_fit(ns, nbytes):
    """(rc, CostModel) of frc_costmodel_fit over bursts 1..len(ns)."""
    ns = np.ascontiguousarray(ns, np.float64)
    nbytes = np.ascontiguousarray(nbytes, np.uint64)
    m = CostModel()
    rc = library().frc_costmodel_fit(_ptr(ns), _ptr(nbytes), len(ns), ctypes.byref(m))
    return rc, m


def round_half(x):
    """(rc, x rounded through fp16 as the head sends it) of frc_round_half."""
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros_like(x)
    rc = library().frc_round_half(_ptr(x) if x.size else None, x.size, _ptr(out) if x.size else None)
    return rc, out


class Plane:
    """In-box head plane over contexts (frc_plane_*): one layer fanned out to
    every participant, the parts done by the deadline summed in order."""

    def __init__(self, contexts):
        self.lib = library()
        self.contexts = list(contexts)          # they must outlive the plane
        arr = (ctypes.c_void_p * len(self.contexts))(*[c.h.value for c in self.contexts])
        h = ctypes.c_void_p()
        rc = self.lib.frc_plane_open(arr, len(self.contexts), ctypes.byref(h))
        if rc:
            raise FrcError(rc, "plane_open")
        self.h = h
        self.hidden = self.contexts[0].hidden

    def run(self, layer, expert, gate, x, deadline_ns=2_000_000_000, out=None):
        """(rc, y, missing mask)."""
        expert = np.ascontiguousarray(expert, np.uint16)
        gate = np.ascontiguousarray(gate, np.float32)
        x = np.ascontiguousarray(x, np.float32)
        tokens = x.shape[0]
        y = out if out is not None else np.zeros((tokens, self.hidden), np.float32)
        m = ctypes.c_uint32()
        rc = self.lib.frc_plane_run(self.h, layer, tokens, _ptr(expert), _ptr(gate), _ptr(x), deadline_ns, _ptr(y),
                                    ctypes.byref(m))
        return rc, y, m.value

    def late_status(self, participant):
        """frc_plane_late_status: the device status of the participant's last part that missed its deadline."""
        st = ctypes.c_int()
        rc = self.lib.frc_plane_late_status(self.h, participant, ctypes.byref(st))
        if rc:
            raise FrcError(rc, "plane_late_status")
        return st.value

    def close(self):
        if self.h:
            self.lib.frc_plane_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def unit_verify(directory, block, unit_bytes=0, verify=True):
    """frc_unit_verify: the unit-file checks of one block without a device; returns the status code."""
    return library().frc_unit_verify(os.fsencode(directory), block, unit_bytes, 1 if verify else 0)


def slice_offset(g, layer, expert):
    return library().frc_slice_offset(ctypes.byref(g), layer, expert)


# ------------------------------------------------------------ synthetic data

def synth_slice(g, seed, key):
    out = np.zeros(slice_bytes(g), np.uint8)
    rc = library().frc_synth_slice(ctypes.byref(g), seed, key, _ptr(out))
    if rc:
        raise FrcError(rc, "synth_slice")
    return out


def synth_shared(g, seed, key):
    out = np.zeros(shared_bytes(g), np.uint8)
    rc = library().frc_synth_shared(ctypes.byref(g), seed, key, _ptr(out))
    if rc:
        raise FrcError(rc, "synth_shared")
    return out


def synth_request(hidden, tokens, seed, zipf=None):
    """(expert [T,10] u16, gate [T,11] f32, x [T,d] f32) of frc_synth_request
    (frc_synth_request_zipf with exponent `zipf`)."""
    e = np.zeros((tokens, TOPK), np.uint16)
    gt = np.zeros((tokens, ACTIVE), np.float32)
    x = np.zeros((tokens, hidden), np.float32)
    if zipf is None:
        rc = library().frc_synth_request(hidden, tokens, seed, _ptr(e), _ptr(gt), _ptr(x))
    else:
        rc = library().frc_synth_request_zipf(hidden, tokens, seed, float(zipf), _ptr(e), _ptr(gt), _ptr(x))
    if rc:
        raise FrcError(rc, "synth_request")
    return e, gt, x


def encode_row(type_, w):
    w = np.ascontiguousarray(w, np.float32)
    out = np.zeros(row_bytes(type_, w.size), np.uint8)
    rc = library().frc_encode_row(type_, _ptr(w), w.size, _ptr(out))
    if rc:
        raise FrcError(rc, "encode_row")
    return out


def pool_pick(seed, block, layer, expert, count):
    return library().frc_pool_pick(seed, block, layer, expert, count)


def rand64(seed, index):
    return library().frc_rand64(seed, index)


# ------------------------------------------------------------------ context

class Context:
    """One device context (frc_context): loaded units, scratch, streams."""

    def __init__(self, device=0, hidden=2048, layers=LAYERS, gate_type=Q4_K, down_type=MXFP4):
        self.lib = library()
        self.g = geometry(hidden, layers, gate_type, down_type)
        self.hidden = hidden
        h = ctypes.c_void_p()
        rc = self.lib.frc_open(device, ctypes.byref(self.g), ctypes.byref(h))
        if rc:
            raise FrcError(rc, "frc_open", "device %d" % device)
        self.h = h
        self.device = device

    def close(self):
        if self.h:
            self.lib.frc_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, rc, where):
        if rc:
            raise FrcError(rc, where, (self.lib.frc_last_error(self.h) or b"").decode())

    @property
    def last_error(self):
        return (self.lib.frc_last_error(self.h) or b"").decode()

    @property
    def launches(self):
        return self.lib.frc_launch_count(self.h)

    def load_unit(self, block, unit):
        return self.lib.frc_load_unit(self.h, block, _ptr(unit), unit.nbytes)

    def units_open(self, directory, mask, verify=True):
        """frc_units_open: load the blocks of `mask` from a unit directory
        (unit-BB.bin + unit-BB.sha256); returns the status code."""
        return self.lib.frc_units_open(self.h, os.fsencode(directory), mask, 1 if verify else 0)

    def costmodel(self, layer=0, burst_max=4, samples=15, act=ACT_Q8):
        """(rc, CostModel) of frc_costmodel_measure on this context."""
        m = CostModel()
        rc = self.lib.frc_costmodel_measure(self.h, ctypes.byref(self.g), layer, burst_max, samples, act,
                                            ctypes.byref(m))
        return rc, m

    def load_layer(self, block, layer, data):
        """data: a numpy uint8 array of layer_bytes (reference layout)."""
        return self.lib.frc_load_layer(self.h, block, layer, _ptr(data), data.nbytes)

    def unload(self, block):
        return self.lib.frc_unload_unit(self.h, block)

    def refresh_layer(self, block, layer, data):
        """frc_refresh_layer: copy one loaded layer again from host memory."""
        return self.lib.frc_refresh_layer(self.h, block, layer, _ptr(data), data.nbytes)

    def set_avx2_workers(self, workers):
        """frc_set_avx2_workers: the AVX2 backend worker count ACT_AVX2 reproduces."""
        self._check(self.lib.frc_set_avx2_workers(self.h, int(workers)), "set_avx2_workers")

    def avx2_timing(self, enable=True):
        """frc_avx2_timing: CUDA events around the three ACT_AVX2 launches of each call."""
        self._check(self.lib.frc_avx2_timing(self.h, 1 if enable else 0), "avx2_timing")

    def avx2_times(self):
        """ms of the last ACT_AVX2 call's quantization, job and reduction launches."""
        ms = np.zeros(3, np.float32)
        self._check(self.lib.frc_avx2_times(self.h, _ptr(ms)), "avx2_times")
        return ms

    def set_wait_limit(self, ns):
        """frc_set_wait_limit: every bounded wait of the layer kernel gives up after ns."""
        self._check(self.lib.frc_set_wait_limit(self.h, int(ns)), "set_wait_limit")

    def layer_variant(self, variant):
        """frc_debug_layer_variant: which kernel serves one-token Q8 calls: 1 the default (row-owner up to
        two slices), 0 always the item kernel, 2 the row-owner kernel whenever it fits."""
        self._check(self.lib.frc_debug_layer_variant(self.h, variant), "layer_variant")

    def debug_barrier_extra(self, extra):
        """Tests only: the grid barrier waits for `extra` arrivals that never come."""
        self._check(self.lib.frc_debug_barrier_extra(self.h, extra), "debug_barrier_extra")

    def loaded_mask(self):
        m = ctypes.c_uint32()
        self._check(self.lib.frc_loaded_mask(self.h, ctypes.byref(m)), "loaded_mask")
        return m.value

    def run(self, layer, expert, gate, x, act=ACT_Q8, out=None, flags=0):
        """Synchronous host-memory run (fr_backend.run semantics; flags:
        frc_run_flags, RUN_PEER).  Returns (rc, y); on failure y is the
        untouched `out` (or None)."""
        expert = np.ascontiguousarray(expert, np.uint16)
        gate = np.ascontiguousarray(gate, np.float32)
        x = np.ascontiguousarray(x, np.float32)
        tokens = x.shape[0]
        y = out if out is not None else np.zeros((tokens, self.hidden), np.float32)
        if flags:
            rc = self.lib.frc_run_flags(self.h, layer, tokens, _ptr(expert), _ptr(gate), _ptr(x), _ptr(y), act, flags)
        else:
            rc = self.lib.frc_run(self.h, layer, tokens, _ptr(expert), _ptr(gate), _ptr(x), _ptr(y), act)
        return rc, y

    def run_device(self, layer, tokens, expert_ptr, gate_ptr, x_ptr, x_add_ptr, x_out_ptr, y_ptr, act=ACT_Q8,
                   flags=0, stream=None):
        rc = self.lib.frc_run_device(self.h, layer, tokens, expert_ptr, gate_ptr, x_ptr, x_add_ptr, x_out_ptr,
                                     y_ptr, act, flags, stream)
        self._check(rc, "run_device")

    def run_device_fixed(self, layer, tokens, expert_ptr, gate_ptr, x_ptr, x_add_ptr, x_out_ptr, y_ptr,
                         act=ACT_Q8, flags=0, stream=None):
        """run_device with the hidden hand-off in the library's fixed device
        array (allocates nothing; see frc_run_device_fixed)."""
        rc = self.lib.frc_run_device_fixed(self.h, layer, tokens, expert_ptr, gate_ptr, x_ptr, x_add_ptr,
                                           x_out_ptr, y_ptr, act, flags, stream)
        self._check(rc, "run_device_fixed")

    def host_pass(self, first_layer, expert, gate, h, act=ACT_Q8, flags=0):
        """Decode pass from the host (frc_host_pass_flags).  expert: [layers][10] or
        [layers][tokens][10]; h ([hidden] or [tokens][hidden], fp32) is updated in place.
        flags: RUN_PEER sums every layer over the in-box reduce group."""
        expert = np.ascontiguousarray(expert, np.uint16)
        gate = np.ascontiguousarray(gate, np.float32)
        assert h.dtype == np.float32 and h.flags.c_contiguous
        tokens = expert.shape[1] if expert.ndim == 3 else 1
        hidden = h.shape[-1]
        rc = self.lib.frc_host_pass_flags(self.h, first_layer, expert.shape[0], tokens, _ptr(expert), _ptr(gate),
                                          _ptr(h), hidden, act, flags)
        self._check(rc, "host_pass")

    def peer_export(self, world):
        """Allocates this context's in-box reduce inbox; returns its IPC handle (bytes)."""
        h = ctypes.create_string_buffer(PEER_HANDLE_BYTES)
        self._check(self.lib.frc_peer_export(self.h, world, h), "peer_export")
        return h.raw

    def peer_attach(self, rank, world, handles):
        """handles: every rank's peer_export bytes, in rank order."""
        buf = ctypes.create_string_buffer(b"".join(handles), PEER_HANDLE_BYTES * world)
        self._check(self.lib.frc_peer_attach(self.h, rank, world, buf), "peer_attach")

    def peer_detach(self):
        self._check(self.lib.frc_peer_detach(self.h), "peer_detach")

    def status(self, stream=None):
        return self.lib.frc_status(self.h, stream)

    def pool_load(self, slices, shared):
        slices = np.ascontiguousarray(slices, np.uint8)
        count = slices.size // slice_bytes(self.g)
        self._check(self.lib.frc_pool_load(self.h, _ptr(slices), count, _ptr(np.ascontiguousarray(shared))),
                    "pool_load")
        return count

    def fill_layer(self, block, layer, seed):
        self._check(self.lib.frc_fill_layer(self.h, block, layer, seed), "fill_layer")

    def debug_decode(self, type_, rows, n, count):
        out = np.zeros((count, n), np.float32)
        self._check(self.lib.frc_debug_decode(self.h, type_, _ptr(np.ascontiguousarray(rows, np.uint8)), n, count,
                                              _ptr(out)), "debug_decode")
        return out

    def debug_quantize(self, x):
        x = np.ascontiguousarray(x, np.float32)
        tokens = x.shape[0]
        q = np.zeros(x.shape, np.int8)
        s = np.zeros((tokens, self.hidden // 64), np.float32)
        deq = np.zeros(x.shape, np.float32)
        self._check(self.lib.frc_debug_quantize(self.h, tokens, _ptr(x), _ptr(q), _ptr(s), _ptr(deq)),
                    "debug_quantize")
        return q, s, deq

    def debug_umma(self, a, b):
        """int32 a[128][k] @ b[n][k]^T through the tcgen05 kind::i8 check kernel."""
        a = np.ascontiguousarray(a, np.int8)
        b = np.ascontiguousarray(b, np.int8)
        d = np.zeros((128, b.shape[0]), np.int32)
        self._check(self.lib.frc_debug_umma(self.h, b.shape[0], a.shape[1], _ptr(a), _ptr(b), _ptr(d)), "debug_umma")
        return d

    def prefill_timing(self, enable):
        self._check(self.lib.frc_prefill_timing(self.h, 1 if enable else 0), "prefill_timing")

    def prefill_times(self):
        """ms of the last timed prefill call: quantize, group, gate/up MMA, down MMA, combine."""
        ms = np.zeros(5, np.float32)
        self._check(self.lib.frc_prefill_times(self.h, _ptr(ms)), "prefill_times")
        return ms

    def debug_prefill_hidden(self):
        """(hq [pair][block][32] int8, hs [pair][block] f32) of the last prefill burst."""
        n = ctypes.c_size_t()
        self._check(self.lib.frc_debug_prefill_hidden(self.h, None, None, 0, ctypes.byref(n)), "debug_prefill_hidden")
        S = bin(self.loaded_mask()).count("1")
        hq = np.zeros((n.value, S, 32), np.int8)
        hs = np.zeros((n.value, S), np.float32)
        self._check(self.lib.frc_debug_prefill_hidden(self.h, _ptr(hq), _ptr(hs), n.value, ctypes.byref(n)),
                    "debug_prefill_hidden")
        return hq, hs

    def debug_phases(self):
        """[cta][16] globaltimer stamps of the last launch (FRC_PHASES builds)."""
        n = ctypes.c_size_t()
        rc = self.lib.frc_debug_phases(self.h, None, 0, ctypes.byref(n))
        if rc:
            raise FrcError(rc, "debug_phases", self.last_error)
        out = np.zeros(n.value, np.uint64)
        self._check(self.lib.frc_debug_phases(self.h, _ptr(out), n.value, ctypes.byref(n)), "debug_phases")
        return out.reshape(-1, 16)

    def debug_hidden(self):
        n = ctypes.c_size_t()
        self._check(self.lib.frc_debug_hidden(self.h, None, 0, ctypes.byref(n)), "debug_hidden")
        out = np.zeros(n.value, np.float32)
        self._check(self.lib.frc_debug_hidden(self.h, _ptr(out), n.value, ctypes.byref(n)), "debug_hidden")
        return out


def cuda_available():
    """True when the library loads and device 0 is an sm_100 part."""
    try:
        lib = library()
    except FrcError:
        return False
    return lib.frc_probe_device(0, None, 0, None, None) == OK


def probe_device(device=0):
    """(rc, name, hbm_bytes, sms) of frc_probe_device (no context is opened)."""
    name = ctypes.create_string_buffer(128)
    hbm, sms = ctypes.c_uint64(), ctypes.c_uint()
    rc = library().frc_probe_device(device, name, 128, ctypes.byref(hbm), ctypes.byref(sms))
    return rc, name.value.decode(), hbm.value, sms.value
