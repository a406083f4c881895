"""Test oracle bindings.  TEST INFRASTRUCTURE ONLY: imported by tests/, by
__graft_entry__.smoke() and by bench.py's CPU-baseline leg, never by the
product (fronk_b200/).

  Oracle     this project's C restatement (liboracle.so, fronk_oracle.c)
  Reference  the reference compiled from its own sources (oracle/_ref/*.so),
             when it was built; fr_ref / fr_ref_q8 / fr_avx2 and its helpers.
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_LIB = os.path.join(HERE, "liboracle.so")
REF_DIR = os.path.join(HERE, "_ref")

OK, INVALID, STATE, NUMERIC = 0, -1, -2, -3
Q4_0, Q8_0, Q4_K, MXFP4 = 2, 8, 12, 39

_vp = ctypes.c_void_p


def _p(a):
    return None if a is None else ctypes.c_void_p(a.ctypes.data)


class OrModel(ctypes.Structure):
    _fields_ = [("hidden", ctypes.c_uint), ("gate_type", ctypes.c_uint), ("down_type", ctypes.c_uint),
                ("legacy", ctypes.c_uint), ("layer", ctypes.c_void_p * 20)]


class Oracle:
    def __init__(self, path=ORACLE_LIB):
        if not os.path.exists(path):
            from . import build as _b
            _b.build_oracle()
        L = ctypes.CDLL(path)
        sig = {
            "or_f16": (ctypes.c_float, [ctypes.c_uint16]),
            "or_q8_activation": (ctypes.c_int, [_vp, _vp, ctypes.c_size_t]),
            "or_q8_quantize": (ctypes.c_int, [_vp, ctypes.c_size_t, _vp, _vp]),
            "or_native_dot": (ctypes.c_int, [_vp, ctypes.c_uint, _vp, ctypes.c_uint, _vp]),
            "or_q4_0_dot": (ctypes.c_int, [_vp, _vp, ctypes.c_size_t, _vp]),
            "or_decode_row": (ctypes.c_int, [_vp, ctypes.c_uint, ctypes.c_uint, _vp]),
            "or_row_bytes": (ctypes.c_size_t, [ctypes.c_uint, ctypes.c_uint]),
            "or_slice_bytes": (ctypes.c_size_t, [ctypes.c_uint, ctypes.c_uint, ctypes.c_uint]),
            "or_shared_bytes": (ctypes.c_size_t, [ctypes.c_uint]),
            "or_layer_bytes": (ctypes.c_size_t, [ctypes.c_uint, ctypes.c_uint, ctypes.c_uint]),
            "or_legacy_layer_bytes": (ctypes.c_size_t, [ctypes.c_uint]),
            "or_ref_run": (ctypes.c_int, [_vp, ctypes.c_uint, _vp, _vp, _vp, _vp, ctypes.c_int]),
            "or_avx2_run": (ctypes.c_int, [_vp, ctypes.c_uint, _vp, _vp, _vp, _vp, ctypes.c_uint, ctypes.c_int, _vp,
                                           ctypes.c_uint]),
            "or_port_run": (ctypes.c_int, [_vp, ctypes.c_uint, _vp, _vp, _vp, _vp, _vp, ctypes.c_size_t, _vp]),
            "or_prefill_run": (ctypes.c_int, [_vp, ctypes.c_uint, _vp, _vp, _vp, _vp, _vp, _vp, ctypes.c_size_t,
                                              _vp]),
            "or_block_idots": (ctypes.c_int, [_vp, ctypes.c_uint, ctypes.c_uint, _vp, _vp]),
            "or_compare": (ctypes.c_int, [_vp, _vp, ctypes.c_size_t, _vp]),
        }
        for name, (res, args) in sig.items():
            f = getattr(L, name)
            f.restype, f.argtypes = res, args
        self.L = L

    # scalar helpers -----------------------------------------------------
    def f16(self, bits):
        return self.L.or_f16(bits)

    def q8_activation(self, x):
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros_like(x)
        rc = self.L.or_q8_activation(_p(x), _p(out), x.size)
        return rc, out

    def q8_quantize(self, x):
        x = np.ascontiguousarray(x, np.float32)
        q = np.zeros(x.size, np.int8)
        s = np.zeros((x.size + 63) // 64, np.float32)
        rc = self.L.or_q8_quantize(_p(x), x.size, _p(q), _p(s))
        return rc, q, s

    def native_dot(self, row, type_, x):
        out = ctypes.c_double()
        x = np.ascontiguousarray(x, np.float32)
        rc = self.L.or_native_dot(_p(np.ascontiguousarray(row, np.uint8)), type_, _p(x), x.size, ctypes.byref(out))
        return rc, out.value

    def decode_row(self, row, type_, n):
        w = np.zeros(n, np.float32)
        rc = self.L.or_decode_row(_p(np.ascontiguousarray(row, np.uint8)), type_, n, _p(w))
        return rc, w

    def block_idots(self, row, type_, v):
        v = np.ascontiguousarray(v, np.int8)
        out = np.zeros(v.size // 32, np.int32)
        rc = self.L.or_block_idots(_p(np.ascontiguousarray(row, np.uint8)), type_, v.size, _p(v), _p(out))
        return rc, out

    def compare(self, ref, actual):
        out = (ctypes.c_double * 3)()
        ref = np.ascontiguousarray(ref, np.float32)
        actual = np.ascontiguousarray(actual, np.float32)
        rc = self.L.or_compare(_p(ref), _p(actual), ref.size, out)
        return rc, tuple(out)

    # runs ------------------------------------------------------------------
    def model(self, hidden, gate_type, down_type, layers, legacy=0):
        """layers: {block: uint8 array covering the requested layer}.  The
        model keeps a reference to the arrays it points into."""
        m = OrModel(hidden, gate_type, down_type, legacy)
        for b, arr in layers.items():
            m.layer[b] = arr.ctypes.data
        m._keep = dict(layers)
        return m

    def ref_run(self, m, expert, gate, x, q8):
        x = np.ascontiguousarray(x, np.float32)
        y = np.zeros_like(x)
        rc = self.L.or_ref_run(ctypes.byref(m), x.shape[0], _p(np.ascontiguousarray(expert, np.uint16)),
                               _p(np.ascontiguousarray(gate, np.float32)), _p(x), _p(y), int(q8))
        return rc, y

    def avx2_run(self, m, expert, gate, x, workers=1, libm_expf=True, order=None):
        """The AVX2 backend's arithmetic (backends/avx2.c) with `workers`
        workers; libm_expf False gives the CUDA AVX2 mode's SiLU; order: the
        blocks in load order (None: ascending)."""
        x = np.ascontiguousarray(x, np.float32)
        y = np.zeros_like(x)
        o = None if order is None else np.ascontiguousarray(order, np.uint8)
        rc = self.L.or_avx2_run(ctypes.byref(m), x.shape[0], _p(np.ascontiguousarray(expert, np.uint16)),
                                _p(np.ascontiguousarray(gate, np.float32)), _p(x), _p(y), int(workers),
                                int(bool(libm_expf)), None if o is None else _p(o), 0 if o is None else o.size)
        return rc, y

    def port_run(self, m, expert, gate, x, want_hidden=False):
        x = np.ascontiguousarray(x, np.float32)
        y = np.zeros_like(x)
        n = ctypes.c_size_t()
        e = np.ascontiguousarray(expert, np.uint16)
        g = np.ascontiguousarray(gate, np.float32)
        h = None
        if want_hidden:
            rc = self.L.or_port_run(ctypes.byref(m), x.shape[0], _p(e), _p(g), _p(x), _p(y), None, 0, ctypes.byref(n))
            h = np.zeros(max(n.value, 1), np.float32)
            rc = self.L.or_port_run(ctypes.byref(m), x.shape[0], _p(e), _p(g), _p(x), _p(y), _p(h), h.size,
                                    ctypes.byref(n))
            h = h[:n.value]
        else:
            rc = self.L.or_port_run(ctypes.byref(m), x.shape[0], _p(e), _p(g), _p(x), _p(y), None, 0, None)
        return rc, y, h

    def prefill_run(self, m, expert, gate, x, want_hidden=False):
        """The CUDA prefill arithmetic: (rc, y, hq [pair][block][32] | None, hs [pair][block] | None)."""
        x = np.ascontiguousarray(x, np.float32)
        y = np.zeros_like(x)
        e = np.ascontiguousarray(expert, np.uint16)
        g = np.ascontiguousarray(gate, np.float32)
        if not want_hidden:
            return self.L.or_prefill_run(ctypes.byref(m), x.shape[0], _p(e), _p(g), _p(x), _p(y), None, None, 0,
                                         None), y, None, None
        S = sum(1 for p in m.layer if p)
        cap = x.shape[0] * 11  # ten routed pairs a token, and the shared expert's
        hq = np.zeros((cap, S, 32), np.int8)
        hs = np.zeros((cap, S), np.float32)
        n = ctypes.c_size_t()
        rc = self.L.or_prefill_run(ctypes.byref(m), x.shape[0], _p(e), _p(g), _p(x), _p(y), _p(hq), _p(hs), cap,
                                   ctypes.byref(n))
        return rc, y, hq[:n.value], hs[:n.value]


# ------------------------------------------------------- compiled reference

def reference_lib_path(hidden=2560):
    return os.path.join(REF_DIR, "libfronk_ref.so" if hidden == 2560 else "libfronk_ref%d.so" % hidden)


def reference_available(hidden=2560):
    return os.path.exists(reference_lib_path(hidden))


class FrBackend(ctypes.Structure):
    pass


def _backend_fields(hidden):
    class Hw(ctypes.Structure):
        _fields_ = [("os", ctypes.c_char * 16), ("arch", ctypes.c_char * 16), ("version", ctypes.c_char * 64),
                    ("cpu", ctypes.c_char * 128), ("gpu", ctypes.c_char * 128), ("name", ctypes.c_char * 64),
                    ("cores", ctypes.c_uint), ("logical_cores", ctypes.c_uint), ("isa", ctypes.c_uint),
                    ("metal", ctypes.c_uint), ("translated", ctypes.c_uint)] + \
                   [(n, ctypes.c_uint64) for n in ("id", "total", "available", "margin", "cap", "blocks",
                                                    "metal_limit", "frequency", "wired_mb", "head_reserve",
                                                    "head_cap", "head_blocks", "head_fixed")]

    class Req(ctypes.Structure):
        _fields_ = [("layer", ctypes.c_uint), ("burst", ctypes.c_uint), ("expert", (ctypes.c_uint16 * 10) * 8),
                    ("gate", (ctypes.c_float * 11) * 8), ("x", (ctypes.c_float * hidden) * 8)]

    class Part(ctypes.Structure):
        _fields_ = [("layer", ctypes.c_uint), ("burst", ctypes.c_uint), ("y", (ctypes.c_float * hidden) * 8)]

    class Cost(ctypes.Structure):
        _fields_ = [("burst_max", ctypes.c_uint), ("t0_ns", ctypes.c_double), ("bw_eff", ctypes.c_double),
                    ("ns", ctypes.c_double * 8), ("bytes", ctypes.c_uint64 * 8)]

    class Backend(ctypes.Structure):
        _fields_ = [("name", ctypes.c_char_p),
                    ("probe", ctypes.CFUNCTYPE(ctypes.c_int, ctypes.POINTER(Hw))),
                    ("load", ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t)),
                    ("unload", ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_int)),
                    ("run", ctypes.CFUNCTYPE(ctypes.c_int, ctypes.POINTER(Req), ctypes.POINTER(Part))),
                    ("bench", ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_int, ctypes.POINTER(Cost))),
                    ("self_test", ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_char_p))]
    return Hw, Req, Part, Cost, Backend


class Reference:
    """The reference compiled from its own sources (fr_ref, fr_ref_q8, fr_avx2 ...)."""

    def __init__(self, hidden=2560):
        path = reference_lib_path(hidden)
        self.L = ctypes.CDLL(path, mode=ctypes.RTLD_GLOBAL)
        self.hidden = hidden
        self.Hw, self.Req, self.Part, self.Cost, self.Backend = _backend_fields(hidden)
        self.L.fr_f16.restype = ctypes.c_float
        self.L.fr_f16.argtypes = [ctypes.c_uint16]
        self.L.fr_q8_activation.argtypes = [_vp, _vp, ctypes.c_size_t]
        self.L.fr_native_dot.argtypes = [_vp, ctypes.c_uint, _vp, ctypes.c_uint, _vp]
        self.L.fr_native_self_test.argtypes = [_vp]
        self.L.fr_compare.argtypes = [_vp, _vp, ctypes.c_size_t, _vp]
        self.L.fr_native_fixture.argtypes = [_vp, ctypes.c_uint, ctypes.c_uint32]

    def backend(self, name):
        sym = {"ref": "fr_ref", "ref-q8": "fr_ref_q8", "avx2": "fr_avx2"}[name]
        return self.Backend.in_dll(self.L, sym)

    def configure_avx2(self, blocks, workers):
        """Fix fr_avx2's worker count for its next engine, which it makes at
        the first load (backends/avx2.c:561-566, :729-742); no block may be
        loaded.  Both reference builds are loaded RTLD_GLOBAL, so the
        fr_avx2_close inside one build's fr_avx2_configure can bind to the
        other build's: this build's engine is closed through its own handle
        first."""
        self.L.fr_avx2_set_tuning.argtypes = [ctypes.c_uint] * 4
        self.L.fr_avx2_configure.argtypes = [ctypes.c_uint, ctypes.c_uint]
        rc = self.L.fr_avx2_close()
        if rc:
            return rc
        for burst in range(1, 9):
            self.L.fr_avx2_set_tuning(blocks, burst, workers, 0)
        return self.L.fr_avx2_configure(blocks, 1)

    def avx2_engine_workers(self):
        """The worker count of fr_avx2's current engine (fr_avx2_sample_get,
        src/avx2.h:11-15): fr_avx2_configure caps the configured count at the
        host's logical CPUs minus one (backends/avx2.c:739-741)."""
        class Sample(ctypes.Structure):
            _fields_ = [("runs", ctypes.c_uint64), ("weight_bytes", ctypes.c_uint64),
                        ("hot_allocations", ctypes.c_uint64), ("blocks", ctypes.c_uint),
                        ("unique_experts", ctypes.c_uint), ("workers", ctypes.c_uint), ("features", ctypes.c_uint),
                        ("prefetch", ctypes.c_uint), ("total_ns", ctypes.c_double)]
        smp = Sample()
        self.L.fr_avx2_sample_get.argtypes = [ctypes.c_void_p]
        if self.L.fr_avx2_sample_get(ctypes.byref(smp)):
            raise RuntimeError("fr_avx2_sample_get failed")
        return smp.workers

    def backend_addr(self, sym, lib=None):
        return ctypes.addressof(self.Backend.in_dll(lib or self.L, sym))

    def unit_bytes(self):
        return 48 * (512 * (2 * 32 * (self.hidden // 256) * 144 + self.hidden * 17) + 3 * self.hidden * 34)

    def request(self, layer, expert, gate, x):
        r = self.Req()
        r.layer, r.burst = layer, x.shape[0]
        ctypes.memmove(ctypes.addressof(r.expert), np.ascontiguousarray(expert, np.uint16).ctypes.data, expert.size * 2)
        ctypes.memmove(ctypes.addressof(r.gate), np.ascontiguousarray(gate, np.float32).ctypes.data, gate.size * 4)
        ctypes.memmove(ctypes.addressof(r.x), np.ascontiguousarray(x, np.float32).ctypes.data, x.size * 4)
        return r

    def run(self, backend, req):
        part = self.Part()
        rc = backend.run(ctypes.byref(req), ctypes.byref(part))
        y = np.ctypeslib.as_array(part.y)[:req.burst].copy()
        return rc, y
