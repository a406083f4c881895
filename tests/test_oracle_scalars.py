"""The oracle's scalar layer against the reference's own known-answer tests
(tests/test_q4.c, tests/test_native.c, restated) and, where the reference was
compiled here, against its functions bit for bit."""
import ctypes

import numpy as np
import pytest

from oracle import Q4_K, MXFP4, Q8_0, NUMERIC, INVALID, OK, Reference, reference_available

FLT_MAX = np.finfo(np.float32).max


def test_f16_all_encodings(oracle):
    # tests/test_q4.c:11-20: all 65536 encodings, signed zero and specials
    bits = np.arange(65536, dtype=np.uint16)
    expect = bits.view(np.float16).astype(np.float32)
    got = np.array([oracle.f16(int(b)) for b in bits], np.float32)
    finite = np.isfinite(expect)
    assert np.array_equal(got[finite].view(np.uint32), expect[finite].view(np.uint32))
    assert np.array_equal(np.isnan(got), np.isnan(expect))
    assert np.array_equal(np.isinf(got), np.isinf(expect))


def test_q8_known_answers(oracle):
    # tests/test_q4.c:40-56
    x = np.zeros(96, np.float32)
    x[:7] = [127, 0.5, 1.5, 2.5, -0.5, -1.5, -2.5]
    x[64], x[65] = 254, 3
    rc, out = oracle.q8_activation(x)
    assert rc == OK
    assert list(out[:7]) == [127, 0, 2, 2, 0, -2, -2]
    assert out[64] == 254 and out[65] == 4
    rc, z = oracle.q8_activation(np.zeros(96, np.float32))
    assert rc == OK and not z.any()
    big = np.zeros(32, np.float32)
    big[0] = FLT_MAX
    rc, o = oracle.q8_activation(big)
    assert rc == OK and np.isfinite(o[0]) and o[0] > FLT_MAX * np.float32(0.99)
    tiny = np.zeros(32, np.float32)
    tiny[0] = np.float32(2.0 ** -149)
    rc, o = oracle.q8_activation(tiny)
    assert rc == OK and o[0] == 0
    small = np.zeros(32, np.float32)
    small[0] = np.float32(2.0 ** -125)
    rc, o = oracle.q8_activation(small)
    assert rc == OK and np.isfinite(o[0]) and o[0] > 0
    nan = np.zeros(32, np.float32)
    nan[0] = np.nan
    assert oracle.q8_activation(nan)[0] == NUMERIC
    assert oracle.q8_activation(np.zeros(31, np.float32))[0] == INVALID


def _q4k_kat_block():
    # tests/test_native.c:7-12: every sub-block scale/min encoding, both nibbles
    q = np.zeros(144, np.uint8)
    sc = [1, 2, 3, 4, 17, 34, 51, 63]
    mi = [63, 51, 34, 17, 4, 3, 2, 1]
    q[1], q[3] = 0x3c, 0x38   # d = 1, dmin = 0.5
    for g in range(4):
        q[4 + g] = sc[g] | ((sc[g + 4] >> 4) << 6)
        q[8 + g] = mi[g] | ((mi[g + 4] >> 4) << 6)
        q[12 + g] = (sc[g + 4] & 15) | ((mi[g + 4] & 15) << 4)
    for j in range(128):
        q[16 + j] = (j % 16) | ((15 - j % 16) << 4)
    return q, sc, mi


def test_q4k_known_answers(oracle):
    q, sc, mi = _q4k_kat_block()
    for j in range(256):
        x = np.zeros(256, np.float32)
        x[j] = 1
        g = j // 32
        v = 15 - j % 16 if g % 2 else j % 16
        rc, y = oracle.native_dot(q, Q4_K, x)
        assert rc == OK and y == sc[g] * v - 0.5 * mi[g], j
    bad = q.copy()
    bad[1] = 0x7c
    assert oracle.native_dot(bad, Q4_K, np.ones(256, np.float32))[0] == NUMERIC
    assert oracle.native_dot(q, Q4_K, np.ones(32, np.float32))[0] == INVALID


def test_mxfp4_and_q80_known_answers(oracle):
    # tests/test_native.c:15-27
    values = [0, .5, 1, 1.5, 2, 3, 4, 6, 0, -.5, -1, -1.5, -2, -3, -4, -6]
    mx = np.zeros(17, np.uint8)
    mx[0] = 127
    for j in range(16):
        mx[j + 1] = j | ((15 - j) << 4)
    for j in range(32):
        x = np.zeros(32, np.float32)
        x[j] = 1
        rc, y = oracle.native_dot(mx, MXFP4, x)
        assert rc == OK and y == values[j if j < 16 else 31 - j]
    x = np.zeros(32, np.float32)
    x[2] = 1
    mx[0] = 0
    rc, y = oracle.native_dot(mx, MXFP4, x)
    assert rc == OK and y == 2.0 ** -127
    mx[0] = 255
    assert oracle.native_dot(mx, MXFP4, x)[0] == NUMERIC
    shared = np.zeros(34, np.uint8)
    shared[1] = 0x38
    shared[4] = 128
    rc, y = oracle.native_dot(shared, Q8_0, x)
    assert rc == OK and y == -64


def test_block_integer_dots_match_decoded_weights(oracle):
    # The integer block dots (the GPU's Q8 arithmetic) reproduce the exact
    # decoded weights: Q4_K q*v, MXFP4 2*E2M1*v, Q8_0 q*v.
    rng = np.random.default_rng(3)
    v = rng.integers(-127, 128, 256).astype(np.int8)
    q, _, _ = _q4k_kat_block()
    rc, idots = oracle.block_idots(q, Q4_K, v)
    assert rc == OK
    for g in range(8):
        nib = [(q[16 + (g // 2) * 32 + j] >> (4 * (g % 2))) & 15 for j in range(32)]
        assert idots[g] == int(np.dot(np.array(nib), v[32 * g:32 * g + 32].astype(np.int64)))
    mx = rng.integers(0, 256, 17 * 8).astype(np.uint8)
    mx[::17] = 120
    rc, w = oracle.decode_row(mx, MXFP4, 256)
    rc2, idots = oracle.block_idots(mx, MXFP4, v)
    assert rc == OK and rc2 == OK
    for b in range(8):
        assert idots[b] == int(np.round((w[32 * b:32 * b + 32] / 2.0 ** (120 - 128)).astype(np.int64) @ v[32 * b:32 * b + 32]))


@pytest.mark.skipif(not reference_available(), reason="reference not compiled here")
def test_against_compiled_reference_bitwise(oracle):
    ref = Reference(2560)
    # fp16 decode, all encodings
    for b in range(0, 65536, 7):
        a, r = oracle.f16(b), ref.L.fr_f16(b)
        assert (np.isnan(a) and np.isnan(r)) or np.float32(a).view(np.uint32) == np.float32(r).view(np.uint32)
    rng = np.random.default_rng(11)
    # Q8 activations incl. ties and mixed magnitudes
    for trial in range(50):
        x = (rng.standard_normal(2560) * 10.0 ** rng.integers(-30, 30)).astype(np.float32)
        if trial % 5 == 0:
            x[:64] = np.round(x[:64]) + 0.5
        rc, mine = oracle.q8_activation(x)
        theirs = np.zeros_like(x)
        rc2 = ref.L.fr_q8_activation(theirs.ctypes.data if False else x.ctypes.data, theirs.ctypes.data, x.size)
        assert rc == rc2 == OK
        assert np.array_equal(mine.view(np.uint32), theirs.view(np.uint32))
    # native dots in double, random bytes with finite scales
    for type_, n, bsz in ((Q4_K, 2560, 144), (MXFP4, 2560, 17), (Q8_0, 2560, 34)):
        for trial in range(20):
            row = rng.integers(0, 256, n // (256 if type_ == Q4_K else 32) * bsz).astype(np.uint8)
            if type_ == Q4_K:
                row[1::144] &= 0x3b
                row[3::144] &= 0x3b
            elif type_ == MXFP4:
                row[::17] = rng.integers(100, 140, n // 32)
            else:
                row[1::34] &= 0x3b
            x = rng.standard_normal(n).astype(np.float32)
            rc, mine = oracle.native_dot(row, type_, x)
            out = ctypes.c_double()
            rc2 = ref.L.fr_native_dot(row.ctypes.data, type_, x.ctypes.data, n, ctypes.byref(out))
            assert rc == rc2 == OK and mine == out.value
