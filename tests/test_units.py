"""Unit files from disk without a GPU: the library's SHA-256 (FIPS 180-4)
against the standard's examples and hashlib, and the unit-directory checks
of frc_unit_verify (the reference node's loader rules, src/units.c:25-75):
digest file format, file size and digest match."""
import hashlib
import os

import numpy as np
import pytest

import fronk_b200 as fb


# FIPS 180-2 appendix B examples
KNOWN = [
    (b"abc", "ba7816bf8f01cfea414140de5dae2223b00361a396177a9cb410ff61f20015ad"),
    (b"abcdbcdecdefdefgefghfghighijhijkijkljklmklmnlmnomnopnopq",
     "248d6a61d20638b8e5c026930c3e6039a33ce45964ff2167f6ecedd419db06c1"),
    (b"a" * 1000000, "cdc76e5c9914fb9281a1c7e284d73e67f1809a48a497200e046d39ccc7112cd0"),
    (b"", "e3b0c44298fc1c149afbf4c8996fb92427ae41e4649b934ca495991b7852b855"),
]


@pytest.mark.parametrize("msg,hexd", KNOWN)
def test_sha256_known_answers(built, msg, hexd):
    assert fb.sha256(msg).hex() == hexd


def test_sha256_matches_hashlib_across_block_edges(built):
    rng = np.random.default_rng(7)
    for n in list(range(0, 200)) + [511, 512, 513, 4095, 4096, 4097, 1 << 20]:
        m = rng.integers(0, 256, n, dtype=np.uint8).tobytes()
        assert fb.sha256(m) == hashlib.sha256(m).digest(), n


def _unit_dir(tmp_path, block, payload, digest=None):
    (tmp_path / ("unit-%02u.bin" % block)).write_bytes(payload)
    d = hashlib.sha256(payload).hexdigest() if digest is None else digest
    (tmp_path / ("unit-%02u.sha256" % block)).write_bytes(d.encode() + b"\n")
    return str(tmp_path)


def test_unit_verify_accepts_a_matching_unit(built, tmp_path):
    payload = os.urandom(100_000)
    d = _unit_dir(tmp_path, 3, payload)
    assert fb.unit_verify(d, 3, len(payload)) == fb.OK
    assert fb.unit_verify(d, 3, 0) == fb.OK                    # any size


def test_unit_verify_rejects_what_the_reference_rejects(built, tmp_path):
    payload = os.urandom(65_536)
    good = hashlib.sha256(payload).hexdigest()
    bad = ("0" if good[0] != "0" else "1") + good[1:]
    d = _unit_dir(tmp_path, 5, payload, bad)
    assert fb.unit_verify(d, 5, len(payload)) == fb.MISMATCH   # digest differs
    assert fb.unit_verify(d, 5, len(payload), verify=False) == fb.OK
    assert fb.unit_verify(d, 5, len(payload) + 1) == fb.IO     # another size
    assert fb.unit_verify(d, 6, 0) == fb.IO                    # no such unit
    assert fb.unit_verify(d, 20, 0) == fb.INVALID              # no such block
    for text in (good.upper() + "\n", good[:63] + "\n", good, good + "\n\n", good[:-1] + "g\n"):
        (tmp_path / "unit-05.sha256").write_bytes(text.encode())
        assert fb.unit_verify(d, 5, 0) == fb.INVALID, text     # 64 lowercase hex digits and a newline only
    (tmp_path / "unit-05.sha256").unlink()
    assert fb.unit_verify(d, 5, 0) == fb.IO                    # digest file missing
