"""The C-ABI library without a GPU: it loads, it exports every function the
headers in include/ declare, its fr_backend contract has the reference's
binary layout, and the host-side planner split matches the reference's
rule.  No compute call is made (the kernels need an sm_100 device)."""
import os
import re
import subprocess
import tempfile

import pytest

import fronk_b200 as fb
from fronk_b200 import planner

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INCLUDE = os.path.join(ROOT, "include")
# the reference's source tree: FRONK_REFERENCE, else a checkout beside this repository
REF_TREE = os.environ.get("FRONK_REFERENCE") or os.path.normpath(
    os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "..", "reference"))


def declared_symbols():
    names = set()
    for h in os.listdir(INCLUDE):
        text = open(os.path.join(INCLUDE, h)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names |= set(re.findall(r"\b((?:frc|fr_cuda)\w*)\s*\(", text))
        names |= set(re.findall(r"extern\s+const\s+fr_backend\s+([\w\s,]+);", text)[0].replace(" ", "").split(",")
                     if "extern const fr_backend" in text else [])
    return names


def test_library_exports_every_declared_symbol(built):
    lib = fb.library()
    names = declared_symbols()
    assert "frc_run_device" in names and "fr_cuda" in names and len(names) > 30
    missing = [n for n in sorted(names) if not hasattr(lib, n)]
    assert not missing, missing
    assert set(fb.EXPORTS) <= names | {"fr_cuda", "fr_cuda_f32", "fr_cuda_avx2"}


def test_status_strings_and_geometry_without_gpu(built):
    for rc in (fb.OK, fb.INVALID, fb.STATE, fb.NUMERIC, fb.IO, fb.UNSUPPORTED):
        assert fb.library().frc_strerror(rc)
    g = fb.geometry(2560)
    assert fb.unit_bytes(g) == 3347005440      # FR_NATIVE_BLOCK_BYTES (src/native.h)
    assert fb.slice_bytes(fb.geometry(2048)) == 108544
    assert fb.slice_bytes(fb.geometry(2048, 48, fb.MXFP4, fb.Q8_0)) == 139264


LAYOUT_PROBE = r"""
#include <stdio.h>
#include <stddef.h>
#include HEADER
int main(void) {
    printf("%zu %zu %zu %zu %zu %zu %zu %zu %zu %zu\n", sizeof(fr_req), sizeof(fr_part), sizeof(fr_costmodel),
           sizeof(fr_hwinfo), sizeof(fr_backend), offsetof(fr_req, x), offsetof(fr_part, y),
           offsetof(fr_costmodel, bytes), offsetof(fr_hwinfo, head_fixed), offsetof(fr_backend, self_test));
    return 0;
}
"""


def _layout(header, incs):
    with tempfile.TemporaryDirectory() as d:
        src = os.path.join(d, "p.c")
        open(src, "w").write(LAYOUT_PROBE.replace("HEADER", '"%s"' % header))
        exe = os.path.join(d, "p")
        subprocess.run(["gcc", "-std=c11", "-D_DEFAULT_SOURCE", *["-I" + i for i in incs], src, "-o", exe],
                       check=True, capture_output=True)
        return subprocess.run([exe], check=True, capture_output=True, text=True).stdout.split()


@pytest.mark.skipif(not os.path.isfile(os.path.join(REF_TREE, "src", "backend.h")), reason="reference sources absent")
def test_backend_abi_matches_reference_headers():
    ours = _layout(os.path.join(INCLUDE, "fr_backend_abi.h"), [INCLUDE])
    theirs = _layout(os.path.join(REF_TREE, "src", "backend.h"), [os.path.join(REF_TREE, "src")])
    assert ours == theirs


def test_planner_split_matches_reference_rule():
    # identical GPUs (src/planner.c:56-127 with equal cost curves)
    assert planner.equal_shares(1) == [20]
    assert planner.equal_shares(2) == [10, 10]
    assert planner.equal_shares(4) == [5, 5, 5, 5]
    assert planner.equal_shares(8) == [2, 2, 2, 2, 3, 3, 3, 3]
    assert planner.assign([2, 3]) == [[0, 1], [2, 3, 4]]
    assert [planner.owned_blocks(r, 2) for r in range(2)] == [list(range(10)), list(range(10, 20))]
    # a faster participant takes more; ties keep the first index (strict '>')
    fast = [0.0] + [float(b) for b in range(1, 21)]
    slow = [0.0] + [2.0 * b for b in range(1, 21)]
    s = planner.compute_shares([fast, slow])
    assert sum(s) == 20 and s[0] > s[1]
    # a non-monotone sweep point never makes a larger share look cheaper
    bumpy = [0.0, 5.0, 3.0] + [5.0 + b for b in range(3, 21)]
    assert sum(planner.compute_shares([bumpy, fast])) == 20
    with pytest.raises(ValueError):
        planner.compute_shares([[0.0, 1.0]] * 3)   # capacity 3 < 20
