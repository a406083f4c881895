"""Builds the test oracle and, when the reference sources are present, the
reference itself.  TEST INFRASTRUCTURE ONLY.

  oracle/liboracle.so            this project's C restatement (fronk_oracle.c)
  oracle/_ref/libfronk_ref.so    reference src/{backend,q4,native,vectors,bench,
                                 ssd,hw,sha256}.c + backends/{ref,avx2}.c, d=2560
  oracle/_ref/libfronk_ref2048.so  the same sources with ref2048_model.h
                                 pre-included (d=2048; nothing is copied)
  oracle/_ref/ref_bench[_2048]   CPU-baseline harness (ref_bench.c) linked
                                 with those sources

The reference is compiled straight from where it lies; its own Makefile and
module generator are not run.  Outputs under oracle/_ref/ are git-ignored but
travel with the repository snapshot to the GPU host.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
# the reference's source tree: FRONK_REFERENCE, else a checkout beside this repository
REF = os.environ.get("FRONK_REFERENCE") or os.path.normpath(os.path.join(ROOT, "..", "reference"))
REF_OUT = os.path.join(HERE, "_ref")
ORACLE_LIB = os.path.join(HERE, "liboracle.so")

REF_SOURCES = ["src/backend.c", "src/q4.c", "src/native.c", "src/vectors.c", "src/bench.c", "src/ssd.c",
               "src/hw.c", "src/sha256.c", "backends/ref.c", "backends/avx2.c"]
REF_FLAGS = ["-O2", "-std=c11", "-D_POSIX_C_SOURCE=200809L", "-D_DEFAULT_SOURCE", '-DFR_VERSION="0.3.0"',
             '-DFR_BUILD_OS="linux"', '-DFR_BUILD_ARCH="x86_64"', "-DFR_BENCH_RUNTIME=1", "-DFR_AVX2_COMPUTE=1"]


def _run(cmd):
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError("oracle build failed: " + " ".join(cmd))


def _stale(target, sources):
    return not os.path.exists(target) or any(os.path.getmtime(s) > os.path.getmtime(target) for s in sources)


def build_oracle(force=False):
    src = [os.path.join(HERE, "fronk_oracle.c"), os.path.join(HERE, "fronk_oracle.h")]
    if force or _stale(ORACLE_LIB, src):
        _run(["gcc", "-O2", "-std=c11", "-fPIC", "-shared", "-Wall", "-ffp-contract=off", "-fno-fast-math",
              src[0], "-o", ORACLE_LIB, "-lm"])
    return ORACLE_LIB


def reference_present():
    return all(os.path.exists(os.path.join(REF, s)) for s in REF_SOURCES)


def build_reference(force=False):
    """Returns the dict of built artefacts, or {} when the reference is absent."""
    if not reference_present():
        return {}
    os.makedirs(REF_OUT, exist_ok=True)
    srcs = [os.path.join(REF, s) for s in REF_SOURCES]
    synth = os.path.join(ROOT, "fronk_b200", "csrc", "frc_synth.c")
    harness = os.path.join(HERE, "ref_bench.c")
    out = {}
    for tag, extra in (("", []), ("2048", ["-include", os.path.join(HERE, "ref2048_model.h")])):
        lib = os.path.join(REF_OUT, "libfronk_ref%s.so" % tag)
        if force or _stale(lib, srcs + [os.path.join(HERE, "ref2048_model.h")]):
            _run(["gcc", *REF_FLAGS, *extra, "-fPIC", "-shared", "-Wl,--no-undefined", *srcs, "-o", lib,
                  "-lm", "-pthread"])
        out["lib" + tag] = lib
        exe = os.path.join(REF_OUT, "ref_bench" + ("_" + tag if tag else ""))
        if force or _stale(exe, srcs + [harness, synth]):
            _run(["gcc", *REF_FLAGS, *extra, "-ffp-contract=off", "-I" + os.path.join(REF, "src"), harness, synth,
                  *srcs, "-o", exe, "-lm", "-pthread"])
        out["bench" + tag] = exe
    return out


def build(force=False):
    res = {"oracle": build_oracle(force)}
    res.update(build_reference(force))
    return res


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
