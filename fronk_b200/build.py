"""Builds libfronk_b200.so in-tree: the sm_100a kernels, the C ABI and the
fr_backend plugin table.  nvcc cross-compiles without a GPU."""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libfronk_b200.so")
PHASES_LIB = os.path.join(HERE, "libfronk_b200_phases.so")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUDA_SOURCES = ["frc.cu"]
C_SOURCES = ["frc_synth.c", "fr_cuda_backend.c", "frc_host.c", "frc_units.c", "frc_cost.c"]
DEPS = sorted(f for f in os.listdir(CSRC) if f.endswith((".cu", ".cuh", ".c", ".h")))  # every source and header


def _run(cmd):
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError("build step failed: " + " ".join(cmd))
    return proc.stdout + proc.stderr


def _stale(target, sources):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    headers = [os.path.join(ROOT, "include", h) for h in os.listdir(os.path.join(ROOT, "include"))]
    return any(os.path.getmtime(s) > t for s in sources + headers)


def build(force=False, verbose=False, phases=False):
    """Compile when a source is newer than the library; returns its path.
    phases=True builds the FRC_PHASES variant (per-CTA phase stamps)."""
    lib = PHASES_LIB if phases else LIB
    sources = [os.path.join(CSRC, s) for s in DEPS]
    if not force and not _stale(lib, sources):
        return lib
    os.makedirs(OUT, exist_ok=True)
    objs = []
    tag = "_phases" if phases else ""
    for s in CUDA_SOURCES:
        o = os.path.join(OUT, s + tag + ".o")
        log = _run([NVCC, *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-Xptxas", "-v",
                    *(["-DFRC_PHASES"] if phases else []), "-c", os.path.join(CSRC, s), "-o", o])
        with open(os.path.join(OUT, s + tag + ".ptxas.txt"), "w") as f:
            f.write(log)
        if verbose:
            print(log)
        objs.append(o)
    for s in C_SOURCES:
        o = os.path.join(OUT, s + ".o")
        _run(["gcc", "-O2", "-std=c11", "-fPIC", "-Wall", "-Wextra", "-ffp-contract=off", "-c",
              os.path.join(CSRC, s), "-o", o])
        objs.append(o)
    tmp = lib + ".tmp"
    _run([NVCC, *ARCH, "-shared", "-o", tmp, *objs, "-ldl", "-lm"])
    os.replace(tmp, lib)
    return lib


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv, phases="--phases" in sys.argv))
