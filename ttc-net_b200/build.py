"""Build the in-tree CUDA library ``ttc_b200/libttc_b200.so`` for sm_100a.

    python ttc-net_b200/build.py [--force] [-j JOBS]

Every ``csrc/*.cu`` translation unit is compiled by nvcc in parallel into
``_build/`` and linked into one shared library with the CUDA runtime linked
statically.  The library lands next to the Python package so it travels with
the source tree (nothing is installed into site-packages).  A rebuild is skipped
when the library is newer than every source, header and this script.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(REPO, "include")
OBJDIR = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "ttc_b200", "libttc_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ARCH + ["-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
                 "-Xptxas", "-v", "-I", INCLUDE, "-I", CSRC]


def _nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand) and shutil.which(cand) is None:
        raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")
    return cand


def _inputs():
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    deps = srcs + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))
    return srcs, deps + [os.path.abspath(__file__)]


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    _, deps = _inputs()
    return os.path.getmtime(LIB) >= max(os.path.getmtime(p) for p in deps)


def _compile(nvcc: str, src: str, objdir: str = OBJDIR, extra=()) -> tuple[str, str]:
    obj = os.path.join(objdir, os.path.splitext(os.path.basename(src))[0] + ".o")
    r = subprocess.run([nvcc, *CFLAGS, *extra, "-c", src, "-o", obj], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{r.stderr}")
    return obj, r.stderr


def build(force: bool = False, jobs: int | None = None, verbose: bool = False, out: str | None = None,
          defines=()) -> str:
    """Compile and link the library; returns its path.  `out` and `defines` (NAME=VALUE
    macros, e.g. the kernels' tuning switches) build a variant elsewhere, always from scratch;
    the package loads such a build when TTC_B200_LIB names it."""
    lib = out or LIB
    if out is None and not defines and not force and up_to_date():
        return LIB
    nvcc = _nvcc()
    srcs, _ = _inputs()
    objdir = OBJDIR if out is None else tempfile.mkdtemp(prefix="ttc_b200_obj_")
    os.makedirs(objdir, exist_ok=True)
    extra = [f"-D{d}" for d in defines]
    jobs = jobs or min(len(srcs), os.cpu_count() or 1)
    objs, logs = [], []
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        for obj, log in ex.map(lambda s: _compile(nvcc, s, objdir, extra), srcs):
            objs.append(obj)
            logs.append(log)
    os.makedirs(os.path.dirname(os.path.abspath(lib)), exist_ok=True)
    tmp = lib + ".tmp"
    r = subprocess.run([nvcc, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", tmp, *objs],
                       capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stderr}")
    os.replace(tmp, lib)
    if out is not None:
        shutil.rmtree(objdir, ignore_errors=True)
    if verbose:
        for log in logs:
            for line in log.splitlines():
                if "registers" in line or "spill" in line or "Compiling entry" in line:
                    print(line)
    return lib


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--force", action="store_true", help="rebuild even if up to date")
    ap.add_argument("-j", "--jobs", type=int, default=None)
    ap.add_argument("-v", "--verbose", action="store_true", help="print ptxas register/spill lines")
    ap.add_argument("--out", default=None, help="build a variant library at this path")
    ap.add_argument("-D", "--define", action="append", default=[], help="NAME=VALUE macro for the variant")
    a = ap.parse_args(argv)
    print(build(force=a.force, jobs=a.jobs, verbose=a.verbose, out=a.out, defines=a.define))
    return 0


if __name__ == "__main__":
    sys.exit(main())
