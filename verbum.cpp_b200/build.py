"""Builds libverbum_b200.so in-tree (verbum.cpp_b200/lib/) with nvcc for sm_100a.

Usage:  python verbum.cpp_b200/build.py [--force] [--verbose]

Every .cu / .cpp under csrc/ (and host/) is compiled to an object in
verbum.cpp_b200/_build/ and linked into one shared library with the shared
CUDA runtime.  Objects are rebuilt only when a source or header is newer, or
when the preprocessor definitions differ from the last build's
(--define VB_STEP_TRACE=1 gives the profiling build whose clustered step
records its phase trace).
"""
import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
HOST = PKG / "host"
BUILD = PKG / "_build"
LIB = PKG / "lib"
LIBNAME = "libverbum_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path():
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return cand


def cuda_home():
    return Path(nvcc_path()).resolve().parent.parent


def sources():
    srcs = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))
    if HOST.exists():
        srcs += sorted(HOST.glob("*.cpp"))
    return srcs


def headers():
    hs = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list((ROOT / "include").glob("*.h"))
    if HOST.exists():
        hs += list(HOST.rglob("*.h")) + list(HOST.rglob("*.hpp"))
    return hs


DEFINES = []


def compile_one(src, verbose=False, ptxas_v=False):
    obj = BUILD / (src.name + ".o")
    newest_hdr = max((h.stat().st_mtime for h in headers()), default=0)
    if obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, newest_hdr) and not ptxas_v:
        return obj, ""
    inc = ["-I", str(ROOT / "include"), "-I", str(CSRC)]
    if HOST.exists():
        inc += ["-I", str(HOST / "include")]
    cmd = [nvcc_path(), *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
           "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr", *inc,
           *[f"-D{d}" for d in DEFINES], "-c", str(src), "-o", str(obj)]
    if ptxas_v and src.suffix == ".cu":
        cmd.insert(1, "-Xptxas=-v")
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(force=False, verbose=False, ptxas_v=False, defines=(), build_dir=None, out=None, src_dir=None):
    global BUILD, CSRC
    if build_dir:
        BUILD = Path(build_dir)
    if src_dir:
        CSRC = Path(src_dir).resolve()
    BUILD.mkdir(parents=True, exist_ok=True)
    LIB.mkdir(exist_ok=True)
    DEFINES[:] = sorted(defines)
    stamp = BUILD / "defines.txt"
    if not stamp.exists() or stamp.read_text() != " ".join(DEFINES):
        force = True
        stamp.write_text(" ".join(DEFINES))
    if force:
        for o in BUILD.glob("*.o"):
            o.unlink()
    srcs = sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        results = list(ex.map(lambda s: compile_one(s, verbose, ptxas_v), srcs))
    objs = [r[0] for r in results]
    if ptxas_v:
        for s, (_, log) in zip(srcs, results):
            if log:
                print(f"== {s.name}\n{log}")
    out = Path(out) if out else LIB / LIBNAME
    out.parent.mkdir(parents=True, exist_ok=True)
    if out.exists() and not force and all(o.stat().st_mtime <= out.stat().st_mtime for o in objs):
        return out
    cudalib = cuda_home() / "lib64"
    cmd = [nvcc_path(), *ARCH, "-shared", "-cudart", "shared", "-o", str(out), *map(str, objs),
           "-Xlinker", f"-rpath={cudalib}", "-lcuda", "-lpthread"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print register/smem usage")
    ap.add_argument("--define", action="append", default=[], help="NAME=VALUE passed to nvcc as -D")
    ap.add_argument("--build-dir", default=None, help="object directory (default verbum.cpp_b200/_build)")
    ap.add_argument("--out", default=None, help="library path (default verbum.cpp_b200/lib/libverbum_b200.so)")
    ap.add_argument("--src-dir", default=None, help="kernel sources (default verbum.cpp_b200/csrc)")
    a = ap.parse_args()
    out = build(a.force, a.verbose, a.ptxas_v, a.define, a.build_dir, a.out, a.src_dir)
    print(out)


if __name__ == "__main__":
    sys.exit(main())
