"""Build libtdsa.so (the C-ABI library) in-tree for sm_100a with nvcc.

    python -m dsa_b200.build [-v] [--force] [--timeline]

Objects go to ``dsa_b200/_build/``, the library to ``dsa_b200/_lib/libtdsa.so``.  Each
translation unit compiles in its own nvcc process (in parallel); the library is rebuilt
when any source or header is newer than it.  ``--timeline`` builds the measurement variant
``dsa_b200/_lib/libtdsa_timeline.so`` instead (TDSA_TIMELINE defined: device timestamps in
the decode step's kernels and a read-stream probe, read by ``python -m dsa_b200.timeline``);
its objects go to ``dsa_b200/_build_timeline/``.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
BUILD = HERE / "_build"
LIB = HERE / "_lib" / "libtdsa.so"
BUILD_TIMELINE = HERE / "_build_timeline"
LIB_TIMELINE = HERE / "_lib" / "libtdsa_timeline.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
         "--expt-relaxed-constexpr", f"-I{ROOT / 'include'}", f"-I{CSRC}"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _deps() -> list[Path]:
    return _sources() + sorted(CSRC.glob("*.cuh")) + sorted((ROOT / "include").glob("*.h"))


def needs_build(lib: Path = LIB) -> bool:
    if not lib.exists():
        return True
    t = lib.stat().st_mtime
    return any(p.stat().st_mtime > t for p in _deps())


def build(verbose: bool = False, force: bool = False, ptxas_info: bool = False,
          timeline: bool = False) -> Path:
    lib, objdir = (LIB_TIMELINE, BUILD_TIMELINE) if timeline else (LIB, BUILD)
    if not force and not needs_build(lib):
        return lib
    objdir.mkdir(parents=True, exist_ok=True)
    lib.parent.mkdir(parents=True, exist_ok=True)
    cc = nvcc()
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    if timeline:
        extra.append("-DTDSA_TIMELINE")

    def compile_one(src: Path) -> Path:
        obj = objdir / (src.stem + ".o")
        cmd = [cc, *ARCH, *FLAGS, *extra, "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
        if (verbose or ptxas_info) and res.stderr:
            print(res.stderr, flush=True)
        return obj

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as pool:
        objs = list(pool.map(compile_one, _sources()))
    tmp = lib.with_suffix(".so.tmp")
    cmd = [cc, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", str(tmp), *map(str, objs),
           "-cudart", "static"]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, lib)
    return lib


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    ap.add_argument("--timeline", action="store_true",
                    help="build the measurement variant libtdsa_timeline.so")
    args = ap.parse_args()
    print(build(verbose=args.verbose, force=args.force, ptxas_info=args.ptxas_info,
                timeline=args.timeline))


if __name__ == "__main__":
    main()
