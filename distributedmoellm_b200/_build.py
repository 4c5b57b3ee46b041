"""Build libmoelan_b200.so (sm_100a) in-tree with nvcc.

Each ``csrc/*.cu`` is compiled to an object in ``_build/`` (in parallel, only
when it or a header changed) and the objects are linked into
``_lib/libmoelan_b200.so``, which the package loads with ctypes.
"""

from __future__ import annotations

import os
import shutil
import subprocess
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
BUILD = HERE / "_build"
LIB = HERE / "_lib" / "libmoelan_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
         "-I", str(ROOT / "include")]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA extension cannot be built")


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.cuh")) + list((ROOT / "include").glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    srcs = sorted(CSRC.glob("*.cu"))
    BUILD.mkdir(exist_ok=True)
    LIB.parent.mkdir(exist_ok=True)
    hdr = _headers_mtime()
    cc = nvcc()

    def obj(src: Path) -> tuple[Path, str]:
        o = BUILD / (src.stem + ".o")
        if not force and o.exists() and o.stat().st_mtime >= max(src.stat().st_mtime, hdr):
            return o, ""
        cmd = [cc, *ARCH, *FLAGS, "-c", str(src), "-o", str(o)]
        if ptxas_info:
            cmd.insert(1, "-Xptxas=-v")
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stderr}")
        return o, r.stderr

    with ThreadPoolExecutor(max(1, min(len(srcs), os.cpu_count() or 4))) as pool:
        results = list(pool.map(obj, srcs))
    if verbose or ptxas_info:
        for (o, log) in results:
            if log:
                print(f"--- {o.name}\n{log}")
    objs = [o for o, _ in results]
    if force or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        r = subprocess.run([cc, *ARCH, "-shared", "-o", str(tmp), *map(str, objs)],
                           capture_output=True, text=True)
        if r.returncode:
            raise RuntimeError(f"link failed:\n{r.stderr}")
        tmp.replace(LIB)
    return LIB


if __name__ == "__main__":
    import sys
    print(build(force="--force" in sys.argv, verbose=True, ptxas_info="-v" in sys.argv))
