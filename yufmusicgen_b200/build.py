"""Build recipe for ``libyufb200.so`` (sm_100a only).

Each ``csrc/*.cu`` / ``*.cpp`` file is compiled to an object under
``yufmusicgen_b200/_build/`` (in parallel, skipped when up to date) and linked
into ``yufmusicgen_b200/libyufb200.so`` in the source tree, so the library
travels with the checkout.  ``python -m yufmusicgen_b200.build [-v]``.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
OUT_DIR = PKG / "_build"
LIB = PKG / "libyufb200.so"
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I", str(INCLUDE),
              "--expt-relaxed-constexpr"]
LINK_LIBS = ["-lcudart"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libyufb200")
    return cand


def _sources():
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")))


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: Path, ptxas_verbose: bool) -> tuple[Path, str]:
    obj = OUT_DIR / (src.stem + ".o")
    if obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, _headers_mtime()):
        return obj, ""
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if ptxas_verbose and src.suffix == ".cu":
        cmd += ["-Xptxas", "-v"]
    p = subprocess.run(cmd, capture_output=True, text=True)
    if p.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{p.stdout}\n{p.stderr}")
    return obj, p.stderr


def build(verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    OUT_DIR.mkdir(exist_ok=True)
    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        results = list(ex.map(lambda s: _compile(s, ptxas_verbose), srcs))
    objs = [o for o, _ in results]
    if verbose:
        for o, log in results:
            if log:
                print(f"--- {o.name}\n{log}", file=sys.stderr)
    newest = max(o.stat().st_mtime for o in objs)
    if not LIB.exists() or LIB.stat().st_mtime < newest:
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs), *LINK_LIBS]
        p = subprocess.run(cmd, capture_output=True, text=True)
        if p.returncode != 0:
            raise RuntimeError(f"link failed:\n{p.stdout}\n{p.stderr}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    v = "-v" in sys.argv
    print(build(verbose=v, ptxas_verbose=v))
