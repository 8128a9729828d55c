"""Build libdoe_cuda.so in-tree for sm_100a.

    python -m doe_b200.build [--verbose-ptxas]

Every translation unit under doe_b200/csrc is compiled by nvcc for
`-gencode arch=compute_100a,code=sm_100a` and linked (with the CUDA runtime
linked statically) into doe_b200/libdoe_cuda.so, which ships beside the
package.  Object files go to doe_b200/_build/.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libdoe_cuda.so"
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2", "--expt-relaxed-constexpr",
          "-I", str(INCLUDE), "-I", str(CSRC)]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libdoe_cuda.so")


def sources() -> list[Path]:
    return sorted([*CSRC.glob("*.cu"), *CSRC.glob("*.cpp")])


def _compile(src: Path, verbose_ptxas: bool) -> tuple[Path, str]:
    obj = BUILD / (src.name + ".o")
    cmd = [nvcc(), *ARCH, *COMMON, "-c", str(src), "-o", str(obj)]
    if src.suffix == ".cpp":
        cmd = [nvcc(), *COMMON, "-Wno-deprecated-gpu-targets", "-x", "c++", "-c", str(src), "-o", str(obj)]
    elif verbose_ptxas:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    return obj, res.stderr


def _stale(objs: list[Path]) -> bool:
    if not LIB.exists():
        return True
    newest_src = max(p.stat().st_mtime for p in [*sources(), *CSRC.glob("*.cuh"), *CSRC.glob("*.h"),
                                                 *INCLUDE.glob("*.h")])
    return newest_src > LIB.stat().st_mtime


def build(force: bool = False, verbose_ptxas: bool = False) -> Path:
    """Compile every kernel for sm_100a and link libdoe_cuda.so; returns its path."""
    BUILD.mkdir(exist_ok=True)
    srcs = sources()
    if not force and not verbose_ptxas and not _stale([]):
        return LIB
    logs = []
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = []
        for obj, log in ex.map(lambda s: _compile(s, verbose_ptxas), srcs):
            objs.append(obj)
            if log.strip():
                logs.append(log)
    link = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(LIB), *map(str, objs)]
    res = subprocess.run(link, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    if verbose_ptxas:
        (BUILD / "ptxas.log").write_text("\n".join(logs))
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    args = ap.parse_args()
    lib = build(force=args.force, verbose_ptxas=args.verbose_ptxas)
    print(lib)
    if args.verbose_ptxas:
        print((BUILD / "ptxas.log").read_text())


if __name__ == "__main__":
    sys.exit(main())
