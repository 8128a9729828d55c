"""Build libdoe_cuda.so and the ONNX Runtime plugin EP in-tree for sm_100a.

    python -m doe_b200.build [--verbose-ptxas]

Every translation unit under doe_b200/csrc is compiled by nvcc for
`-gencode arch=compute_100a,code=sm_100a` and linked (with the CUDA runtime
linked statically) into doe_b200/libdoe_cuda.so, which ships beside the
package.  Object files go to doe_b200/_build/.

doe_b200/ort_ep/doe_ort_ep.cpp is compiled by g++ into
doe_b200/libdoe_ort_ep.so (CreateEpFactories / ReleaseEpFactory), linked
against libdoe_cuda.so and the shared CUDA runtime (the static one carries
its own copy of the C++ exception runtime, which the EP's error handling must
not pick up).  It needs ONNX Runtime's C API headers
(onnxruntime_c_api.h and onnxruntime_ep_c_api.h, API version 23 or later):
the directory named by ORT_INCLUDE_DIR, else the copy the doerun/doe tree
vendors under runtime/bridge/onnxruntime-ep/vendor/onnxruntime/include when
that tree is at DOE_REFERENCE_ROOT (default /root/reference).  Without the
headers the EP library is skipped, or kept if it was built before.
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


EP_SRC = PKG / "ort_ep" / "doe_ort_ep.cpp"
EP_LIB = PKG / "libdoe_ort_ep.so"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))


def ort_include_dir() -> Path | None:
    """ONNX Runtime's C API header directory (see the module docstring)."""
    cands = []
    if os.environ.get("ORT_INCLUDE_DIR"):
        cands.append(Path(os.environ["ORT_INCLUDE_DIR"]))
    ref = Path(os.environ.get("DOE_REFERENCE_ROOT", "/root/reference"))
    cands.append(ref / "runtime" / "bridge" / "onnxruntime-ep" / "vendor" / "onnxruntime" / "include")
    for c in cands:
        if (c / "onnxruntime_c_api.h").exists() and (c / "onnxruntime_ep_c_api.h").exists():
            return c
    return None


def host_cxx() -> str:
    """The C++ compiler for the host-side libraries: DOE_CXX, else the system
    g++.  Not $CXX: a toolchain that links libstdc++ statically would give a
    library its own copy of the C++ runtime (exception handling included)
    inside a process that already has the shared one."""
    for cand in (os.environ.get("DOE_CXX"), "/usr/bin/g++", shutil.which("g++")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("no C++ compiler for libdoe_ort_ep.so (set DOE_CXX)")


def build_ort_ep(force: bool = False) -> Path | None:
    """Compile libdoe_ort_ep.so (needs libdoe_cuda.so and the ORT headers)."""
    inc = ort_include_dir()
    if inc is None:
        return EP_LIB if EP_LIB.exists() else None
    if (not force and EP_LIB.exists() and EP_LIB.stat().st_mtime >= max(
            EP_SRC.stat().st_mtime, LIB.stat().st_mtime, (INCLUDE / "doe_cuda.h").stat().st_mtime)):
        return EP_LIB
    cmd = [host_cxx(), "-std=c++17", "-O2", "-g", "-fPIC", "-shared", "-Wall", "-Wextra", "-fvisibility=hidden",
           "-I", str(inc), "-I", str(INCLUDE), "-I", str(CUDA_HOME / "include"), str(EP_SRC),
           "-o", str(EP_LIB), "-L", str(PKG), "-ldoe_cuda", "-L", str(CUDA_HOME / "lib64"), "-lcudart",
           f"-Wl,-rpath,$ORIGIN:{CUDA_HOME / 'lib64'}"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"g++ failed on {EP_SRC.name}:\n{res.stdout}\n{res.stderr}")
    return EP_LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    args = ap.parse_args()
    lib = build(force=args.force, verbose_ptxas=args.verbose_ptxas)
    print(lib)
    print(build_ort_ep(force=args.force) or "libdoe_ort_ep.so skipped: no ONNX Runtime headers")
    if args.verbose_ptxas:
        print((BUILD / "ptxas.log").read_text())


if __name__ == "__main__":
    sys.exit(main())
