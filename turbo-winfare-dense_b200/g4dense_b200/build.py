"""Builds libg4dense_b200.so in-tree with nvcc for sm_100a.

Every .cu/.cpp under csrc/ is compiled (in parallel, incrementally) into _build/ and linked
into g4dense_b200/lib/libg4dense_b200.so together with a static CUDA runtime. nvcc
cross-compiles, so this runs on machines without a GPU.
"""
from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent          # .../turbo-winfare-dense_b200/g4dense_b200
ROOT = PKG.parent                               # .../turbo-winfare-dense_b200
REPO = ROOT.parent
CSRC = ROOT / "csrc"
BUILD = ROOT / "_build"
LIB = PKG / "lib" / "libg4dense_b200.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nccl_paths():
    """(include dir, lib dir) of an NCCL install: torch's bundled wheel first, then the system."""
    try:
        import nvidia.nccl  # type: ignore
        base = Path(list(nvidia.nccl.__path__)[0])
        if (base / "include" / "nccl.h").exists():
            return base / "include", base / "lib"
    except Exception:
        pass
    for inc, lib in [("/usr/include", "/usr/lib/x86_64-linux-gnu"), ("/usr/local/cuda/include", "/usr/local/cuda/lib64")]:
        if Path(inc, "nccl.h").exists():
            return Path(inc), Path(lib)
    return None, None


def _flags():
    inc = ["-I", str(CSRC), "-I", str(REPO / "include")]
    nccl_inc, _ = _nccl_paths()
    if nccl_inc:
        inc += ["-I", str(nccl_inc), "-DG4B_HAVE_NCCL=1"]
    common = ["-O3", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden", "-lineinfo"] + inc
    return common


def _compile(src: Path, verbose: bool) -> Path:
    obj = BUILD / (src.name + ".o")
    deps = [src] + sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + sorted((REPO / "include").rglob("*.h"))
    if obj.exists() and obj.stat().st_mtime >= max(d.stat().st_mtime for d in deps):
        return obj
    cmd = [NVCC] + ARCH + _flags() + ["-c", str(src), "-o", str(obj)]
    if src.suffix == ".cu":
        cmd += ["-Xptxas", "-v"] if verbose else []
    else:
        cmd = [NVCC] + _flags() + ["-x", "c++", "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {src.name}\n{r.stderr[-6000:]}")
    if verbose and r.stderr:
        sys.stderr.write(r.stderr)
    return obj


def build(verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    LIB.parent.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    newest = max(o.stat().st_mtime for o in objs)
    if LIB.exists() and LIB.stat().st_mtime >= newest:
        return LIB
    _, nccl_lib = _nccl_paths()
    link = [NVCC] + ARCH + ["-shared", "-cudart", "static", "-o", str(LIB)] + [str(o) for o in objs]
    if nccl_lib:
        link += ["-L", str(nccl_lib), "-Xlinker", f"-rpath,{nccl_lib}", "-l:libnccl.so.2"]
    link += ["-lcuda"]
    r = subprocess.run(link, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed\n{r.stderr[-6000:]}")
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
