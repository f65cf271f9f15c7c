"""Build libtops_gla.so in-tree with nvcc for sm_100a.

    python pallas-kernel_b200/build.py [--debug] [--jobs N]

Every .cu under csrc/ is compiled to an object (in parallel) and linked into
pallas-kernel_b200/tops/_lib/libtops_gla.so.  Objects are rebuilt when their
source or any header is newer.  No GPU is needed (nvcc cross-compiles).
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INC = HERE.parent / "include"
OUT = HERE / "tops" / "_lib"
OBJ = HERE / "_build"
LIB = OUT / "libtops_gla.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def nccl_include() -> str | None:
    """Directory of nccl.h (the nvidia-nccl wheel torch ships with, or the system's)."""
    try:
        import nvidia.nccl as n  # type: ignore
        for p in n.__path__:
            if (Path(p) / "include" / "nccl.h").exists():
                return str(Path(p) / "include")
    except ImportError:
        pass
    for p in ("/usr/include", "/usr/local/cuda/include"):
        if (Path(p) / "nccl.h").exists():
            return p
    return None


def _flags(debug: bool) -> list[str]:
    f = ARCH + ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
                "--expt-relaxed-constexpr", "-I", str(INC), "-I", str(CSRC)]
    inc = nccl_include()
    if inc is None:
        raise RuntimeError("nccl.h not found (needed for the state-exchange entry points)")
    f += ["-I", inc]
    if debug:
        f += ["-DTOPS_DEBUG=1"]
    return f


def _newest_header() -> float:
    hs = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INC.glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def build(debug: bool = False, jobs: int | None = None, verbose: bool = False) -> Path:
    OUT.mkdir(parents=True, exist_ok=True)
    OBJ.mkdir(parents=True, exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    hdr = _newest_header()
    cc = nvcc()
    flags = _flags(debug)

    def one(src: Path) -> Path:
        obj = OBJ / (src.stem + ".o")
        if obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, hdr):
            return obj
        cmd = [cc, *flags, "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
        if verbose and r.stderr.strip():
            print(r.stderr, flush=True)
        return obj

    with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(one, srcs))
    newest = max(o.stat().st_mtime for o in objs)
    if not LIB.exists() or LIB.stat().st_mtime < newest:
        # static cudart (nvcc's default): no libcudart/libcuda link-time dependency, so the
        # library loads on machines without a GPU; the driver is opened on first use.
        cmd = [cc, *ARCH, "-shared", "--cudart", "static", "-o", str(LIB), *map(str, objs)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--debug", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.debug, a.jobs, a.verbose))
    sys.exit(0)
