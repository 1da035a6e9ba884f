"""Builds libqmtp.so (all CUDA kernels + the C ABI of include/qmtp.h) for sm_100a, in-tree.

    python qwen-mtp-mac_b200/build.py [--force] [-j N]

Each csrc/*.cu is compiled to _build/*.o (skipped when newer than its sources), then linked into
qmtp/libqmtp.so next to the Python package, so the library travels with the repository snapshot.
"""
import argparse
import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
OUT = PKG / "qmtp" / "libqmtp.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

# -fmad=false: no implicit fma contraction; kernels spell out every fma they want (bit-exactness
# with the CPU oracle).  Default precise division / sqrt, no flush-to-zero.
NVCC_FLAGS = [
    "-O3", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo",
    "-fmad=false", "-Xcompiler", "-fPIC,-O2", "--expt-relaxed-constexpr",
    "-I", str(ROOT / "include"),
]


def _deps(src: Path):
    return [src, *sorted(CSRC.glob("*.cuh")), ROOT / "include" / "qmtp.h"]


def _stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(d.stat().st_mtime > t for d in _deps(src) if d.exists())


def _compile(src: Path, verbose: bool):
    obj = BUILD / (src.stem + ".o")
    cmd = [NVCC, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(force: bool = False, jobs: int = 8, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    todo = [s for s in srcs if force or _stale(BUILD / (s.stem + ".o"), s)]
    logs = []
    with cf.ThreadPoolExecutor(max_workers=max(1, jobs)) as ex:
        for obj, log in ex.map(lambda s: _compile(s, verbose), todo):
            logs.append(log)
    objs = [BUILD / (s.stem + ".o") for s in srcs]
    if todo or not OUT.exists() or force:
        cmd = [NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", str(OUT), *map(str, objs)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    if verbose:
        for log in logs:
            sys.stderr.write(log)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=8)
    ap.add_argument("-v", action="store_true", help="print ptxas register/spill reports")
    a = ap.parse_args()
    print(build(a.force, a.j, a.v))
