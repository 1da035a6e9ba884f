"""Builds the C oracle (qmtp_oracle.c) into oracle/_build/libqmtp_oracle.so with gcc.

-ffp-contract=off keeps every fp32 operation exactly as written (explicit fmaf only); -mfma makes
fmaf a single instruction.  The reference has no C/C++ sources to compile (it is Python + Metal
strings), so there is no oracle/_ref build."""
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "qmtp_oracle.c"
OUT = HERE / "_build" / "libqmtp_oracle.so"
FLAGS = ["-O2", "-std=c11", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off", "-fno-fast-math",
         "-mfma", "-mavx2", "-Wall", "-Wno-unused-function"]


def build(force: bool = False) -> Path:
    OUT.parent.mkdir(exist_ok=True)
    if force or not OUT.exists() or OUT.stat().st_mtime < SRC.stat().st_mtime:
        r = subprocess.run(["gcc", *FLAGS, str(SRC), "-o", str(OUT), "-lm"], capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"oracle build failed:\n{r.stderr}")
    return OUT


if __name__ == "__main__":
    print(build("--force" in sys.argv))
