"""The C-ABI library: loads without a GPU, exports every symbol include/qmtp.h declares, and the
Python binding's table agrees with the header; ops refuse CPU tensors (no fallback)."""
import ctypes
import re
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "qmtp.h"


def declared():
    txt = HEADER.read_text()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(qmtp_\w+)\s*\(", txt)))


def test_library_exports_header_symbols():
    from qmtp import _lib

    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    names = declared()
    assert names, "no declarations parsed"
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_table_matches_header():
    from qmtp import _lib

    assert sorted(_lib.exported_symbols()) == declared()


def test_strerror_and_version_without_gpu():
    from qmtp import _lib

    L = _lib.lib()
    assert L.qmtp_version() >= 100
    assert L.qmtp_strerror(-1) == b"unsupported or inconsistent sizes"


def test_ops_refuse_cpu_tensors():
    from qmtp import qmv_kernel

    x = torch.zeros(1, 1024, dtype=torch.bfloat16)
    w = torch.zeros(8, 128, dtype=torch.int32)
    s = torch.zeros(8, 16, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        qmv_kernel.qmv_affine(x, w, s, s)
