"""ctypes binding of libqmtp.so (the C ABI declared in include/qmtp.h).

The shared library sits next to this file and is built by ``qwen-mtp-mac_b200/build.py``.  There is
no CPU or library fallback: if the library cannot be loaded, or no CUDA device is present, every
op raises.  Arguments cross the boundary as plain device pointers, ints and the raw cudaStream_t of
torch's current stream.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libqmtp.so"

QMTP_OK = 0
_ERRORS = {
    -1: ValueError,  # QMTP_ERR_SHAPE
    -2: ValueError,  # QMTP_ERR_ALIGN
    -3: NotImplementedError,  # QMTP_ERR_UNSUPPORTED
    -4: RuntimeError,  # QMTP_ERR_CUDA
    -5: ValueError,  # QMTP_ERR_ARG
}

_P = ctypes.c_void_p
_I = ctypes.c_int
_U64 = ctypes.c_uint64
_F = ctypes.c_float

# name -> argtypes (every entry point returns int)
SIGNATURES: dict[str, list] = {
    "qmtp_version": [],
    "qmtp_device_error": [ctypes.POINTER(ctypes.c_uint), _I],
    "qmtp_qmv_affine_g64": [_P, _P, _P, _P, _P, _I, _I, _I, _I, _P],
    "qmtp_qmv_nvfp4_g16": [_P, _P, _P, _P, _I, _I, _I, _I, _P],
    "qmtp_quantize_affine_g64": [_P, _P, _P, _P, _I, _I, _P],
    "qmtp_qmv_affine_g64_split": [_P, ctypes.c_longlong, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P, ctypes.c_size_t,
                                  _P],
    "qmtp_qmv_plan": [_I, _I, _I, ctypes.POINTER(_I), ctypes.POINTER(_I), ctypes.POINTER(_I), ctypes.POINTER(_I)],
    "qmtp_qmv_set_mode": [_I],
    "qmtp_qmv_affine_g64_swiglu": [_P, ctypes.c_longlong, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P],
    "qmtp_qmv_affine_g64_gated": [_P, ctypes.c_longlong, _P, ctypes.c_longlong, _P, ctypes.c_float, _P, _P, _P, _P, _P,
                                  _I, _I, _I, _I, _P],
    "qmtp_qmv_affine_g64_norm": [_P, ctypes.c_longlong, _P, ctypes.c_float, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P,
                                 ctypes.c_size_t, _P],
}



class GdnArgs(ctypes.Structure):
    """Mirror of qmtp_gdn_args (include/qmtp.h)."""
    _fields_ = [("conv_src", _P), ("ld_conv", ctypes.c_longlong), ("conv_row_off", _P),
                ("qkv", _P), ("ld_qkv", ctypes.c_longlong), ("win_out", _P), ("win_out_row_off", _P),
                ("conv_w", _P), ("a", _P), ("b", _P), ("ld_ab", ctypes.c_longlong),
                ("A_log", _P), ("dt_bias", _P),
                ("state_in", _P), ("state_out", _P), ("state_mid", _P),
                ("ring", _P), ("ring_cur", _P), ("ring_slots", _I),
                ("y", _P),
                ("S", _I), ("Hk", _I), ("Hv", _I), ("Dk", _I), ("Dv", _I), ("KC", _I), ("snap", _I),
                ("gate_z", _P), ("ld_gate_z", ctypes.c_longlong), ("gate_w", _P), ("gate_out", _P),
                ("ld_gate_out", ctypes.c_longlong), ("gate_eps", _F), ("preload", _I)]


SIGNATURES.update({
    "qmtp_gdn_step": [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P],
    "qmtp_gdn_fused": [_P, _P, _P, _P, _I, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P],
    "qmtp_gdn_fused_ex": [ctypes.POINTER(GdnArgs), _P],
    "qmtp_gdn_set_mode": [_I],
    "qmtp_gdn_norm_gate": [_P, _P, _I, _P, _P, _I, _I, _I, _I, _F, _P],
    "qmtp_lmhead2": [_P, _P, _P, _P, _P, _I, _I, _I, _I, _P, _P, _P, _P, _P, ctypes.c_size_t, _P],
    "qmtp_topk_rescore": [_P, _I, _I, _I, _I, _P, _P, _I, _P, _P, _P, _P, ctypes.c_size_t, _P],
    "qmtp_argmax_bf16": [_P, _I, _I, _I, _P, _P, ctypes.c_size_t, _P],
    "qmtp_argmax_bf16_ids": [_P, _I, _I, _I, _P, _P, _P, _P, ctypes.c_size_t, _P],
    "qmtp_qmv_affine_g64_res": [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P],
    "qmtp_lmhead2_noalloc": [_P, _P, _P, _P, _P, _I, _I, _I, _I, _P, _P, _P, _P],
    "qmtp_lmhead2_shard": [_P, _P, _P, _P, _P, _I, _I, _I, _I, ctypes.c_longlong, _P, _P, _P, ctypes.c_size_t, _P],
    "qmtp_lmhead2_merge": [_P, _P, _I, _I, _I, _P, _P, _P, _P],
    "qmtp_lmhead2_nvfp4": [_P, _P, _P, _P, _I, _I, _I, _I, _P, _P, _P, _P, _P, ctypes.c_size_t, _P],
    "qmtp_embed": [_P, _I, _P, _P, _P, _I, _I, _P, _I, _P],
    "qmtp_embed_nvfp4": [_P, _I, _P, _P, _I, _I, _P, _I, _P],
    "qmtp_qmv_nvfp4_g16_res": [_P, _P, _P, _P, _P, _I, _I, _I, _I, _P],
    "qmtp_rmsnorm": [_P, _I, _P, _P, _F, _P, _I, _I, _I, _P],
    "qmtp_attn_prep": [_P, _I, _I, _I, _I, _I, _I, _P, _P, _F, _P, _P, _P, _I, _P, _P, _P, _P, _I, _P],
    "qmtp_attention": [_P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _I, _P, _P],
    "qmtp_embed_rmsnorm": [_P, _I, _P, _P, _P, _I, _I, _P, _I, _P, _P, _I, _P, _I, _P, _P, _P, _I, _F, _P],
    "qmtp_attention_fused": [_P, _I, _I, _I, _I, _I, _I, _P, _P, _F, _P, _P, _P, _I, _P, _P, _I, _P, _P],
    "qmtp_swiglu": [_P, _I, _I, _I, _P, _P],
    "qmtp_mtp_accept": [_P, _P, _I, _P, _P, _I, _I, _I, _I, _P],
    "qmtp_draft_prob": [_P, _I, _P, _P, _P],
    "qmtp_mtp_nuse": [_P, _I, ctypes.c_double, _P, _P],
    "qmtp_mtp_advance": [_P, _P],
    "qmtp_next_tokens": [_P, _P, _I, _P, _P, _P],
    "qmtp_quantize_fp4": [_I, _P, ctypes.c_longlong, _I, _P, _P, _P],
    "qmtp_moe_route": [_P, _I, _I, _I, _I, _F, _P, _P, _P],
    "qmtp_moe": [_I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _F, _P, ctypes.c_size_t, _P],
    "qmtp_moe_experts": [_I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _F, _P, ctypes.c_size_t, _P],
    "qmtp_moe_combine": [_P, _P, _P, _I, _I, _I, _P, _P],
    "qmtp_moe_dispatch": [_P, _I, _I, _P, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P],
    "qmtp_math_eval": [_I, _P, _I, _P, _P],
    "qmtp_wait_selftest": [ctypes.c_uint, _P, _P],
})

# control block layout (include/qmtp.h QMTP_CTRL_*)
CTRL = dict(SLOT=0, CONV_ROW=1, WOUT_ROW=2, WPAR=3, POS=4, MPOS=5, KEEP=6, SEL=7, NOUT=8, CYCLES=9, ACC0=10, NUSE=18, VERIFIED=19,
            EMIT0=20, RNG=29, SEED_LO=30, SEED_HI=31)


class SamplingArgs(ctypes.Structure):
    """Mirror of qmtp_sampling (include/qmtp.h)."""
    _fields_ = [("temperature", ctypes.c_float), ("top_k", ctypes.c_int), ("top_p", ctypes.c_float),
                ("min_p", ctypes.c_float)]


SIGNATURES["qmtp_sample"] = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                             ctypes.c_int, ctypes.c_int, ctypes.POINTER(SamplingArgs), ctypes.c_int,
                             ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
CTRL_SIZE = 32
# size queries return size_t
SIZE_QUERIES: dict[str, list] = {
    "qmtp_qmv_workspace": [_I, _I],
    "qmtp_lmhead2_workspace": [_I, _I, _I],
    "qmtp_lmhead2_shard_workspace": [_I, _I, _I],
    "qmtp_topk_workspace": [_I, _I, _I],
    "qmtp_argmax_workspace": [_I, _I],
    "qmtp_moe_workspace": [_I, _I, _I, _I, _I],
}

_lib = None
_lock = threading.Lock()


class LibraryUnavailable(RuntimeError):
    pass


def lib() -> ctypes.CDLL:
    """Loads libqmtp.so once; raises LibraryUnavailable if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise LibraryUnavailable(
                    f"{LIB_PATH} not built; run `python qwen-mtp-mac_b200/build.py` (no CPU fallback exists)")
            L = ctypes.CDLL(str(LIB_PATH))
            for name, args in SIGNATURES.items():
                f = getattr(L, name)
                f.argtypes = args
                f.restype = _I
            for name, args in SIZE_QUERIES.items():
                f = getattr(L, name)
                f.argtypes = args
                f.restype = ctypes.c_size_t
            L.qmtp_strerror.argtypes = [_I]
            L.qmtp_strerror.restype = ctypes.c_char_p
            _lib = L
    return _lib


def exported_symbols() -> list[str]:
    return [*SIGNATURES, *SIZE_QUERIES, "qmtp_strerror"]


def check(rc: int, what: str) -> None:
    if rc != QMTP_OK:
        msg = lib().qmtp_strerror(rc).decode()
        raise _ERRORS.get(rc, RuntimeError)(f"{what}: {msg} (code {rc})")


def require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("qmtp ops run on CUDA tensors only (no CPU fallback)")
        if not t.is_contiguous():
            raise ValueError("qmtp ops need contiguous tensors")


def stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def device_error(clear: bool = True) -> int:
    v = ctypes.c_uint(0)
    check(lib().qmtp_device_error(ctypes.byref(v), int(clear)), "qmtp_device_error")
    return v.value


def qmv_set_mode(mode: int) -> None:
    """Planner override of the affine qmv kernel (0 cost model, 1 whole tiles, 2 clusters, 3 workspace
    split); process-wide."""
    check(lib().qmtp_qmv_set_mode(int(mode)), "qmv_set_mode")


def qmv_plan(N: int, K: int, split: bool = True) -> dict:
    """Tiling the affine qmv kernel picks for an N x K matrix: rows per tile, CTAs, work units and
    CTAs per cluster (1: no cluster)."""
    vals = [ctypes.c_int(0) for _ in range(4)]
    check(lib().qmtp_qmv_plan(N, K, int(split), *[ctypes.byref(v) for v in vals]), "qmv_plan")
    return dict(zip(("rows_per_tile", "grid", "units", "cluster"), (v.value for v in vals)))
