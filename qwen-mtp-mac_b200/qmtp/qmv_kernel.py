"""Multi-row 4-bit quantized GEMV on B200 -- the qmv_kernel.py surface of qwen-mtp-mac.

Reference: qmv_kernel.py:86-101 (``qmv_nvfp4(x, w, s, rows=None, nsg=1)``), qmv_kernel.py:104-120
(the ``QuantizedLinear.__call__`` patch and ``install``) and MLX's
``quantized_matmul(x, w, scales, biases, transpose=True, group_size=64, bits=4)`` for the affine
format the B200 build is judged on.

Every call runs an sm_100a kernel of libqmtp: the affine format on the tensor cores (csrc/qmv_tc.cu,
tcgen05 kind::i8 with exact integer group sums), NVFP4 on the CUDA cores (csrc/qmv.cu).  Unlike the
reference there is no "fall back to the library path" branch: the kernels read each weight once for
any number of rows, so ``install`` only records the row window for API compatibility.
"""
from __future__ import annotations

import torch

from . import _lib

MIN_ROWS, MAX_ROWS = 3, 4  # reference defaults (qmv_kernel.py:105); informational here
GROUP_SIZE = 64

def _flat(x: torch.Tensor):
    K = x.shape[-1]
    return x.reshape(-1, K), K


def quantize(w: torch.Tensor, group_size: int = 64, bits: int = 4, mode: str = "affine"):
    """``mx.quantize`` for the affine 4-bit group-64 format: bf16 [N, K] -> (wq uint32 [N, K/8],
    scales bf16 [N, K/64], biases bf16 [N, K/64]).  Runs on the GPU (libqmtp quantizer)."""
    if mode != "affine" or bits != 4 or group_size != 64:
        raise NotImplementedError("only affine 4-bit group-64 quantization is implemented on the GPU")
    _lib.require_cuda(w)
    if w.dtype != torch.bfloat16 or w.dim() != 2:
        raise ValueError("quantize expects a 2-D bf16 tensor")
    N, K = w.shape
    wq = torch.empty((N, K // 8), dtype=torch.int32, device=w.device)
    sc = torch.empty((N, K // 64), dtype=torch.bfloat16, device=w.device)
    bi = torch.empty((N, K // 64), dtype=torch.bfloat16, device=w.device)
    _lib.check(_lib.lib().qmtp_quantize_affine_g64(w.data_ptr(), wq.data_ptr(), sc.data_ptr(), bi.data_ptr(),
                                                    N, K, _lib.stream()), "quantize")
    return wq, sc, bi


def qmv_affine_swiglu(gu: torch.Tensor, w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                      out: torch.Tensor | None = None, res: torch.Tensor | None = None) -> torch.Tensor:
    """y = (silu(gate) * up) @ dequant(w).T with gu = [gate | up] bf16 [M, 2K] (the MLP's down
    projection with its SwiGLU computed in the kernel's prologue)."""
    M, K2 = gu.shape
    K, N = K2 // 2, w.shape[0]
    _lib.require_cuda(gu, w, scales, biases, res)
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=gu.device)
    _lib.check(_lib.lib().qmtp_qmv_affine_g64_swiglu(gu.data_ptr(), gu.stride(0), w.data_ptr(), scales.data_ptr(),
                                                      biases.data_ptr(), out.data_ptr(), _lib.ptr(res), M, N, K,
                                                      out.shape[-1], _lib.stream()), "qmv_affine_swiglu")
    return out


def qmv_affine_gated(yg: torch.Tensor, z: torch.Tensor, norm_w: torch.Tensor, eps: float, w: torch.Tensor,
                     scales: torch.Tensor, biases: torch.Tensor, out: torch.Tensor | None = None,
                     res: torch.Tensor | None = None) -> torch.Tensor:
    """y = bf16(RMSNorm_head(yg) * silu(z)) @ dequant(w).T over heads of 128 (the GatedDeltaNet output
    gate computed in the out-projection's prologue); yg fp32 [M, K], z bf16 [M, >=K] (row stride any)."""
    M, K = yg.shape
    N = w.shape[0]
    _lib.require_cuda(yg, norm_w, w, scales, biases, res)
    if not z.is_cuda or z.stride(-1) != 1 or z.dtype != torch.bfloat16:
        raise ValueError("z must be a bf16 CUDA tensor with unit stride along its rows")
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=yg.device)
    _lib.check(_lib.lib().qmtp_qmv_affine_g64_gated(yg.data_ptr(), yg.stride(0), z.data_ptr(), z.stride(0),
                                                     norm_w.data_ptr(), float(eps), w.data_ptr(), scales.data_ptr(),
                                                     biases.data_ptr(), out.data_ptr(), _lib.ptr(res), M, N, K,
                                                     out.shape[-1], _lib.stream()), "qmv_affine_gated")
    return out


def qmv_affine(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
               group_size: int = 64, out: torch.Tensor | None = None, res: torch.Tensor | None = None,
               ws: torch.Tensor | None = None, split: bool = True, norm=None) -> torch.Tensor:
    """y = x @ dequant(w).T for the affine 4-bit group-64 format (bf16 in, bf16 out).
    x: [..., K] bf16; w: uint32/int32 [N, K/8]; scales, biases: bf16 [N, K/64] -> [..., N].
    res (bf16, same shape as out): y = bf16(res + bf16(x . W^T)), may alias out.
    split=True (default) calls the strided entry point (qmtp_qmv_affine_g64_split), split=False the
    plain ones; both give the same bits, and either may share a tile between the CTAs of a cluster.
    ws: accepted for compatibility, not needed.
    norm=(weight bf16 [K], eps): x is first RMS-normalised (mlx_lm RMSNorm) inside the kernel."""
    if group_size != 64:
        raise NotImplementedError("affine qmv is implemented for group_size=64")
    xf, K = _flat(x)
    N = w.shape[0]
    M = xf.shape[0]
    if x.dtype != torch.bfloat16:
        raise ValueError("qmv_affine expects bf16 activations")
    _lib.require_cuda(xf, w, scales, biases, res)
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    elif out.dim() != 2 or out.shape[0] != M or out.shape[1] < N or out.dtype != torch.bfloat16:
        raise ValueError("out must be bf16 [M, >=N]")
    if res is not None and (res.shape != out.shape or res.dtype != torch.bfloat16):
        raise ValueError("res must match out")
    L = _lib.lib()
    if norm is not None:
        nw, eps = norm
        _lib.require_cuda(nw)
        rc = L.qmtp_qmv_affine_g64_norm(xf.data_ptr(), K, nw.data_ptr(), float(eps), w.data_ptr(), scales.data_ptr(),
                                        biases.data_ptr(), out.data_ptr(), _lib.ptr(res), M, N, K, out.shape[-1],
                                        None, 0, _lib.stream())
    elif split:
        rc = L.qmtp_qmv_affine_g64_split(xf.data_ptr(), K, w.data_ptr(), scales.data_ptr(), biases.data_ptr(),
                                         out.data_ptr(), _lib.ptr(res), M, N, K, out.shape[-1], None, 0,
                                         _lib.stream())
    elif res is not None:
        rc = L.qmtp_qmv_affine_g64_res(xf.data_ptr(), w.data_ptr(), scales.data_ptr(), biases.data_ptr(),
                                       out.data_ptr(), res.data_ptr(), M, N, K, out.shape[-1], _lib.stream())
    else:
        rc = L.qmtp_qmv_affine_g64(xf.data_ptr(), w.data_ptr(), scales.data_ptr(), biases.data_ptr(),
                                   out.data_ptr(), M, N, K, out.shape[-1], _lib.stream())
    _lib.check(rc, "qmv_affine")
    if out.shape[-1] != N:  # caller-provided wider output (leading dimension ldy > N)
        return out[:, :N]
    return out.reshape(*x.shape[:-1], N)


def qmv_nvfp4(x: torch.Tensor, w: torch.Tensor, s: torch.Tensor, rows=None, nsg=1) -> torch.Tensor:
    """Reference signature (qmv_kernel.py:86): x [..., K] bf16, w uint32 [N, K/8] e2m1 nibbles,
    s uint8 [N, K/16] e4m3 scales -> [..., N].  ``rows``/``nsg`` were Metal tiling knobs; the B200
    kernel picks its own tiling, so they are accepted and ignored."""
    xf, K = _flat(x)
    N = w.shape[0]
    M = xf.shape[0]
    _lib.require_cuda(xf, w, s)
    out = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    _lib.check(_lib.lib().qmtp_qmv_nvfp4_g16(xf.data_ptr(), w.data_ptr(), s.data_ptr(), out.data_ptr(), M, N, K,
                                              N, _lib.stream()), "qmv_nvfp4")
    return out.reshape(*x.shape[:-1], N)


class QuantizedLinear:
    """Bias-free 4-bit linear layer (the module the reference patches, qmv_kernel.py:108-113)."""

    def __init__(self, weight, scales, biases=None, group_size=64, bits=4, mode="affine"):
        self.weight, self.scales, self.biases = weight, scales, biases
        self.group_size, self.bits, self.mode = group_size, bits, mode
        self.out_features = weight.shape[0]
        self.in_features = weight.shape[1] * 8

    @classmethod
    def from_linear(cls, w_bf16: torch.Tensor, group_size=64, bits=4, mode="affine"):
        wq, s, b = quantize(w_bf16, group_size, bits, mode)
        return cls(wq, s, b, group_size, bits, mode)

    def __call__(self, x, out=None):
        if self.mode == "affine":
            return qmv_affine(x, self.weight, self.scales, self.biases, self.group_size, out=out)
        if self.mode == "nvfp4":
            return qmv_nvfp4(x, self.weight, self.scales)
        raise NotImplementedError(self.mode)

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.weight, self.scales, self.biases) if t is not None)


def install(min_rows: int = 3, max_rows: int = 4) -> None:
    """API parity with qmv_kernel.py:116.  Records the row window; QuantizedLinear here always uses
    the B200 kernel (there is no second, slower path to route to)."""
    global MIN_ROWS, MAX_ROWS
    MIN_ROWS, MAX_ROWS = min_rows, max_rows
