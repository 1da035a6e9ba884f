"""qmtp -- B200-native (sm_100a) decode hot path of qwen-mtp-mac.

Modules mirror the reference's Python surface (aulafy/qwen-mtp-mac):
  qmv_kernel   multi-row 4-bit GEMV (affine g64, NVFP4 g16)        <- qmv_kernel.py
and are backed by libqmtp.so (C ABI in include/qmtp.h, kernels in csrc/).
"""
__version__ = "0.1.0"
