"""qmtp -- B200-native (sm_100a) decode hot path of qwen-mtp-mac.

Modules mirror the reference's Python surface (aulafy/qwen-mtp-mac):
  qmv_kernel   multi-row 4-bit GEMV (affine g64, NVFP4 g16)            <- qmv_kernel.py
  gdn_kernel   GatedDeltaNet recurrence with per-token snapshots      <- gdn_kernel.py
  gdn_fused    conv + norms + gates + recurrence of the verify step    <- gdn_fused.py
  lm_head2     two-stage lm_head, k_for                                <- lm_head2.py
  mtp          MTP decoder: greedy or sampled verify, prefix cache     <- mtp.py, engine.py
  loader       safetensors / Ollama checkpoints -> decoder weights     <- qwen_ollama.py, mtp.py:61-70
  moe, moe_ep  MXFP4 / NVFP4 expert decode, expert parallelism         <- experiments/deepseek_moe
and are backed by libqmtp.so (C ABI in include/qmtp.h, kernels in csrc/).
"""
__version__ = "0.1.0"
