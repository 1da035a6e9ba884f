"""CPU oracle for the qmtp CUDA library -- TEST INFRASTRUCTURE ONLY.

A plain-C / numpy restatement of the arithmetic of qwen-mtp-mac's decode hot path
(aulafy/qwen-mtp-mac: qmv_kernel.py, gdn_kernel.py, gdn_fused.py, lm_head2.py, mtp.py,
experiments/deepseek_moe/kernels.py).  Only tests/, __graft_entry__.smoke() and bench.py's CPU
baseline leg may import it, and only as the checker or the timed CPU baseline -- never as a product
path.

Parity status: UNPINNED against MLX (MLX 0.31.2 / mlx-lm 0.31.3 and an Apple GPU are needed to run
the reference; neither exists here and the reference commits no golden vectors).  The reference's
own bit-level decoders and bf16 formulas are pinned by re-executing them in numpy (tests).
"""
