"""Benchmark of the B200 decode hot path: greedy MTP speculative decoding (the config-4 workload).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one verify cycle of mtp.py:268-294 on the synthetic Qwen3.5-9B-shaped model (32 layers,
3:1 GatedDeltaNet : gated attention, 4-bit affine g64 weights, two-stage lm_head, 1-layer MTP head,
k = 2 drafts, batch 1) after a 512-token uniform-random prompt.  Prints one JSON line on rank 0.

  value      tokens emitted per second over K graph replays, device-timed with CUDA events (the
             replays run back to back, no host round trip);
  e2e        the same tokens/s through qmtp.mtp.decode_mtp, the call a user makes: one replay,
             stream sync and 128-byte control-block read per cycle, as the reference's loop does;
  roofline   the 4-bit GEMV (qmv) kernels: algorithmic bytes of every qmv launch of one cycle over
             their CUDA-event durations, against the measured HBM copy peak;
  cpu_baseline  the C oracle (oracle/) running the same decode cycles from the GPU's post-prefill
             state on the host cores (bounded sample), with a token-for-token parity check.

--impl reference: the reference's CPU path restated by the oracle (the reference itself is MLX +
Metal and cannot run here), full-size weights, the same 512-token prompt (prefilled in one oracle
pass), W + K cycles on all host cores.
Multi-GPU: replicas of the decode (batch-1 decoding does not shard; every rank decodes its own
prompt), and in the same line ("moe_ep") config 5's MoE layer expert-parallel over the same ranks.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path[:0] = [str(ROOT), str(ROOT / "qwen-mtp-mac_b200")]

METRIC = "MTP greedy decode tok/s (batch 1); qmv/GDN achieved HBM GB/s vs roofline"
PROMPT_LEN, K_DRAFTS = 512, 2


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return float(d["hbm_gbs"]), "measured"
        except Exception:
            pass
    return 6650.0, "fallback"


def _traffic_ratio(summary="qmv_affine_g64_inproj_M3.md"):
    """DRAM bytes / algorithmic bytes of the qmv kernel from the committed ncu summary, if any."""
    p = ROOT / "profiles" / summary
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("traffic_ratio:"):
            try:
                return float(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi samples (200 ms) during the timed region: median SM MHz and active throttle reasons."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.f = None

    def __enter__(self):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        self.f.flush()

    def summary(self):
        rows = []
        try:
            for line in Path(self.f.name).read_text().splitlines():
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        finally:
            os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "", 1).isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "", 1).isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------------------------------ our arm
def run_ours(args):
    import numpy as np
    import torch
    import torch.distributed as dist

    from qmtp import _lib
    from qmtp import model as qm
    from qmtp.mtp import MTPDecoder, Sampling, _restore, _snapshot, export_state, decode_mtp

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    cfg = qm.ModelArgs(max_pos=2048)
    t_build = time.time()
    W = qm.synthetic_weights(cfg, seed=0, device=dev, fmt=args.weights)
    torch.cuda.synchronize()
    t_build = time.time() - t_build
    rng = np.random.default_rng(1000 + rank)
    prompt = rng.integers(0, cfg.vocab, args.prompt).tolist()
    K, Wu = args.steps, args.warmup
    sp = (Sampling(args.temperature, args.top_k, args.top_p, args.min_p, args.seed) if args.temperature > 0
          else None)
    gen_tokens = 256  # config 4 generates 256 tokens; the e2e leg decodes all of them
    dec = MTPDecoder(cfg, W, k=K_DRAFTS, max_tokens=max(Wu + 3 * K + 64, gen_tokens + 64), device=dev,
                     sampling=sp)
    if args.draft_vocab:
        # draft head over the first draft_vocab ids (mtp.py:170-196 load_draft_head; the reference's
        # bench_ab.py compares such heads with the full one).  Config 4 itself drafts over the full head.
        from qmtp.mtp import load_draft_head

        dec.set_draft_head(load_draft_head(args.draft_vocab, {"bits": 4, "group_size": 64}, lm=qm.Model(cfg, W)))

    # ---- prefill, one eager cycle (library setup), capture
    t = dec.prefill(prompt)
    post_prefill = export_state(dec) if (rank == 0 and world == 1 and args.cpu_cycles > 0) else None
    snap = _snapshot(dec)
    dec.launches = 0
    dec.run_cycle()
    launches_per_cycle = dec.launches
    # roofline: the 4-bit projections of one cycle (same order, shapes and buffers) captured alone
    # in a CUDA graph and timed with CUDA events over back-to-back replays on the launch stream
    dec.prof = []
    dec.qmv_log = []
    dec.run_cycle()
    torch.cuda.synchronize()
    prof = [(b, shp) for b, _, _, shp in dec.prof]
    qlog, dec.prof, dec.qmv_log = dec.qmv_log, None, None
    qstream = torch.cuda.Stream(dev)
    qstream.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(qstream):
        for args_ in qlog:
            dec._qmv(*args_)
    qgraph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(qgraph, stream=qstream):
        for args_ in qlog:
            dec._qmv(*args_)
    torch.cuda.current_stream(dev).wait_stream(qstream)
    for _ in range(3):
        qgraph.replay()
    qe0, qe1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    q_reps = 20
    qe0.record()
    for _ in range(q_reps):
        qgraph.replay()
    qe1.record()
    torch.cuda.synchronize()
    qmv_ms_cycle = qe0.elapsed_time(qe1) / q_reps
    del qgraph
    _restore(dec, snap)
    dec.capture()
    _restore(dec, snap)
    # warm-up replays (their tokens are the first W cycles of the generation)
    for _ in range(Wu):
        dec.run_cycle()
    n0 = int(dec.ctrl[_lib.CTRL["NOUT"]])

    # ---- timed region: K back-to-back graph replays
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push("timed")
        ev0.record()
        for _ in range(K):
            dec.graph.replay()
        ev1.record()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
    elapsed_ms = ev0.elapsed_time(ev1)
    n1 = int(dec.ctrl[_lib.CTRL["NOUT"]])
    tokens = n1 - n0
    gpu_stream = dec.out_tokens[:n1].tolist()  # every token decoded after the prompt (warm-up + timed)
    clocks = clk.summary()
    if world > 1:
        tt = torch.tensor([elapsed_ms, float(tokens)], dtype=torch.float64, device=dev)
        mx = tt.clone()
        dist.all_reduce(mx[:1], op=dist.ReduceOp.MAX)
        dist.all_reduce(tt[1:], op=dist.ReduceOp.SUM)
        elapsed_ms, tokens_all = float(mx[0]), float(tt[1])
    else:
        tokens_all = float(tokens)
    value = tokens_all / (elapsed_ms / 1e3)

    # ---- e2e: the public decode_mtp call (per-cycle host sync + control-block read), config 4's 256 tokens
    out, st = decode_mtp(dec, prompt, gen_tokens, use_graph=True)
    e2e_tps = st["tps"]
    if world > 1:
        e = torch.tensor([st["seconds"], float(len(out) - 1)], dtype=torch.float64, device=dev)
        dist.all_reduce(e[:1], op=dist.ReduceOp.MAX)
        tot = e[1:].clone()
        dist.all_reduce(tot, op=dist.ReduceOp.SUM)
        e2e_tps = float(tot[0]) / float(e[0])

    peak, peak_kind = _peaks()
    qbytes = sum(b for b, _ in prof)
    achieved = qbytes / (qmv_ms_cycle / 1e3) / 1e9
    tsum = "qmv_affine_g64_inproj_M3.md" if args.weights == "affine" else "qmv_nvfp4_g16_head_M1.md"
    ratio = _traffic_ratio(tsum)
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                "traffic": None if ratio is None else round(ratio * qbytes / len(prof)),
                "traffic_source": f"DRAM bytes / algorithmic bytes of one launch in profiles/{tsum} (ncu), times "
                                  "this cycle's mean algorithmic bytes per launch",
                "kernel": ("qmv_affine_g64" if args.weights == "affine" else "qmv_nvfp4_g16 (trunk) + qmv_affine_g64 (coarse head)")
                          + " (all 4-bit projections + coarse head of a cycle)",
                "bytes_per_cycle": qbytes, "qmv_ms_per_cycle": round(qmv_ms_cycle, 4),
                "launches_per_cycle": len(prof),
                "timing": "the cycle's projections alone in a CUDA graph, back-to-back replays"}

    res = {"metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": Wu,
           "ms_per_step": round(elapsed_ms / K, 4), "higher_is_better": True, "scaling": "weak",
           "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
           "config": {"workload": "config4: synthetic Qwen3.5-9B-shaped hybrid decoder (32 layers, 3:1 GDN:attention, "
                                  + ("4-bit affine g64" if args.weights == "affine" else "4-bit NVFP4 g16")
                                  + "), 1-layer MTP head, "
                                  + ("greedy" if sp is None else "exact speculative sampling")
                                  + f" MTP decode k=2, batch 1, {args.prompt}-token uniform random prompt",
                      "step": "one verify cycle (verify 3 tokens + accept/rollback + 2 draft steps)",
                      "prompt_tokens": args.prompt, "drafts": K_DRAFTS, "parallelism": f"replicas x{world}",
                      "draft_head": (f"first {args.draft_vocab} ids (load_draft_head)" if args.draft_vocab
                                     else "full vocabulary"),
                      "l2": "weights ~7.5 GB per cycle >> 126 MB L2 (no flush needed)",
                      "weights_build_s": round(t_build, 1),
                      **({} if sp is None else {"sampling": {"temperature": sp.temperature, "top_k": sp.top_k,
                                                             "top_p": sp.top_p, "min_p": sp.min_p,
                                                             "seed": sp.seed, "head_candidates": dec.K}})},
           "e2e": {"value": round(e2e_tps, 2), "unit": "tok/s", "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 4 * _lib.CTRL_SIZE, "tokens": len(out),
                   "h2d_note": "a decode cycle takes no host input: the prompt is copied once before the "
                               "timed region and every later token is produced on the device; each cycle "
                               "reads the 128-byte control block (emitted tokens) back to the host"},
           "roofline": roofline, "clocks": clocks, "gpu_launches": launches_per_cycle * K,
           "stats": {"tokens_timed": int(tokens_all), "tok_per_cycle": round(tokens / K, 4),
                     "acceptance": st["acept"], "first_token": t}}

    # ---- CPU oracle on a bounded sample of the same decode, from the same post-prefill state
    if post_prefill is not None:
        res["cpu_baseline"] = cpu_baseline_from_state(cfg, W, post_prefill, gpu_stream, args.cpu_cycles, sp,
                                                      args.draft_vocab)
    if world > 1:
        # the sharded workload of the build: config 5's MoE layer expert-parallel over the same ranks
        dist.barrier()
        dec.graph = None
        del dec, W
        torch.cuda.empty_cache()
        res["moe_ep"] = moe_ep_measure(args, dev, rank, world)
        dist.barrier()
        res["lmhead_shard"] = head_shard_measure(args, dev, rank, world)
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(res), flush=True)


def cpu_baseline_from_state(cfg, W, state, gpu_tokens, cycles, sampling=None, draft_vocab=0):
    import numpy as np

    from oracle import model as om
    from qmtp import model as qm

    threads = os.cpu_count() or 1
    t0 = time.time()
    Wn = qm.to_numpy(W)
    ocfg = om.ModelArgs(**{k: getattr(cfg, k) for k in om.ModelArgs.__dataclass_fields__})
    orc = om.OracleModel(ocfg, Wn)
    if draft_vocab:
        orc.set_draft_head(draft_vocab)
    layers, mtp, pending = state
    cache, mcache = orc.load_state(layers, mtp)
    copy_s = time.time() - t0
    # with sampling, the first verify cycle after the prompt uses Philox call counter 1 (0 drew the first token)
    out, st = orc.decode(cache, mcache, pending[0], pending[1:], max_tokens=10 ** 6, k=K_DRAFTS, max_cycles=cycles,
                         sampling=sampling, rng_ctr=1)
    got = out[1:]
    ref = gpu_tokens[:len(got)]
    return {"value": round(st["tps"], 4), "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"{cycles} decode cycles of the full-size model from the GPU's post-prefill state "
                      f"({st['tokens']} tokens, {st['seconds']:.1f} s; weights/state copy {copy_s:.1f} s not timed)",
            "parity": {"cycles": cycles, "tokens": len(got), "identical": got == ref}}


# ------------------------------------------------------------------------------ single kernels
def run_kernel(args):
    """Standalone timing of one kernel at a BASELINE config shape (graph-captured launches, weights
    rotated over enough copies to exceed L2).  Used for the ncu captures and the per-kernel numbers."""
    import numpy as np
    import torch

    from qmtp import _lib, qmv_kernel
    from qmtp.lm_head2 import TwoStageHead

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    peak, peak_kind = _peaks()
    K, Wu = args.steps, args.warmup
    if args.kernel == "qmv":
        parts = args.shape.split(",")
        N, Kd, M = (int(v) for v in parts[:3])
        fmt = parts[3] if len(parts) > 3 else "affine"
        copies = max(1, -(-300_000_000 // (N * Kd // 2)))  # > 2x L2 of weights in rotation
        x = torch.randn(M, Kd, generator=g, device=dev).to(torch.bfloat16)
        y = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
        if fmt == "nvfp4":
            from qmtp import moe

            Ls = []
            for _ in range(copies):
                wq_, s_ = moe.quantize((torch.randn(1, N, Kd, generator=g, device=dev) * 0.02).to(torch.bfloat16),
                                       "nvfp4")
                Ls.append((wq_[0], s_[0]))
            nbytes = N * Kd // 2 + N * (Kd // 16) + M * Kd * 2 + M * N * 2
            run = lambda i: qmv_kernel.qmv_nvfp4(x, *Ls[i % copies])
            label = f"qmv NVFP4 g16 N={N} K={Kd} M={M}"
        else:
            Ls = [qmv_kernel.quantize((torch.randn(N, Kd, generator=g, device=dev) * 0.02).to(torch.bfloat16))
                  for _ in range(copies)]
            nbytes = N * Kd // 2 + N * (Kd // 64) * 4 + M * Kd * 2 + M * N * 2
            if fmt == "affine-whole":
                _lib.qmv_set_mode(1)
            run = lambda i: qmv_kernel.qmv_affine(x, *Ls[i % copies], out=y)
            label = f"qmv affine g64 N={N} K={Kd} M={M}" + (" (whole tiles)" if fmt == "affine-whole" else "")
        unit_bytes = nbytes
    elif args.kernel == "gdn":
        S, Hk, Hv, D, KC = 3, 16, 32, 128, 4
        Cd = 2 * Hk * D + Hv * D
        copies = 16  # 16 rings of 4 x 2 MiB states in rotation (> L2)

        # the decoder's form (MTPDecoder._make_gdn_args): state ring with a snapshot per token, conv rows
        # at a device row offset, the next window written back, the gated norm attached
        conv_w = (torch.randn(Cd, KC, generator=g, device=dev) * 0.5).to(torch.bfloat16)
        A_log = torch.log(torch.rand(Hv, generator=g, device=dev) * 15 + 1)
        dt_bias = torch.randn(Hv, generator=g, device=dev).to(torch.bfloat16)
        norm_w = (1 + 0.1 * torch.randn(D, generator=g, device=dev)).to(torch.bfloat16)
        Z = Hv * D
        ldp = Cd + Z + 2 * Hv
        proj = torch.randn(S, ldp, generator=g, device=dev).to(torch.bfloat16)
        slots = S + 1
        rings = [torch.randn(slots, Hv, D, D, generator=g, device=dev) * 0.1 for _ in range(copies)]
        wins = [torch.randn(2 * (S + KC - 1), Cd, generator=g, device=dev).to(torch.bfloat16) for _ in range(copies)]
        ctrl = torch.tensor([0, S + KC - 1, 0], dtype=torch.int32, device=dev)  # slot, conv row, window-out row
        y_ = torch.empty(S, Hv, D, dtype=torch.float32, device=dev)
        gout = torch.empty(S, Z, dtype=torch.bfloat16, device=dev)
        gargs = [_lib.GdnArgs(conv_src=wins[i].data_ptr(), ld_conv=Cd, conv_row_off=ctrl.data_ptr() + 4,
                              qkv=proj.data_ptr(), ld_qkv=ldp, win_out=wins[i].data_ptr(),
                              win_out_row_off=ctrl.data_ptr() + 8, conv_w=conv_w.data_ptr(),
                              a=proj.data_ptr() + 2 * (Cd + Z + Hv), b=proj.data_ptr() + 2 * (Cd + Z), ld_ab=ldp,
                              A_log=A_log.data_ptr(), dt_bias=dt_bias.data_ptr(), ring=rings[i].data_ptr(),
                              ring_cur=ctrl.data_ptr(), ring_slots=slots, y=y_.data_ptr(), S=S, Hk=Hk, Hv=Hv, Dk=D,
                              Dv=D, KC=KC, snap=1, gate_z=proj.data_ptr() + 2 * Cd, ld_gate_z=ldp,
                              gate_w=norm_w.data_ptr(), gate_out=gout.data_ptr(), ld_gate_out=Z, gate_eps=1e-6)
                 for i in range(copies)]
        import ctypes

        run = lambda i: _lib.check(_lib.lib().qmtp_gdn_fused_ex(ctypes.byref(gargs[i % copies]), _lib.stream()),
                                   "gdn_fused_ex")
        unit_bytes = Hv * D * D * 4 * (1 + S) + (S + KC - 1) * Cd * 2 * 2 + S * Z * 2 * 2 + S * Hv * D * 4
        label = "GatedDeltaNet verify step T=3 (ring snapshots, window write-back, gated norm)"
    elif args.kernel == "moe":
        from qmtp import moe

        mode = args.shape if args.shape in ("mxfp4", "nvfp4") else "mxfp4"
        E, H, I, T, TOPK, NSH = 66, 2048, 1408, 256, 6, 2
        copies = 2  # 2 x ~303 MB of expert weights in rotation (> 2x L2)
        layers = []
        for _ in range(copies):
            wts = []
            for shape in ((E, I, H), (E, I, H), (E, H, I)):
                w = (torch.randn(shape, generator=g, device=dev) * 0.02).to(torch.bfloat16)
                wts.extend(moe.quantize(w, mode))
                del w
            layers.append(wts)
        x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
        idx, sc = moe.route(torch.randn(T, E - NSH, generator=g, device=dev), TOPK, NSH)
        y = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
        run = lambda i: moe.moe_decode(x, *layers[i % copies], idx, sc, limit=None, mode=mode, out=y)
        G = 32 if mode == "mxfp4" else 16
        wbytes = E * 3 * H * I * (0.5 + 1 / G)
        unit_bytes = int(wbytes + T * H * 2 * 2 + idx.numel() * 8)
        flops = 2.0 * T * (TOPK + NSH) * 3 * H * I
        label = f"MoE config5 {mode}: T={T} E={E - NSH}+{NSH} top{TOPK} H={H} I={I}"
    else:  # head
        V, D, M = 248320, 4096, 3
        W = (torch.randn(V, D, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        head = TwoStageHead(W, 64)
        h = torch.randn(M, D, generator=g, device=dev).to(torch.bfloat16)
        outs = (torch.empty(M, 64, dtype=torch.int32, device=dev), torch.empty(M, 64, dtype=torch.bfloat16, device=dev),
                torch.empty(M, dtype=torch.int32, device=dev))
        run = lambda i: head.select(h, out=outs)
        unit_bytes = V * D // 2 + V * (D // 64) * 4 + M * 64 * D * 2 + M * D * 2
        label = "two-stage lm_head V=248320 D=4096 M=3 k=64"
    for i in range(max(Wu, 3)):
        run(i)
    torch.cuda.synchronize()
    s_ = torch.cuda.Stream()
    s_.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s_):
        for i in range(K):
            run(i)
    torch.cuda.current_stream().wait_stream(s_)
    graph.replay()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        ev0.record()
        graph.replay()
        ev1.record()
        torch.cuda.synchronize()
    us = ev0.elapsed_time(ev1) * 1e3 / K
    gbs = unit_bytes / (us * 1e-6) / 1e9
    extra = {}
    if args.kernel == "moe":
        extra = {"tflops": round(flops / (us * 1e-6) / 1e12, 1)}
    print(json.dumps({**extra, "kernel": args.kernel, "workload": label, "us_per_call": round(us, 3),
                      "bytes_per_call": unit_bytes, "achieved_GBps": round(gbs, 1), "peak": peak,
                      "peak_kind": peak_kind, "frac": round(gbs / peak, 4), "calls": K, "clocks": clk.summary(),
                      "device_error": _lib.device_error()}), flush=True)


def run_moe_ep(args):
    """Config 5 expert-parallel over WORLD_SIZE GPUs (launched by torch.distributed.run): every rank holds
    256 tokens, 64/G routed experts and both shared experts; one step = one MoE layer (route -> all-to-all
    dispatch -> local experts -> all-to-all back -> shared experts -> combine).  Device time per step is
    the max over ranks (CUDA events, all-reduce MAX)."""
    import datetime

    import torch
    import torch.distributed as dist

    world = int(os.environ["WORLD_SIZE"])
    rank = int(os.environ["RANK"])
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    out = moe_ep_measure(args, dev, rank, world)
    if rank == 0:
        print(json.dumps(out), flush=True)
    dist.destroy_process_group()


def moe_ep_measure(args, dev, rank, world):
    """Config 5 expert-parallel layer over the initialised process group; returns the line (rank 0)."""
    import torch
    import torch.distributed as dist

    from qmtp import _lib, moe
    from qmtp.moe_ep import ExpertParallelMoE, local_expert_table

    mode = args.shape if args.shape in ("mxfp4", "nvfp4") else "mxfp4"
    E_R, NSH, H, I, T, TOPK = 64, 2, 2048, 1408, 256, 6
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    full = []
    for shape in ((E_R + NSH, I, H), (E_R + NSH, I, H), (E_R + NSH, H, I)):
        w = (torch.randn(shape, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        full.extend(moe.quantize(w, mode))
        del w
    loc = local_expert_table(*full, E_R, NSH, rank, world)
    del full
    torch.cuda.empty_cache()
    gt = torch.Generator(device=dev)
    gt.manual_seed(1000 + rank)
    x = torch.randn((T, H), generator=gt, device=dev).to(torch.bfloat16)
    idx, sc = moe.route(torch.randn((T, E_R), generator=gt, device=dev), TOPK, NSH)
    # fixed capacity: a rank sends at most T * TOPK routed rows to any one peer; a slot of `factor` times
    # the average load T * TOPK / G keeps the all-to-alls near the real traffic, and any row it would
    # drop is reported through the device error word (printed below)
    cap = T * TOPK
    if args.ep_capacity_factor > 0:
        cap = min(cap, int(math.ceil(args.ep_capacity_factor * T * TOPK / world)))
    layer = ExpertParallelMoE(E_R, NSH,
                              lambda xr, e, out=None: moe.experts(xr, *loc, e, limit=None, mode=mode, out=out),
                              lambda tab, ro, s_: moe.combine(tab, ro, s_), capacity=cap)
    for _ in range(max(args.warmup, 3)):
        layer(x, idx, sc)
    torch.cuda.synchronize()
    # the sync-free layer (dispatch, three NCCL all-to-alls, expert pass, combine) as one CUDA graph
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        layer(x, idx, sc)
    torch.cuda.current_stream(dev).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        layer(x, idx, sc)
    for _ in range(max(args.warmup, 3)):
        graph.replay()
    torch.cuda.synchronize()
    dist.barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(args.steps):
        graph.replay()
    ev1.record()
    torch.cuda.synchronize()
    del graph  # a graph holding NCCL calls goes before the process group
    ms = torch.tensor([ev0.elapsed_time(ev1) / args.steps], device=dev)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    derr = torch.tensor([_lib.device_error()], dtype=torch.int64, device=dev)  # includes dispatch overflow
    dist.all_reduce(derr, op=dist.ReduceOp.MAX)
    dist.barrier()
    Gs = 32 if mode == "mxfp4" else 16
    wbytes = (E_R // world + NSH) * 3 * H * I * (0.5 + 1 / Gs)
    us = float(ms.item()) * 1e3
    return {"kernel": "moe_ep", "workload": f"MoE config5 {mode} expert-parallel: {world} GPUs x T={T}",
            "n_gpus": world, "us_per_layer": round(us, 2), "tokens_per_s": round(world * T / (us * 1e-6), 1),
            "local_weight_bytes": int(wbytes), "local_weight_GBps": round(wbytes / (us * 1e-6) / 1e9, 1),
            "steps": args.steps, "scaling": "weak",
            "dispatch": f"fixed capacity {cap} rows per peer (exact bound {T * TOPK}), no host sync, "
                        "one CUDA graph per layer",
            "timing": "CUDA events around graph replays, max over ranks",
            "device_error": int(derr.item())}


def head_shard_measure(args, dev, rank, world):
    """Config 3's two-stage head (V = 248320, D = 4096, M = 3, k = 64) sharded by vocabulary over the
    initialised process group (ShardedTwoStageHead: local coarse GEMV + top-k + rescoring on V/G rows,
    NCCL all-gather of the candidate lists, merge), against the whole head on one GPU.  Device time per
    call, max over ranks; `identical` = every rank's result equals the single-GPU head's bit for bit."""
    import torch
    import torch.distributed as dist

    from qmtp.lm_head2 import ShardedTwoStageHead, TwoStageHead
    from qmtp.qmv_kernel import QuantizedLinear, quantize

    V, D, M, k = 248320, 4096, 3, 64
    g = torch.Generator(device=dev)
    g.manual_seed(3)
    W = (torch.randn(V, D, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    h = torch.randn(M, D, generator=g, device=dev).to(torch.bfloat16)
    coarse = QuantizedLinear(*quantize(W))
    whole = TwoStageHead(W, k, coarse)
    sharded = ShardedTwoStageHead.from_full(W, k, coarse=coarse)

    def timed(fn, reps):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) * 1e3 / reps], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    reps = max(args.steps, 10)
    ref = [t.clone() for t in whole.select(h)]
    got = sharded.select(h)
    same = all(torch.equal(a.view(torch.int16) if a.dtype == torch.bfloat16 else a,
                           b.view(torch.int16) if b.dtype == torch.bfloat16 else b) for a, b in zip(ref, got))
    ok = torch.tensor([1 if same else 0], device=dev)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    us_whole = timed(lambda: whole.select(h), reps)
    us_shard = timed(lambda: sharded.select(h), reps)
    local_bytes = sharded.weight.shape[0] * (D // 2 + (D // 64) * 4)
    del whole, sharded, W, coarse
    torch.cuda.empty_cache()
    return {"kernel": "lmhead2_shard", "workload": f"two-stage head V={V} D={D} M={M} k={k} sharded by "
                                                   f"vocabulary over {world} GPUs",
            "n_gpus": world, "us_per_call": round(us_shard, 2), "us_per_call_1gpu": round(us_whole, 2),
            "speedup": round(us_whole / us_shard, 3), "local_coarse_bytes": int(local_bytes),
            "identical": bool(ok.item()), "reps": reps,
            "timing": "CUDA events around eager calls (local head, 2 NCCL all-gathers, merge), max over ranks"}


# ------------------------------------------------------------------------------ reference arm
def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import numpy as np

    from oracle import model as om

    threads = os.cpu_count() or 1
    cfg = om.ModelArgs(max_pos=2048)
    t0 = time.time()
    Wn = om.synthetic_weights_fast(cfg, seed=0)
    build_s = time.time() - t0
    orc = om.OracleModel(cfg, Wn)
    prompt = np.random.default_rng(1000).integers(0, cfg.vocab, args.prompt).astype(np.int32)
    t1 = time.time()
    cache, mcache, t, drafts = orc.prefill(prompt, K_DRAFTS)
    prefill_s = time.time() - t1
    Wu, K = args.warmup, args.steps
    _, st = orc.decode(cache, mcache, t, drafts, 10 ** 6, k=K_DRAFTS, max_cycles=Wu)
    t_next, d_next = st["next"]
    _, st2 = orc.decode(cache, mcache, t_next, d_next, 10 ** 6, k=K_DRAFTS, max_cycles=K)
    v = st2["tps"]
    res = {"metric": METRIC, "value": round(v, 4), "unit": "tok/s", "n_gpus": int(os.environ.get("WORLD_SIZE", "1")),
           "steps": K, "warmup": Wu, "ms_per_step": round(st2["seconds"] * 1e3 / max(st2["cycles"], 1), 2),
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
           "impl": "reference",
           "config": {"workload": "config4 (same model shapes, 4-bit affine g64, k=2, batch 1) on the host CPU",
                      "prompt_tokens": int(args.prompt), "weights": "synthetic_weights_fast (timing-equivalent)",
                      "weights_build_s": round(build_s, 1), "prefill_s": round(prefill_s, 1)},
           "cpu_baseline": {"value": round(v, 4), "unit": "tok/s", "cores": threads, "kind": "port",
                            "sample": f"{args.prompt}-token prompt, {Wu} warm-up + {K} timed decode cycles "
                                      f"({st2['tokens']} tokens) of the oracle restatement (MLX reference not runnable)"},
           "e2e": {"value": round(v, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(res), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=None)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-cycles", type=int, default=3, help="oracle cycles for cpu_baseline (0 = skip)")
    ap.add_argument("--prompt", type=int, default=PROMPT_LEN, help="prompt tokens (ours)")
    ap.add_argument("--weights", default="affine", choices=["affine", "nvfp4"],
                    help="decode: 4-bit format of the linears (affine g64 = config 4; nvfp4 = the Ollama blobs' format)")
    ap.add_argument("--temperature", type=float, default=0.0,
                    help="> 0: exact speculative sampling instead of greedy (engine.py:91-152)")
    ap.add_argument("--top-k", type=int, default=0)
    ap.add_argument("--top-p", type=float, default=1.0)
    ap.add_argument("--min-p", type=float, default=0.0)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--draft-vocab", type=int, default=0,
                    help="draft head over the first N ids (load_draft_head; 0 = the full vocabulary of config 4)")
    ap.add_argument("--kernel", default=None, choices=["qmv", "gdn", "head", "moe"],
                    help="time one kernel at a config shape instead of the decode loop")
    ap.add_argument("--shape", default="12288,4096,3", help="qmv: N,K,M[,affine|affine-whole|nvfp4]")
    ap.add_argument("--ep-capacity-factor", type=float, default=2.0,
                    help="expert-parallel MoE: rows per peer slot = factor x the average load T*TOPK/G, at most "
                         "the exact bound T*TOPK (0 = exact bound); an overflow shows as device_error != 0")
    args = ap.parse_args()
    if args.kernel:
        args.steps = 50 if args.steps is None else args.steps
        args.warmup = 3 if args.warmup is None else args.warmup
        if args.kernel == "moe" and int(os.environ.get("WORLD_SIZE", "1")) > 1:
            run_moe_ep(args)
        else:
            run_kernel(args)
        return
    if args.impl == "reference":
        args.steps = 3 if args.steps is None else args.steps
        args.warmup = 1 if args.warmup is None else args.warmup
        run_reference(args)
    else:
        args.steps = 253 if args.steps is None else args.steps
        args.warmup = 3 if args.warmup is None else max(args.warmup, 0)
        run_ours(args)


if __name__ == "__main__":
    main()
