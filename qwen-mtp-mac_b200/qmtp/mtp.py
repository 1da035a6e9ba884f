"""MTP speculative decoding on B200 -- the mtp.py / engine.py surface of qwen-mtp-mac.

Reference: mtp.py:143-153 ``backbone``, mtp.py:199-209 ``mtp_step``, mtp.py:212-226 ``draft_chain``
(chain="pre"), mtp.py:136-140 ``restore``, mtp.py:241-303 ``generate_mtp`` (fixed k, bb_hidden="pre"),
engine.py:121-128 (greedy verify), engine.py:91-152 (exact speculative sampling, ``Sampling``) and
engine.py:52-88 (prompt-prefix state cache, ``prefill(prompt, prefix_len)``).

B200 design.  Everything a cycle needs lives on the device: the GatedDeltaNet states in a ring of
k+2 slots per layer (the state after each verify token is a slot, so ``restore`` is a slot index),
the conv windows in two buffers per layer (the next conv state is a row offset), the KV caches with
device-side lengths, and a control block (include/qmtp.h QMTP_CTRL_*) updated by the accept kernel.
One verify + draft cycle is therefore a fixed sequence of launches, captured once as a CUDA graph
and replayed; the host reads the control block (emitted tokens) once per cycle, as the reference
evaluates once per cycle (mtp.py:276).  The prompt runs through the same verify-shaped step in
chunks of k+1 tokens; every op is batch-invariant, so this equals one pass over the prompt.
"""
from __future__ import annotations

import ctypes
import time
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from .lm_head2 import TwoStageHead, k_for
from .model import ModelArgs, Weights, rope_tables

C = _lib.CTRL


@dataclass
class Sampling:
    """engine.py:29-35: temperature 0 is greedy; top_k 0, top_p 1 and min_p 0 are off.  seed keys the
    counter-based generator (None: 0), so a seeded request replays exactly."""
    temperature: float = 0.0
    top_k: int = 0
    top_p: float = 1.0
    min_p: float = 0.0
    seed: int | None = None


class MTPDecoder:
    """Device state + launch sequence of one MTP decoding session (batch 1; greedy or sampled)."""

    def __init__(self, args: ModelArgs, W: Weights, k: int = 2, max_tokens: int = 1024, device="cuda",
                 sampling: Sampling | None = None, tau: float | None = None, draft_head=None):
        self.a, self.W, self.k = args, W, k
        self.tau = None
        # sampling with temperature > 0: exact speculative sampling (engine.py:91-152) over the
        # k_for(sampling) candidates of the two-stage head (lm_head2.py:32-36); otherwise greedy
        self.sp, self.K, self._sargs = None, 64, None
        self.set_sampling(sampling, _init=True)
        self.S = k + 1
        self.dev = torch.device(device)
        a, S, dev = args, self.S, self.dev
        self.L = _lib.lib()
        bf, f32, i32 = torch.bfloat16, torch.float32, torch.int32
        z = lambda *shape, dtype=bf: torch.zeros(shape, dtype=dtype, device=dev)
        self.ctrl = z(_lib.CTRL_SIZE, dtype=i32)
        self.ctrl_host = torch.zeros(_lib.CTRL_SIZE, dtype=i32).pin_memory()
        self.tokens_in = z(S, dtype=i32)
        self.a_tok = z(S, dtype=i32)
        self.drafts = z(max(k, 1), dtype=i32)
        self.m_tok = z(S, dtype=i32)
        self.out_cap = max_tokens + S + 8
        self.out_tokens = z(self.out_cap, dtype=i32)
        self.cos, self.sin = rope_tables(a, dev)
        # activations
        H = a.hidden
        self.h, self.xn, self.hn = z(S, H), z(S, H), z(S, H)
        self.lasth = z(1, H)   # last hidden row of a kept prompt prefix (its MTP pair is still owed)
        self.prefix = None     # kept prompt-prefix state (prefill(prefix_len=...))
        self.cached_tokens = 0
        self.proj = z(S, max(a.gdn_proj, a.attn_proj))
        self.ygdn = z(S, a.lin_hv, a.lin_dv, dtype=f32)
        self.gdn_out = z(S, a.lin_hv * a.lin_dv)
        self.att_out = z(S, a.n_heads * a.head_dim)
        self.gu, self.act = z(S, 2 * a.intermediate), z(S, a.intermediate)
        self.memb, self.mcat, self.mx, self.mxn = z(S, H), z(S, 2 * H), z(S, H), z(1, H)
        self._hstage, self._sel, self._last_S = z(S, H), z(1, dtype=i32), None  # reference-style calls
        self.dlogits = z(1, a.vocab)
        # draft head (mtp.py:156-196): the 4-bit full-vocabulary head, or a vocabulary subset
        # (set_draft_head); dloc holds each draft's row in the draft head's logits
        self.dproj, self.dids, self.dloc = W["lm_head_q"], None, z(max(k, 1), dtype=i32)
        self.probs = z(k, dtype=f32)  # adaptive k: the draft head's argmax probability per draft
        self.KMAX = 2048  # k_for's largest candidate count (lm_head2.py:32-36)
        self.fine, self.idx = z(S, self.KMAX), z(S, self.KMAX, dtype=i32)
        self.coarse = z(S, a.vocab)
        self.topk_ws = torch.empty(self.L.qmtp_topk_workspace(S, a.vocab, self.KMAX), dtype=torch.uint8,
                                   device=dev)
        self.argmax_ws = torch.empty(self.L.qmtp_argmax_workspace(1, a.vocab), dtype=torch.uint8, device=dev)
        # recurrent / cache state
        self.lin_ids = [i for i in range(a.layers) if a.is_linear(i)]
        self.att_ids = [i for i in range(a.layers) if not a.is_linear(i)]
        self.slots = k + 2
        self.win_rows = a.conv_k - 1 + S
        self.ring = {i: z(self.slots, a.lin_hv, a.lin_dv, a.lin_dk, dtype=f32) for i in self.lin_ids}
        self.win = {i: z(2 * self.win_rows, a.conv_dim) for i in self.lin_ids}
        self.kv = {i: (z(a.n_kv, a.max_pos, a.head_dim), z(a.n_kv, a.max_pos, a.head_dim)) for i in self.att_ids}
        self.mkv = (z(a.n_kv, a.max_pos, a.head_dim), z(a.n_kv, a.max_pos, a.head_dim))
        self.head = TwoStageHead(W["lm_head"], 64, W["lm_head_q"])
        self._gdn_args = {}
        for i in self.lin_ids:
            self._gdn_args[i] = self._make_gdn_args(i)
        self.graph = None
        self.launches = 0      # kernels launched by the library calls of this decoder
        self.prof = None       # list of (bytes, start event, end event, shape) while profiling qmv
        self.qmv_log = None    # list of the _qmv argument tuples of a cycle while recording
        if tau is not None:
            self.set_tau(tau)
        if draft_head is not None:
            self.set_draft_head(draft_head)

    def set_tau(self, tau: float | None):
        """Adaptive draft count (mtp.py:229-238, generate_mtp's tau): None verifies every draft; a number
        accepts only the first n_drafts(probs, tau) drafts of each cycle, probs being the draft head's
        argmax probabilities.  Greedy decoding only.  A change drops the captured cycle graph."""
        tau = None if tau is None else float(tau)
        if tau is not None and self.sp is not None:
            raise NotImplementedError("the adaptive draft count is built for greedy decoding")
        if tau != self.tau:
            self.graph = None
            if tau is None:
                self.ctrl[C["NUSE"]] = 0
        self.tau = tau

    def set_draft_head(self, head):
        """The head that proposes drafts (mtp.py:156-167 DraftHead): None for the model's full-vocabulary
        4-bit head, or a DraftHead over a vocabulary subset (load_draft_head).  It changes the drafts,
        never the output stream (the full two-stage head verifies).  A change drops the captured graph."""
        proj = self.W["lm_head_q"] if head is None else head.proj
        ids = None if head is None else head.ids
        if proj.in_features != self.a.hidden:
            raise ValueError("the draft head takes the hidden size")
        if ids is not None:
            ids = torch.as_tensor(ids, dtype=torch.int32, device=self.dev).contiguous()
            if ids.numel() != proj.out_features:
                raise ValueError("a draft head needs one vocabulary id per row")
        if proj is self.dproj and (ids is None) == (self.dids is None) and (ids is None or torch.equal(ids, self.dids)):
            return
        self.dproj, self.dids = proj, ids
        self.dlogits = torch.zeros(1, proj.out_features, dtype=torch.bfloat16, device=self.dev)
        self.graph = None

    def set_sampling(self, sampling: Sampling | None, _init: bool = False):
        """Greedy (None or temperature 0) or exact speculative sampling with these parameters; the
        candidate count is k_for(sampling).  A change drops the captured cycle graph (recaptured by the
        next decode), since the sampler's parameters are part of its launches."""
        sp = sampling if sampling is not None and sampling.temperature > 0 else None
        if sp is not None and getattr(self, "tau", None) is not None:
            raise NotImplementedError("the adaptive draft count is built for greedy decoding")
        K = k_for(sp)
        key = None if sp is None else (float(sp.temperature), int(sp.top_k), float(sp.top_p), float(sp.min_p))
        old = None if self.sp is None else (float(self.sp.temperature), int(self.sp.top_k), float(self.sp.top_p),
                                            float(self.sp.min_p))
        self.sp, self.K = sp, K
        self._sargs = None if sp is None else _lib.SamplingArgs(*key)
        if not _init and key != old:
            self.graph = None

    # ------------------------------------------------------------------ helpers
    def _cp(self, slot: int) -> int:
        return self.ctrl.data_ptr() + 4 * slot

    def _st(self):
        return _lib.stream()

    _KERNELS = {"rmsnorm": 1, "attn_prep": 1, "attention": 1, "swiglu": 1, "embed": 1, "embed_norm": 1, "gdn": 1,
                "norm_gate": 1,
                "accept": 1, "advance": 1, "next_tokens": 1, "argmax": 2, "draft_prob": 1, "nuse": 1}

    def _chk(self, rc, what):
        self.launches += self._KERNELS.get(what, 0)
        if rc != 0:
            _lib.check(rc, what)

    def _embed(self, tok, rows, out):
        """Embedding rows of device token ids (affine g64 or NVFP4 table) into out [rows, hidden]."""
        a, E = self.a, self.W["embed"]
        if E.mode == "nvfp4":
            rc = self.L.qmtp_embed_nvfp4(tok, rows, E.weight.data_ptr(), E.scales.data_ptr(), a.vocab, a.hidden,
                                         out.data_ptr(), a.hidden, self._st())
        else:
            rc = self.L.qmtp_embed(tok, rows, E.weight.data_ptr(), E.scales.data_ptr(), E.biases.data_ptr(), a.vocab,
                                   a.hidden, out.data_ptr(), a.hidden, self._st())
        self._chk(rc, "embed")

    def _qmv(self, x, lin, y, M, res=None, ldy=None, norm=None, swiglu=False, gated=None):
        """4-bit GEMV y = x . W^T (+ res): affine layers on the tensor-core kernel with split tiles
        (qmtp_qmv_affine_g64_split, one launch per 4 rows; shared tiles finished inside a cluster), NVFP4 layers (an NVFP4 checkpoint) on
        qmtp_qmv_nvfp4_g16_res.  norm (an RMSNorm weight): x is RMS-normalised first -- inside the
        affine kernel (qmtp_qmv_affine_g64_norm), or by qmtp_rmsnorm into self.xn for NVFP4.
        swiglu: x is [gate | up] and the projection's input is silu(gate) * up (qmtp_qmv_affine_g64_swiglu;
        NVFP4: qmtp_swiglu into self.act first).  gated = (z pointer, z row stride, norm weight): x is the
        GatedDeltaNet core output (fp32) and the input is its gated norm (qmtp_qmv_affine_g64_gated;
        NVFP4: qmtp_gdn_norm_gate into self.gdn_out first)."""
        N, K = lin.out_features, lin.in_features
        ldy = ldy or N
        nv = lin.mode == "nvfp4"
        if norm is not None and nv:
            self._norm(x, norm, self.xn, M)
            x, norm = self.xn, None
        if swiglu and nv:
            self._chk(self.L.qmtp_swiglu(x.data_ptr(), 2 * K, M, K, self.act.data_ptr(), self._st()), "swiglu")
            x, swiglu = self.act, False
        if gated is not None and nv:
            a = self.a
            self._chk(self.L.qmtp_gdn_norm_gate(x.data_ptr(), gated[0], gated[1], gated[2].data_ptr(),
                                                self.gdn_out.data_ptr(), K, M, a.lin_hv, a.lin_dv, a.eps,
                                                self._st()), "norm_gate")
            x, gated = self.gdn_out, None
        if self.qmv_log is not None:
            self.qmv_log.append((x, lin, y, M, res, ldy, norm, swiglu, gated))
        self.launches += (M + 3) // 4
        if self.prof is not None:
            e0 = torch.cuda.Event(enable_timing=True)
            e0.record()
        if nv:
            self._chk(self.L.qmtp_qmv_nvfp4_g16_res(x.data_ptr(), lin.weight.data_ptr(), lin.scales.data_ptr(),
                                                    y.data_ptr(), res.data_ptr() if res is not None else None,
                                                    M, N, K, ldy, self._st()), "qmv")
        elif swiglu:
            self._chk(self.L.qmtp_qmv_affine_g64_swiglu(x.data_ptr(), 2 * K, lin.weight.data_ptr(), lin.scales.data_ptr(),
                                                        lin.biases.data_ptr(), y.data_ptr(),
                                                        res.data_ptr() if res is not None else None, M, N, K, ldy,
                                                        self._st()), "qmv")
        elif gated is not None:
            self._chk(self.L.qmtp_qmv_affine_g64_gated(x.data_ptr(), K, gated[0], gated[1], gated[2].data_ptr(),
                                                       self.a.eps, lin.weight.data_ptr(), lin.scales.data_ptr(),
                                                       lin.biases.data_ptr(), y.data_ptr(),
                                                       res.data_ptr() if res is not None else None, M, N, K, ldy,
                                                       self._st()), "qmv")
        elif norm is not None:
            self._chk(self.L.qmtp_qmv_affine_g64_norm(x.data_ptr(), K, norm.data_ptr(), self.a.eps, lin.weight.data_ptr(),
                                                      lin.scales.data_ptr(), lin.biases.data_ptr(), y.data_ptr(),
                                                      res.data_ptr() if res is not None else None, M, N, K, ldy,
                                                      None, 0, self._st()), "qmv")
        else:
            self._chk(self.L.qmtp_qmv_affine_g64_split(x.data_ptr(), K, lin.weight.data_ptr(), lin.scales.data_ptr(),
                                                       lin.biases.data_ptr(), y.data_ptr(),
                                                       res.data_ptr() if res is not None else None, M, N, K, ldy,
                                                       None, 0, self._st()), "qmv")
        if self.prof is not None:
            e1 = torch.cuda.Event(enable_timing=True)
            e1.record()
            scale_bytes = N * (K // 16) if nv else N * (K // 64) * 4
            nbytes = N * K // 2 + scale_bytes + M * K * 2 + M * N * 2 * (2 if res is not None else 1)
            self.prof.append((nbytes, e0, e1, (M, N, K)))

    def _embed_norm(self, tok, rows, raw, w0, out0, ld_o0, hid=None, hid_sel=None, w1=None, out1=None, ld_o1=None):
        """Embedding rows of tok, optionally kept raw, RMS-normalised with w0 into out0; with hid also the
        RMS norm of hid's rows (from device row hid_sel) with w1 into out1.  One launch for an affine
        table (qmtp_embed_rmsnorm), else the embedding and the norms as separate launches."""
        a, E, H = self.a, self.W["embed"], self.a.hidden
        if E.mode == "nvfp4":
            emb = raw if raw is not None else self.memb
            self._embed(tok, rows, emb)
            self._norm(emb, w0, out0, rows, ld_o=ld_o0)
            if hid is not None:
                self._chk(self.L.qmtp_rmsnorm(hid.data_ptr(), H, hid_sel, w1.data_ptr(), a.eps, out1.data_ptr(),
                                              ld_o1, rows, H, self._st()), "rmsnorm")
            return
        self._chk(self.L.qmtp_embed_rmsnorm(tok, rows, E.weight.data_ptr(), E.scales.data_ptr(), E.biases.data_ptr(),
                                            a.vocab, H, None if raw is None else raw.data_ptr(), H, w0.data_ptr(),
                                            out0.data_ptr(), ld_o0, None if hid is None else hid.data_ptr(), H, hid_sel,
                                            None if w1 is None else w1.data_ptr(),
                                            None if out1 is None else out1.data_ptr(), ld_o1 or H, a.eps, self._st()),
                  "embed_norm")

    def _norm(self, x, w, out, M, ld_x=None, ld_o=None, row_sel=None):
        H = w.shape[0]
        self._chk(self.L.qmtp_rmsnorm(x.data_ptr(), ld_x or H, row_sel, w.data_ptr(), self.a.eps, out.data_ptr(),
                                      ld_o or H, M, H, self._st()), "rmsnorm")

    def _make_gdn_args(self, i):
        a, L = self.a, self.W[f"layers.{i}"]
        Cd, Z, ldp = a.conv_dim, a.lin_hv * a.lin_dv, self.proj.shape[1]
        p = self.proj.data_ptr()
        return _lib.GdnArgs(
            conv_src=self.win[i].data_ptr(), ld_conv=Cd, conv_row_off=self._cp(C["CONV_ROW"]),
            qkv=p, ld_qkv=ldp, win_out=self.win[i].data_ptr(), win_out_row_off=self._cp(C["WOUT_ROW"]),
            conv_w=L["conv1d"].data_ptr(), a=p + 2 * (Cd + Z + a.lin_hv), b=p + 2 * (Cd + Z), ld_ab=ldp,
            A_log=L["A_log"].data_ptr(), dt_bias=L["dt_bias"].data_ptr(), state_in=None, state_out=None,
            state_mid=None, ring=self.ring[i].data_ptr(), ring_cur=self._cp(C["SLOT"]), ring_slots=self.slots,
            y=self.ygdn.data_ptr(), S=self.S, Hk=a.lin_hk, Hv=a.lin_hv, Dk=a.lin_dk, Dv=a.lin_dv, KC=a.conv_k,
            snap=1,
            # the gated norm (gdn_fused.py:114-129) in the same call: z = the in_proj rows after qkv
            gate_z=p + 2 * Cd, ld_gate_z=ldp, gate_w=L["norm"].data_ptr(), gate_out=self.gdn_out.data_ptr(),
            ld_gate_out=Z, gate_eps=a.eps,
            # in_proj (a qmtp GEMV) is the launch before every step; state, windows and control words
            # were written cycles earlier, so they are read before the dependency wait
            preload=1)

    def _gdn_launches(self, i):
        """Kernels one qmtp_gdn_fused_ex call of layer i launches: 1 where the decode-shape kernel
        applies (it folds the gated norm), else the general core plus the gated norm."""
        a, g = self.a, self._gdn_args[i]
        decode = (self.S <= 4 and a.conv_k == 4 and a.lin_dk == 128 and a.lin_dv == 128 and g.conv_w % 16 == 0
                  and g.conv_src % 8 == 0 and g.qkv % 8 == 0 and g.ld_conv % 4 == 0 and g.ld_qkv % 4 == 0)
        return 1 if decode else 2

    # ------------------------------------------------------------------ layers
    def _attn_layer(self, L, x, rows, kc, vc, pos_slot):
        """Gated attention block: x (pre-norm residual stream, [rows, H]) += o_proj(attn(...)); the
        projection input is the normalised rows in self.xn."""
        a = self.a
        self._qmv(self.xn, L["qkv_proj"], self.proj, rows, ldy=self.proj.shape[1])
        # q/k norms, RoPE, the cache writes and the attention in one launch (qmtp_attn_prep's work done by
        # the attention kernel for the rows it reads)
        self._chk(self.L.qmtp_attention_fused(self.proj.data_ptr(), self.proj.shape[1], rows, a.n_heads, a.n_kv,
                                              a.head_dim, a.rotary_dim, L["q_norm"].data_ptr(), L["k_norm"].data_ptr(),
                                              a.eps, self.cos.data_ptr(), self.sin.data_ptr(), self._cp(pos_slot), 0,
                                              kc.data_ptr(), vc.data_ptr(), a.max_pos, self.att_out.data_ptr(),
                                              self._st()), "attention")
        self._qmv(self.att_out, L["o_proj"], x, rows, res=x)

    def _mlp(self, L, x, rows):
        a = self.a
        # post_ln inside gate_up's prologue; the SwiGLU as its own launch (in the graph it overlaps the down
        # projection's prologue; computing it in every CTA of the projection measured 7 us slower)
        self._qmv(x, L["gate_up"], self.gu, rows, norm=L["post_ln"])
        self._chk(self.L.qmtp_swiglu(self.gu.data_ptr(), 2 * a.intermediate, rows, a.intermediate,
                                     self.act.data_ptr(), self._st()), "swiglu")
        self._qmv(self.act, L["down"], x, rows, res=x)

    def backbone(self):
        """mtp.py:143-153 on the k+1 verify tokens in self.tokens_in: h (pre-norm) and hn (post-norm)."""
        a, W, S = self.a, self.W, self.S
        # the embedding rows (the residual stream h) and layer 0's input norm in one launch
        self._embed_norm(self.tokens_in.data_ptr(), S, self.h, W["layers.0"]["input_ln"], self.xn, a.hidden)
        for i in range(a.layers):
            L = W[f"layers.{i}"]
            # input_ln as its own launch: for the 12352- and 10240-row projections it overlaps the
            # projection's prologue better than the RMSNorm prologue (0.5-0.8 us per layer)
            if i:
                self._norm(self.h, L["input_ln"], self.xn, S)
            if a.is_linear(i):
                self._qmv(self.xn, L["in_proj"], self.proj, S, ldy=self.proj.shape[1])
                # conv, norms, gates, delta rule, snapshots and the gated norm into self.gdn_out
                self.launches += self._gdn_launches(i)
                self._chk(self.L.qmtp_gdn_fused_ex(ctypes.byref(self._gdn_args[i]), self._st()), "gdn_ex")
                self._qmv(self.gdn_out, L["out_proj"], self.h, S, res=self.h)
            else:
                kc, vc = self.kv[i]
                self._attn_layer(L, self.h, S, kc, vc, C["POS"])
            self._mlp(L, self.h, S)
        self._norm(self.h, W["norm"], self.hn, S)

    def _head(self):
        """Two-stage head (lm_head2.py:23-29) + greedy argmax: coarse qmv, then selection/rescoring."""
        a = self.a
        self._qmv(self.hn, self.W["lm_head_q"], self.coarse, self.S)
        # selection, then merge + rescoring + argmax (above 256 candidates: radix select, rescoring, argmax)
        self.launches += 2 if self.K <= 256 else 4
        self._chk(self.L.qmtp_topk_rescore(self.coarse.data_ptr(), a.vocab, self.S, a.vocab, self.K,
                                           self.W["lm_head"].data_ptr(), self.hn.data_ptr(), a.hidden,
                                           self.idx.data_ptr(), self.fine.data_ptr(), self.a_tok.data_ptr(),
                                           self.topk_ws.data_ptr(), self.topk_ws.numel(), self._st()), "head")

    def mtp_step(self, hidden, hidden_sel, tok, rows, out_sel, draft_out, with_draft=True):
        """mtp.py:199-209 for `rows` (hidden, token) pairs at MTP positions MPOS + r: the MTP layer
        output lands in self.mx; the draft token of row out_sel (device int, or row 0) goes to
        draft_out, a slot of self.drafts (DraftHead.token = the id of the draft head's argmax row,
        mtp.py:165-167)."""
        a, M = self.a, self.W["mtp"]
        H = a.hidden
        # the embedding and both pre-fc norms (mtp.py:202-203) into [e | h] = mcat, one launch
        mcat_h = self.mcat[:, H:]
        self._embed_norm(tok, rows, None, M["pre_fc_norm_embedding"], self.mcat, 2 * H, hidden, hidden_sel,
                         M["pre_fc_norm_hidden"], mcat_h, 2 * H)
        self._qmv(self.mcat, M["fc"], self.mx, rows)
        Ly = M["layer"]
        self._norm(self.mx, Ly["input_ln"], self.xn, rows)
        self._attn_layer(Ly, self.mx, rows, self.mkv[0], self.mkv[1], C["MPOS"])
        self._mlp(Ly, self.mx, rows)
        if not with_draft:
            return
        self._chk(self.L.qmtp_rmsnorm(self.mx.data_ptr(), H, out_sel, M["norm"].data_ptr(), a.eps,
                                      self.mxn.data_ptr(), H, 1, H, self._st()), "rmsnorm")
        Vd = self.dproj.out_features
        self._qmv(self.mxn, self.dproj, self.dlogits, 1)
        loc = self.dloc.data_ptr() + (draft_out - self.drafts.data_ptr())  # draft_out points into drafts
        self._chk(self.L.qmtp_argmax_bf16_ids(self.dlogits.data_ptr(), Vd, 1, Vd,
                                              None if self.dids is None else self.dids.data_ptr(), draft_out, loc,
                                              self.argmax_ws.data_ptr(), self.argmax_ws.numel(), self._st()),
                  "argmax")

    def _sample(self, first_row=-1):
        """Sampling mode: the emitted tokens (verify) or the first token (first_row) over a_tok."""
        self.launches += 1
        rc = self.L.qmtp_sample(self.idx.data_ptr(), self.fine.data_ptr(), self.K, self.K,
                                self.tokens_in.data_ptr() + 4, self.k, first_row, ctypes.byref(self._sargs),
                                self.a.vocab, self.ctrl.data_ptr(), self.a_tok.data_ptr(), self._st())
        if rc != 0:
            _lib.check(rc, "sample")

    def _accept(self, forced_keep=0):
        self._chk(self.L.qmtp_mtp_accept(self.a_tok.data_ptr(), self.tokens_in.data_ptr(), self.k, self.ctrl.data_ptr(),
                                         self.out_tokens.data_ptr(), self.out_cap, self.slots, self.win_rows,
                                         forced_keep, self._st()), "accept")

    def _draft_chain(self, hidden, tok):
        """mtp.py:212-226, k drafts, chain on the MTP's own pre-norm output (chain="pre")."""
        sel = self._cp(C["SEL"])
        self.mtp_step(hidden, None, tok, self.S, sel, self.drafts.data_ptr())
        self._draft_prob(0)
        self._chk(self.L.qmtp_mtp_advance(self.ctrl.data_ptr(), self._st()), "advance")
        for j in range(1, self.k):
            # the chained step reads the previous step's output row: row SEL after the first step, 0 after
            hsel = sel if j == 1 else None
            self.mtp_step(self.mx, hsel, self.drafts.data_ptr() + 4 * (j - 1), 1, None,
                          self.drafts.data_ptr() + 4 * j)
            self._draft_prob(j)
        if self.tau is not None:
            self._chk(self.L.qmtp_mtp_nuse(self.probs.data_ptr(), self.k, self.tau, self.ctrl.data_ptr(), self._st()),
                      "nuse")
        self._chk(self.L.qmtp_next_tokens(self.a_tok.data_ptr(), self.drafts.data_ptr(), self.k, self.ctrl.data_ptr(),
                                          self.tokens_in.data_ptr(), self._st()), "next_tokens")

    def _draft_prob(self, j):
        """Adaptive k: probability of draft j under the draft head (mtp.py:222-223)."""
        if self.tau is not None:
            self._chk(self.L.qmtp_draft_prob(self.dlogits.data_ptr(), self.dproj.out_features,
                                             self.dloc.data_ptr() + 4 * j, self.probs.data_ptr() + 4 * j, self._st()),
                      "draft_prob")

    def cycle(self):
        """One verify + accept + draft cycle (mtp.py:268-294), device-side only."""
        self.backbone()
        self._head()
        if self.sp is not None:
            self._sample()
        self._accept()
        self._draft_chain(self.h, self.a_tok.data_ptr())
        self.ctrl_host.copy_(self.ctrl, non_blocking=True)

    # ------------------------------------------------------------------ session
    def reset(self):
        self.ctrl.zero_()
        self.ctrl[C["WOUT_ROW"]] = self.win_rows
        if self.sp is not None:
            seed = int(self.sp.seed or 0) & 0xFFFFFFFFFFFFFFFF
            lo, hi = seed & 0xFFFFFFFF, seed >> 32
            self.ctrl[C["SEED_LO"]] = lo - (1 << 32) if lo >= 1 << 31 else lo
            self.ctrl[C["SEED_HI"]] = hi - (1 << 32) if hi >= 1 << 31 else hi
        for i in self.lin_ids:
            self.win[i].zero_()
            self.ring[i][0].zero_()

    def prefill(self, prompt_ids, prefix_len: int = 0) -> int:
        """Runs the prompt (mtp.py:258-263) in chunks of k+1 and leaves [t, d1..dk] in tokens_in.

        prefix_len (engine.py:52-88, 160-172): the first prefix_len tokens are a reusable prefix, e.g.
        the conversation so far without the generation prompt.  The state after them is kept on the
        device (GatedDeltaNet state and conv window, control block, the last hidden row; the KV caches
        only grow, so their entries before the prefix stay valid), and a later prompt that starts with
        the same tokens resumes from it instead of running them again.  A prompt that does not share
        the kept prefix drops it.  The prompt after the prefix is never empty."""
        p = [int(x) for x in prompt_ids]
        if not p:
            raise ValueError("empty prompt")
        prefix_len = max(0, min(int(prefix_len), len(p) - 1))
        snap = self.prefix
        if snap is not None and len(snap["ids"]) <= prefix_len and p[:len(snap["ids"])] == snap["ids"]:
            self._restore_prefix(snap)
            start, pending = len(snap["ids"]), True
        else:
            self.prefix = None
            self.reset()
            start, pending = 0, False
        self.cached_tokens = start
        if prefix_len > start:
            self._prefill_part(p[start:prefix_len], pending, final=False)
            self._take_prefix(p[:prefix_len])
            start, pending = prefix_len, True
        return self._prefill_part(p[start:], pending, final=True)

    def _prefill_part(self, toks, pending: bool, final: bool):
        """Prompt tokens appended to the current state.  pending: the MTP pair (last hidden row of the
        previous part, first token of this one) is still owed.  A non-final part leaves the pair of its
        last row pending (its next token is not known yet) and keeps that row in self.lasth."""
        S = self.S
        if pending:
            self.m_tok[0:1].fill_(toks[0])
            self.mtp_step(self.lasth, None, self.m_tok.data_ptr(), 1, None, self.drafts.data_ptr(), with_draft=False)
            self.ctrl[C["MPOS"]] += 1
        n_chunks = (len(toks) + S - 1) // S
        for c in range(n_chunks):
            chunk = toks[c * S:(c + 1) * S]
            n = len(chunk)
            self.tokens_in.copy_(torch.tensor(chunk + [0] * (S - n), dtype=torch.int32))
            self.backbone()
            last = c == n_chunks - 1
            if last and final:
                self._norm_head_rows()
                if self.sp is not None:  # the first token is drawn from the last prompt row (engine.py:110-115)
                    self._sample(first_row=n - 1)
            self._accept(forced_keep=n)
            nxt = toks[c * S + 1:c * S + 1 + n]
            self.m_tok.copy_(torch.tensor(nxt + [0] * (S - len(nxt)), dtype=torch.int32))
            if last and final:  # the pair of the last prompt position is (h, t): t is the verify argmax of that row
                self.m_tok[n - 1:n].copy_(self.a_tok[n - 1:n])
                self._draft_chain(self.h, self.m_tok.data_ptr())
            elif last:
                if n > 1:
                    self.mtp_step(self.h, None, self.m_tok.data_ptr(), n - 1, None, self.drafts.data_ptr(),
                                  with_draft=False)
                    self.ctrl[C["MPOS"]] += n - 1
                self.lasth.copy_(self.h[n - 1:n])
            else:
                self.mtp_step(self.h, None, self.m_tok.data_ptr(), S, None, self.drafts.data_ptr(), with_draft=False)
                self._chk(self.L.qmtp_mtp_advance(self.ctrl.data_ptr(), self._st()), "advance")
        return int(self.tokens_in[0].item()) if final else None

    def _take_prefix(self, ids):
        cur = int(self.ctrl[C["SLOT"]].item())
        self.prefix = {"ids": list(ids), "ctrl": self.ctrl.clone(), "lasth": self.lasth.clone(),
                       "state": {i: self.ring[i][cur].clone() for i in self.lin_ids},
                       "win": {i: self.win[i].clone() for i in self.lin_ids}}

    def _restore_prefix(self, snap):
        self.ctrl.copy_(snap["ctrl"])
        cur = int(snap["ctrl"][C["SLOT"]].item())
        for i in self.lin_ids:
            self.ring[i][cur].copy_(snap["state"][i])
            self.win[i].copy_(snap["win"][i])
        self.lasth.copy_(snap["lasth"])

    def _norm_head_rows(self):
        self._head()

    def capture(self):
        """Captures cycle() as a CUDA graph (after one eager warm-up cycle elsewhere)."""
        s = torch.cuda.Stream(self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            self.cycle()
        torch.cuda.current_stream(self.dev).wait_stream(s)
        self.graph = g
        return g

    def ensure_graph(self):
        """Captures the cycle graph if there is none.  Capture needs the library's one-time kernel setup
        done, so one eager cycle runs first on a copy of the state, which is then put back."""
        if self.graph is not None:
            return
        snap = _snapshot(self)
        self.run_cycle()
        _restore(self, snap)
        self.capture()
        _restore(self, snap)

    def run_cycle(self):
        """One cycle; returns the tokens it emitted (read from the pinned copy of the control block)."""
        if self.graph is not None:
            self.graph.replay()
        else:
            self.cycle()
        torch.cuda.current_stream(self.dev).synchronize()
        h = self.ctrl_host.tolist()
        keep = h[C["KEEP"]]
        return h[C["EMIT0"]:C["EMIT0"] + keep]


def _linears(W):
    """Every 4-bit linear layer of a weight set (nested dicts of tensors and QuantizedLinear)."""
    from .qmv_kernel import QuantizedLinear

    out, todo = [], [W]
    while todo:
        for v in todo.pop().values():
            if isinstance(v, QuantizedLinear):
                out.append(v)
            elif isinstance(v, dict):
                todo.append(v)
    return out


def decode_mtp(dec: MTPDecoder, prompt_ids, max_tokens, eos=(), use_graph=True, draft_override=None,
               prefix_len=0):
    """The loop of mtp.py:241-303 on a decoder (greedy or the decoder's sampling, k fixed): returns
    (tokens, stats).  tok/s excludes the prefill, as the reference does (mtp.py:264,295).
    draft_override(cycle) -> k tokens or None replaces the drafts a cycle verifies (test hook for the
    acceptance / rollback paths).  prefix_len: see MTPDecoder.prefill (stats["cached_tokens"] = prompt
    tokens resumed from the kept prefix)."""
    t = dec.prefill(prompt_ids, prefix_len)
    if use_graph:
        dec.ensure_graph()
    torch.cuda.synchronize()
    verified0 = int(dec.ctrl[C["VERIFIED"]])
    t0 = time.perf_counter()
    out = [t]
    k = dec.k
    cycles = 0
    while len(out) < max_tokens and out[-1] not in eos:
        if draft_override is not None:
            o = draft_override(cycles)
            if o is not None:
                dec.tokens_in[1:].copy_(torch.tensor([int(v) for v in o], dtype=torch.int32))
        out += dec.run_cycle()
        cycles += 1
    dt = time.perf_counter() - t0
    for i, tok in enumerate(out):
        if tok in eos:
            out = out[:i + 1]
            break
    out = out[:max_tokens]
    ctrl = dec.ctrl.tolist()
    acc = [ctrl[C["ACC0"] + i] for i in range(k)]
    stats = {"tps": (len(out) - 1) / dt if dt > 0 else 0.0, "tok_ciclo": (len(out) - 1) / max(cycles, 1),
             "acept": [n / max(cycles, 1) for n in acc],
             "borradores_ciclo": (ctrl[C["VERIFIED"]] - verified0) / max(cycles, 1) if dec.tau is not None else float(k),
             "cycles": cycles,
             "seconds": dt, "cached_tokens": dec.cached_tokens}
    return out, stats


# ---------------------------------------------------------------------------------------------------
# The reference's loop functions with its names and argument order (mtp.py:136-303), over the device
# state of an MTPDecoder.  `lm` is a qmtp.model.Model; a "cache" (trunk or MTP) is the decoder that
# lm.make_cache() returns.  They run eagerly, one call at a time, like the reference's; decode_mtp is
# the graph-captured loop that generate_mtp hands the work to.


class DraftHead:
    """mtp.py:156-167: the cheap head that proposes drafts.  proj is a 4-bit QuantizedLinear over some
    rows of the lm_head; ids (None, or int32 [rows]) the vocabulary id of each row -- with ids it scores
    only that subset of the vocabulary."""

    def __init__(self, proj, ids=None):
        if ids is not None:
            ids = torch.as_tensor(ids, dtype=torch.int32, device=proj.weight.device).contiguous()
            if ids.numel() != proj.out_features:
                raise ValueError("one vocabulary id per row of proj")
        self.proj, self.ids = proj, ids

    def __call__(self, x):
        return self.proj(x)

    def token(self, logits):
        i = torch.argmax(logits, dim=-1)
        return i if self.ids is None else self.ids[i]


def load_draft_head(vocab, quant=None, freq=False, extra_ids=(), *, lm, counts=None):
    """mtp.py:170-196 with the reference's arguments: a draft head over `vocab` rows of the lm_head, the
    first `vocab` ids or, with freq=True, the `vocab` most frequent ids of a corpus (`counts`: the
    per-id counts build_draft_vocab.py writes, an array or the path of its .npy file) plus extra_ids,
    ascending.  It never changes the output (the full head verifies), only the acceptance.  quant: the
    4-bit g64 affine format of the model's head (the reference's {"bits": 4, "group_size": 64}); its
    rows are quantized row by row, so the subset is a gather of the model's 4-bit head (lm_head_q).
    `lm` (keyword) is the model; the reference reads the head from its checkpoint instead."""
    from .qmv_kernel import QuantizedLinear

    if quant is not None and (quant.get("bits", 4), quant.get("group_size", 64)) != (4, 64):
        raise NotImplementedError("draft heads are 4-bit, group 64 (the model's coarse head format)")
    full = lm.weights["lm_head_q"]
    if full.mode != "affine":
        raise NotImplementedError("a vocabulary-subset draft head over an NVFP4 head is not built")
    V = full.out_features
    if freq:
        if counts is None:
            raise ValueError("freq=True needs the corpus counts (counts=...)")
        c = np.load(counts) if isinstance(counts, (str, bytes)) or hasattr(counts, "__fspath__") else np.asarray(counts)
        c = c[:V]
        top = set(np.argsort(-c)[:vocab].tolist()) | {int(e) for e in extra_ids}
        rows = torch.tensor(sorted(top), dtype=torch.int64, device=full.weight.device)
        proj = QuantizedLinear(full.weight.index_select(0, rows).contiguous(),
                               full.scales.index_select(0, rows).contiguous(),
                               full.biases.index_select(0, rows).contiguous())
        return DraftHead(proj, rows.to(torch.int32))
    n = min(int(vocab), V)
    if n == V:
        return DraftHead(full)
    return DraftHead(QuantizedLinear(full.weight[:n], full.scales[:n], full.biases[:n]))


def _check_head(lm, head):
    if head is not None and not isinstance(head, DraftHead):
        raise TypeError("head must be a DraftHead (load_draft_head) or None")


def _check_mtp(lm, mtp):
    if mtp is not None and mtp is not lm.mtp:
        raise NotImplementedError("mtp must be the model's own MTP weights (lm.mtp)")


def restore(cache: MTPDecoder, keep: int):
    """mtp.py:136-140: leaves the GatedDeltaNet layers (and here the trunk KV caches too) as if only the
    first `keep` tokens of the last backbone() step had been processed: the state is ring slot keep of
    that step and the conv window starts at row keep."""
    S = getattr(cache, "_last_S", None)
    if S is None:
        raise RuntimeError("restore() follows a backbone() step")
    if not 1 <= keep <= S:
        raise ValueError(f"keep must be in 1..{S}")
    c = cache.ctrl.tolist()
    c[C["SLOT"]] = (c[C["SLOT"]] - S + keep) % cache.slots
    c[C["CONV_ROW"]] = c[C["CONV_ROW"]] - S + keep
    c[C["POS"]] = c[C["POS"]] - S + keep
    c[C["KEEP"]], c[C["SEL"]] = keep, keep - 1
    cache.ctrl.copy_(torch.tensor(c, dtype=torch.int32))
    cache._last_S = keep


def backbone(lm, tokens, cache: MTPDecoder, last_only=False):
    """mtp.py:143-153: the trunk over tokens [1, S] (S <= k+1 of the cache): returns (logits, h, hn)
    with the two-stage head's logits (-inf outside the candidates, lm_head2.py:23-29) and the pre-/
    post-norm hidden rows.  The step is committed (all S tokens); restore(cache, keep) rolls it back."""
    t = torch.as_tensor(tokens, dtype=torch.int32).reshape(-1).to(cache.dev)
    n = t.numel()
    if not 1 <= n <= cache.S:
        raise ValueError(f"backbone takes 1..{cache.S} tokens per step with this cache")
    cache.tokens_in.zero_()
    cache.tokens_in[:n].copy_(t)
    cache.backbone()
    cache._accept(forced_keep=n)
    cache._last_S = n
    h, hn = cache.h[:n].clone()[None], cache.hn[:n].clone()[None]
    logits = lm.lm_head(hn[:, -1:] if last_only else hn)
    return logits, h, hn


def mtp_step(lm, mtp, hidden, tokens, mcache: MTPDecoder, head=None):
    """mtp.py:199-209: one MTP pass over the pairs (hidden[i], tokens[i]) (the pairs are committed to
    the MTP cache); returns (logits, x, xn) of the last pair, logits from the draft head."""
    _check_mtp(lm, mtp)
    _check_head(lm, head)
    dec = mcache
    hid = hidden.reshape(-1, dec.a.hidden)
    tok = torch.as_tensor(tokens, dtype=torch.int32).reshape(-1).to(dec.dev)
    n = tok.numel()
    if hid.shape[0] != n or not 1 <= n <= dec.S:
        raise ValueError(f"mtp_step takes 1..{dec.S} (hidden, token) pairs with this cache")
    dec.set_draft_head(head)
    return _mtp_pairs(dec, hid, tok, commit=True)


def _mtp_pairs(dec, hid, tok, commit):
    n = tok.numel()
    dec._hstage[:n].copy_(hid)
    dec.m_tok[:n].copy_(tok)
    dec._sel.fill_(n - 1)
    dec.mtp_step(dec._hstage, None, dec.m_tok.data_ptr(), n, dec._sel.data_ptr(), dec.drafts.data_ptr())
    if commit:
        dec.ctrl[C["MPOS"]] += n
    x = dec.mx[n - 1:n].clone()[None]
    xn = dec.mxn[:1].clone()[None]
    return dec.dlogits.clone()[None], x, xn


def draft_chain(lm, mtp, hidden, tokens, mcache: MTPDecoder, k, head=None, chain="pre", with_probs=False):
    """mtp.py:212-226: k drafts, the first from the real pairs (hidden, tokens) (committed to the MTP
    cache), the next ones chained on the MTP's own pre-norm output (not committed, as the reference
    trims them in the next cycle).  with_probs: also the draft head's probability of each draft."""
    _check_mtp(lm, mtp)
    _check_head(lm, head)
    if chain != "pre":
        raise NotImplementedError('only chain="pre" is built')
    dec = mcache
    hid = hidden.reshape(-1, dec.a.hidden)
    tok = torch.as_tensor(tokens, dtype=torch.int32).reshape(-1).to(dec.dev)
    if hid.shape[0] != tok.numel() or not 1 <= tok.numel() <= dec.S:
        raise ValueError(f"draft_chain takes 1..{dec.S} (hidden, token) pairs with this cache")
    dec.set_draft_head(head)
    drafts, probs = [], []
    logits, x, _ = _mtp_pairs(dec, hid, tok, commit=True)
    mpos = int(dec.ctrl[C["MPOS"]].item())
    for i in range(k):
        if i:
            logits, x, _ = _mtp_pairs(dec, x[0], drafts[-1].reshape(1), commit=False)
            dec.ctrl[C["MPOS"]] += 1  # the chained entry is visible to the next chained step
        local = torch.argmax(logits[0, -1]).to(torch.int32).reshape(1)  # first maximum: the lower row
        drafts.append(local if dec.dids is None else dec.dids[local.long()])
        if with_probs:
            pr = torch.empty(1, dtype=torch.float32, device=dec.dev)
            row = logits[0, -1].contiguous()
            _lib.check(dec.L.qmtp_draft_prob(row.data_ptr(), row.numel(), local.data_ptr(), pr.data_ptr(),
                                             _lib.stream()), "draft_prob")
            probs.append(pr)
    dec.ctrl[C["MPOS"]] = mpos
    d = torch.cat(drafts)[None]
    return (d, torch.cat(probs)[None]) if with_probs else d


def n_drafts(probs, tau):
    """mtp.py:229-238: adaptive k -- verify drafts while their cumulative probability stays above tau
    (at least one)."""
    n, acc = 0, 1.0
    for p in probs:
        acc *= p
        if n and acc < tau:
            break
        n += 1
    return n


def generate_mtp(lm, mtp, prompt_ids, max_tokens, eos, head=None, k=1, bb_hidden="pre", chain="pre", tau=None):
    """mtp.py:241-303 with the reference's signature: greedy MTP decoding of prompt_ids, returns
    (tokens, stats).  Runs decode_mtp (the graph-captured loop) on the model's session for this k.
    bb_hidden and chain must be "pre" (the variant the build implements); tau: None = always k drafts, a
    number = adaptive k (n_drafts over the draft head's probabilities, mtp.py:229-238)."""
    _check_mtp(lm, mtp)
    _check_head(lm, head)
    if bb_hidden != "pre" or chain != "pre":
        raise NotImplementedError('only bb_hidden="pre", chain="pre" are built')
    dec = lm.session(k=k, max_tokens=max_tokens)
    dec.set_sampling(None)
    dec.set_tau(tau)
    dec.set_draft_head(head)
    return decode_mtp(dec, prompt_ids, max_tokens, tuple(eos))


def _snapshot(dec: MTPDecoder):
    """Copies every piece of mutable device state (used around the warm-up cycle before capture)."""
    bufs = [dec.ctrl, dec.tokens_in, dec.a_tok, dec.drafts, dec.out_tokens, dec.mkv[0], dec.mkv[1]]
    bufs += [dec.ring[i] for i in dec.lin_ids] + [dec.win[i] for i in dec.lin_ids]
    bufs += [t for i in dec.att_ids for t in dec.kv[i]]
    return [(b, b.clone()) for b in bufs]


def _restore(dec: MTPDecoder, snap):
    for b, c in snap:
        b.copy_(c)


def export_state(dec: MTPDecoder):
    """The decoding state as host arrays in the layout of a reference-style cache: per layer either
    (conv_state bf16 [KC-1, C], state fp32 [Hv, Dv, Dk]) or (k, v bf16 [nkv, max_pos, Dh], length),
    the MTP cache (k, v, length), and the pending verify input [t, d1..dk]."""
    def bits(t):
        t = t.detach().contiguous().cpu()
        return t.view(torch.int16).numpy().view(np.uint16) if t.dtype == torch.bfloat16 else t.numpy()

    ctrl = dec.ctrl.tolist()
    a = dec.a
    layers = []
    for i in range(a.layers):
        if a.is_linear(i):
            r = ctrl[C["CONV_ROW"]]
            layers.append(("gdn", bits(dec.win[i][r:r + a.conv_k - 1]), bits(dec.ring[i][ctrl[C["SLOT"]]])))
        else:
            layers.append(("attn", bits(dec.kv[i][0]), bits(dec.kv[i][1]), ctrl[C["POS"]]))
    mtp = (bits(dec.mkv[0]), bits(dec.mkv[1]), ctrl[C["MPOS"]])
    pending = dec.tokens_in.tolist()
    return layers, mtp, pending
