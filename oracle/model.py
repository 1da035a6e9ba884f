"""CPU restatement of the synthetic Qwen3.5 decoder and the greedy MTP loop -- TEST INFRASTRUCTURE.

Follows aulafy/qwen-mtp-mac mtp.py:35-70 (MTP / MTPLayer), mtp.py:73-130 (_gdn_call with
snapshots), mtp.py:136-140 (restore), mtp.py:143-153 (backbone), mtp.py:199-226 (mtp_step,
draft_chain, chain="pre"), mtp.py:241-303 (generate_mtp, bb_hidden="pre", fixed k) and the greedy
branch of engine.py:121-128.  The layer structure (3:1 GatedDeltaNet : gated attention, partial RoPE,
q/k RMS norms, sigmoid output gate, SwiGLU MLP) is the Qwen3.5 text model; every op is one of the C
oracle functions, so the arithmetic is the fixed sequence the CUDA kernels reproduce.  Weights are
given as numpy bit arrays (bf16 -> uint16, packed 4-bit -> uint32).

Unlike the B200 engine (which runs the prompt in 3-token chunks through the same graph as a
verify step), this restatement runs the whole prompt through one backbone call, as the reference
does; batch invariance of every op makes the two identical.
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field

import numpy as np

from . import ops


@dataclass
class ModelArgs:
    hidden: int = 4096
    layers: int = 32
    intermediate: int = 12288
    n_heads: int = 16
    n_kv: int = 4
    head_dim: int = 256
    rotary_dim: int = 64  # partial_rotary_factor 0.25
    rope_theta: float = 10_000_000.0
    vocab: int = 248320
    lin_hk: int = 16
    lin_hv: int = 32
    lin_dk: int = 128
    lin_dv: int = 128
    conv_k: int = 4
    eps: float = 1e-6
    full_attention_interval: int = 4
    max_pos: int = 1024

    def is_linear(self, i: int) -> bool:
        return (i + 1) % self.full_attention_interval != 0

    @property
    def conv_dim(self) -> int:
        return 2 * self.lin_hk * self.lin_dk + self.lin_hv * self.lin_dv

    @property
    def gdn_proj(self) -> int:  # qkv | z | b | a
        return self.conv_dim + self.lin_hv * self.lin_dv + 2 * self.lin_hv

    @property
    def attn_proj(self) -> int:  # per q head (query, gate) | k | v
        return self.n_heads * 2 * self.head_dim + 2 * self.n_kv * self.head_dim


CONFIG4 = ModelArgs()
SMALL = ModelArgs(hidden=1024, layers=4, intermediate=2048, n_heads=4, n_kv=2, head_dim=256, vocab=16384,
                  lin_hk=4, lin_hv=8, max_pos=1024)


def rope_tables(args: ModelArgs, max_pos: int | None = None):
    """cos/sin [max_pos, rotary_dim/2] as float32, computed in float64 (HF default rope:
    inv_freq_i = theta^(-2i/R))."""
    max_pos = max_pos or args.max_pos
    half = args.rotary_dim // 2
    inv = 1.0 / (args.rope_theta ** (np.arange(0, args.rotary_dim, 2, dtype=np.float64) / args.rotary_dim))
    ang = np.arange(max_pos, dtype=np.float64)[:, None] * inv[None, :half]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


# ------------------------------------------------------------------ C op wrappers
_P, _I = ops._P, ops._I


def _c(a, dt):
    return np.ascontiguousarray(a, dt)


def rmsnorm(x, w, eps):
    x = _c(x, np.uint16)
    x2 = x.reshape(-1, x.shape[-1])
    out = np.empty_like(x2)
    ops.lib().qo_rmsnorm(_P(x2.ctypes.data), _I(x2.shape[1]), _P(_c(w, np.uint16).ctypes.data),
                         ops.ctypes.c_float(eps), _P(out.ctypes.data), _I(x2.shape[1]), _I(x2.shape[0]),
                         _I(x2.shape[1]))
    return out.reshape(x.shape)


def embed(tokens, *lin_and_d):
    """embed(tokens, wq, s, b, D) for an affine-g64 table, embed(tokens, wq, s, D) for NVFP4."""
    D = lin_and_d[-1]
    tok = _c(tokens, np.int32).ravel()
    out = np.empty((tok.size, D), np.uint16)
    if len(lin_and_d) == 3:
        wq, s = lin_and_d[:2]
        ops.lib().qo_embed_nvfp4(_P(tok.ctypes.data), _I(tok.size), _P(_c(wq, np.uint32).ctypes.data),
                                 _P(_c(s, np.uint8).ctypes.data), _I(D), _P(out.ctypes.data))
        return out
    wq, s, b = lin_and_d[:3]
    ops.lib().qo_embed(_P(tok.ctypes.data), _I(tok.size), _P(_c(wq, np.uint32).ctypes.data),
                       _P(_c(s, np.uint16).ctypes.data), _P(_c(b, np.uint16).ctypes.data), _I(D),
                       _P(out.ctypes.data))
    return out


def add(a, b):
    a, b = _c(a, np.uint16), _c(b, np.uint16)
    out = np.empty_like(a)
    ops.lib().qo_add_bf16(_P(a.ctypes.data), _P(b.ctypes.data), _P(out.ctypes.data), ops.ctypes.c_long(a.size))
    return out


def qmv(x, lin):
    """lin = (wq, scales, biases) affine g64, or (wq, scales) NVFP4 g16."""
    if len(lin) == 2:
        return ops.qmv_nvfp4(x, lin[0], lin[1])
    return ops.qmv_affine(x, lin[0], lin[1], lin[2])


# ------------------------------------------------------------------ caches
@dataclass
class GDNCache:
    conv: np.ndarray  # bf16 [KC-1, C]
    state: np.ndarray  # fp32 [Hv, Dv, Dk]
    rollback: tuple | None = None  # (window, mids) after a snapshot pass


@dataclass
class KVCache:
    k: np.ndarray  # bf16 [nkv, max_pos, Dh]
    v: np.ndarray
    offset: int = 0

    def trim(self, n: int) -> None:
        self.offset -= n


# ------------------------------------------------------------------ model
class OracleModel:
    def __init__(self, args: ModelArgs, W: dict):
        self.a = args
        self.W = W
        self.cos, self.sin = rope_tables(args)
        self.draft_ids = None          # draft head over a vocabulary subset (set_draft_head)
        self.draft_W = None            # its rows; None: the full 4-bit head W["lm_head_q"]

    def set_draft_head(self, vocab=None, counts=None, extra_ids=()):
        """mtp.py:170-196 load_draft_head: the draft head scores `vocab` rows of the lm_head -- the first
        `vocab` ids, or with `counts` the `vocab` most frequent ids plus extra_ids, ascending -- with the
        head's 4-bit g64 quantization (per row and group, so the subset's rows equal the full copy's).
        vocab None: the full-vocabulary head."""
        V = self.a.vocab
        lin = self.W["lm_head_q"]
        if vocab is None or (counts is None and vocab >= V):
            self.draft_ids, self.draft_W = None, None
            return
        if counts is None:
            rows = np.arange(min(vocab, V))
            self.draft_ids = None
        else:
            top = set(np.argsort(-np.asarray(counts)[:V])[:vocab].tolist()) | {int(e) for e in extra_ids}
            rows = np.array(sorted(top), dtype=np.int64)
            self.draft_ids = rows.astype(np.int32)
        self.draft_W = tuple(np.ascontiguousarray(t[rows]) for t in lin)

    def make_cache(self):
        a = self.a
        cache = []
        for i in range(a.layers):
            if a.is_linear(i):
                cache.append(GDNCache(np.zeros((a.conv_k - 1, a.conv_dim), np.uint16),
                                      np.zeros((a.lin_hv, a.lin_dv, a.lin_dk), np.float32)))
            else:
                cache.append(self._kv())
        return cache

    def _kv(self):
        a = self.a
        z = np.zeros((a.n_kv, a.max_pos, a.head_dim), np.uint16)
        return KVCache(z, z.copy())

    # -- token mixers
    def gdn(self, i, x, c: GDNCache, snap: bool):
        a, L = self.a, self.W[f"layers.{i}"]
        S = x.shape[0]
        proj = qmv(x, L["in_proj"])  # [S, qkv | z | b | a]
        C, Z = a.conv_dim, a.lin_hv * a.lin_dv
        win = np.concatenate([c.conv, proj[:, :C]], axis=0)
        y, st, mids = ops.gdn_fused(win, L["conv1d"], proj[:, C + Z + a.lin_hv:], proj[:, C + Z:C + Z + a.lin_hv],
                                    L["A_log"], L["dt_bias"], c.state, a.lin_hk, a.lin_hv, a.lin_dk, a.lin_dv,
                                    a.conv_k, snap=snap and S > 1)
        if snap and S > 1:
            c.rollback = (win, mids)
        c.conv = win[-(a.conv_k - 1):].copy()
        c.state = st
        out = ops.gdn_norm_gate(y, proj[:, C:C + Z], L["norm"], a.eps)
        return qmv(out, L["out_proj"])

    def attn(self, L, x, c: KVCache):
        a = self.a
        S = x.shape[0]
        qkv = qmv(x, L["qkv_proj"])
        q = np.empty((S, a.n_heads, a.head_dim), np.uint16)
        g = np.empty_like(q)
        ops.lib().qo_attn_prep(_P(qkv.ctypes.data), _I(qkv.shape[1]), _I(S), _I(a.n_heads), _I(a.n_kv),
                               _I(a.head_dim), _I(a.rotary_dim), _P(_c(L["q_norm"], np.uint16).ctypes.data),
                               _P(_c(L["k_norm"], np.uint16).ctypes.data), ops.ctypes.c_float(a.eps),
                               _P(self.cos.ctypes.data), _P(self.sin.ctypes.data), _I(c.offset), _P(q.ctypes.data),
                               _P(g.ctypes.data), _P(c.k.ctypes.data), _P(c.v.ctypes.data), _I(a.max_pos))
        o = np.empty((S, a.n_heads * a.head_dim), np.uint16)
        ops.lib().qo_attention(_P(q.ctypes.data), _P(g.ctypes.data), _P(c.k.ctypes.data), _P(c.v.ctypes.data),
                               _I(a.max_pos), _I(S), _I(a.n_heads), _I(a.n_kv), _I(a.head_dim), _I(c.offset),
                               _P(o.ctypes.data))
        c.offset += S
        return qmv(o, L["o_proj"])

    def mlp(self, L, x):
        a = self.a
        gu = qmv(x, L["gate_up"])
        act = np.empty((x.shape[0], a.intermediate), np.uint16)
        ops.lib().qo_swiglu(_P(gu.ctypes.data), _I(gu.shape[1]), _I(x.shape[0]), _I(a.intermediate),
                            _P(act.ctypes.data))
        return qmv(act, L["down"])

    def decoder_layer(self, L, x, mixer):
        h = add(x, mixer(rmsnorm(x, L["input_ln"], self.a.eps)))
        return add(h, self.mlp(L, rmsnorm(h, L["post_ln"], self.a.eps)))

    # -- mtp.py:143-153
    def backbone(self, tokens, cache, snap=False):
        a, W = self.a, self.W
        h = embed(tokens, *W["embed"], a.hidden)
        for i in range(a.layers):
            L = W[f"layers.{i}"]
            if a.is_linear(i):
                h = self.decoder_layer(L, h, lambda x, i=i: self.gdn(i, x, cache[i], snap))
            else:
                h = self.decoder_layer(L, h, lambda x, L=L, i=i: self.attn(L, x, cache[i]))
        hn = rmsnorm(h, W["norm"], a.eps)
        return h, hn

    def head(self, hn, k=64):
        """Two-stage head (lm_head2.py:23-29) + greedy argmax per row."""
        wq, s, b = self.W["lm_head_q"]
        _, idx, fine, amax = ops.two_stage_head(hn, wq, s, b, self.W["lm_head"], k)
        return amax

    def candidates(self, hn, K):
        """Two-stage head candidates (vocabulary ids int32 [M, K], exact logits bf16 [M, K])."""
        wq, s, b = self.W["lm_head_q"]
        _, idx, fine, _ = ops.two_stage_head(hn, wq, s, b, self.W["lm_head"], K)
        return idx, fine

    def _sample(self, hn, sp, ctr, drafts=None):
        """engine.py:110-152 through the C sampler: first token (drafts None) or a verify decision."""
        K = sampling_k(sp)
        idx, fine = self.candidates(hn, K)
        seed = int(sp.seed or 0)
        kw = dict(temperature=sp.temperature, top_k=sp.top_k, top_p=sp.top_p, min_p=sp.min_p, V=self.a.vocab,
                  seed=seed, ctr=ctr)
        if drafts is None:
            return ops.sample(idx, fine, None, first_row=idx.shape[0] - 1, **kw)
        return ops.sample(idx, fine, drafts, **kw)

    def draft_token(self, xn, with_prob=False):
        """Draft head: full-vocabulary 4-bit head (bench_ab.py:24 DRAFT_HEAD, engine.py:46-48) + argmax;
        with_prob: also the probability of the argmax (mtp.py:222-223)."""
        logits = qmv(xn, self.W["lm_head_q"] if self.draft_W is None else self.draft_W)
        i = ops.argmax_bf16(logits)
        d = i if self.draft_ids is None else self.draft_ids[i]
        return (d, ops.draft_prob(logits[0], int(i[0]))) if with_prob else d

    # -- mtp.py:199-209
    def mtp_step(self, hidden, tokens, mcache, with_prob=False):
        a, M = self.a, self.W["mtp"]
        e = rmsnorm(embed(tokens, *self.W["embed"], a.hidden), M["pre_fc_norm_embedding"], a.eps)
        hh = rmsnorm(hidden, M["pre_fc_norm_hidden"], a.eps)
        x = qmv(np.concatenate([e, hh], axis=1), M["fc"])
        L = M["layer"]
        x = self.decoder_layer(L, x, lambda y: self.attn(L, y, mcache))
        x_last = x[-1:]
        xn = rmsnorm(x_last, M["norm"], a.eps)
        if with_prob:
            d, p = self.draft_token(xn, True)
            return d, x_last, p
        return self.draft_token(xn), x_last

    # -- mtp.py:212-226 (chain="pre")
    def draft_chain(self, hidden, tokens, mcache, k, with_probs=False):
        r = self.mtp_step(hidden, tokens, mcache, with_probs)
        drafts, probs = [int(r[0][0])], [r[2]] if with_probs else []
        x = r[1]
        for _ in range(1, k):
            r = self.mtp_step(x, np.int32([drafts[-1]]), mcache, with_probs)
            x = r[1]
            drafts.append(int(r[0][0]))
            if with_probs:
                probs.append(r[2])
        return (drafts, probs) if with_probs else drafts

    # -- mtp.py:241-303 / engine.py:121-128 (greedy)
    def generate_greedy(self, prompt_ids, max_tokens, eos=()):
        """Plain greedy decoding, one token per backbone call (stream_generate in mtp.py:351-369)."""
        cache = self.make_cache()
        h, hn = self.backbone(np.int32(prompt_ids), cache)
        out = [int(self.head(hn[-1:])[0])]
        while len(out) < max_tokens and out[-1] not in eos:
            h, hn = self.backbone(np.int32([out[-1]]), cache)
            out.append(int(self.head(hn)[0]))
        return out

    def prefill(self, prompt_ids, k=2, sampling=None, tau=None):
        """mtp.py:258-263: prompt pass, first token t, first drafts; returns (cache, mcache, t, drafts).
        With sampling (temperature > 0) the first token is drawn (engine.py:110-115, call counter 0)."""
        cache = self.make_cache()
        mcache = self._kv()
        p = np.int32(prompt_ids)
        h, hn = self.backbone(p, cache)
        t = int(self._sample(hn[-1:], sampling, 0)) if _sampled(sampling) else int(self.head(hn[-1:])[0])
        drafts = self.draft_chain(h, np.concatenate([p[1:], np.int32([t])]), mcache, k, tau is not None)
        return cache, mcache, t, drafts

    def decode(self, cache, mcache, t, drafts, max_tokens, eos=(), k=2, max_cycles=None, draft_override=None,
               sampling=None, rng_ctr=1, tau=None):
        """The verify loop of mtp.py:268-294 from a given state; returns (out tokens incl. t, stats).
        With sampling (temperature > 0) each cycle decides by exact speculative sampling (engine.py:
        121-152) with call counter rng_ctr, rng_ctr + 1, ..."""
        t0 = time.perf_counter()
        out = [t]
        cycles = verified = 0
        acc_pos = [0] * k
        # adaptive k (mtp.py:229-238): drafts arrive with their probabilities; only the first
        # n_drafts(probs, tau) may be accepted (verifying all k rows gives the same rows: batch-invariant)
        n_use = k
        if tau is not None:
            drafts, probs = drafts
            n_use = ops.n_drafts(probs, tau)
        while len(out) < max_tokens and out[-1] not in eos:
            if max_cycles is not None and cycles >= max_cycles:
                break
            S = k + 1
            if draft_override is not None:
                o = draft_override(cycles)
                if o is not None:
                    drafts = [int(v) for v in o]
            h, hn = self.backbone(np.int32([t] + drafts), cache, snap=True)
            if _sampled(sampling):
                n_acc, av = self._sample(hn, sampling, rng_ctr, drafts)
                rng_ctr += 1
                for i in range(n_acc):
                    acc_pos[i] += 1
            else:
                av = [int(v) for v in self.head(hn)]
                n_acc = 0
                while n_acc < n_use and av[n_acc] == drafts[n_acc]:
                    acc_pos[n_acc] += 1
                    n_acc += 1
            cycles += 1
            verified += n_use
            keep = n_acc + 1
            out += av[:keep]
            if keep < S:
                for i, c in enumerate(cache):
                    if self.a.is_linear(i):
                        self.restore(c, keep)
                    else:
                        c.trim(S - keep)
            mcache.trim(k - 1)
            t = av[keep - 1]
            drafts = self.draft_chain(h[:keep], np.int32(av[:keep]), mcache, k, tau is not None)
            if tau is not None:
                drafts, probs = drafts
                n_use = ops.n_drafts(probs, tau)
        dt = time.perf_counter() - t0
        for i, tok in enumerate(out):
            if tok in eos:
                out = out[:i + 1]
                break
        out = out[:max_tokens]
        stats = {"tps": (len(out) - 1) / dt if dt > 0 else 0.0, "tok_ciclo": (len(out) - 1) / max(cycles, 1),
                 "acept": [n / max(cycles, 1) for n in acc_pos], "borradores_ciclo": verified / max(cycles, 1),
                 "cycles": cycles, "seconds": dt, "tokens": max(len(out) - 1, 0), "next": (t, drafts)}
        return out, stats

    def load_state(self, layers, mtp):
        """Caches from exported engine state (qmtp.mtp.export_state): lets the decode loop start
        from the B200 engine's post-prefill state (full-size CPU samples without a CPU prefill)."""
        cache = []
        for entry in layers:
            if entry[0] == "gdn":
                cache.append(GDNCache(entry[1].copy(), entry[2].astype(np.float32).copy()))
            else:
                cache.append(KVCache(entry[1].copy(), entry[2].copy(), int(entry[3])))
        return cache, KVCache(mtp[0].copy(), mtp[1].copy(), int(mtp[2]))

    def generate_mtp(self, prompt_ids, max_tokens, eos=(), k=2, max_cycles=None, draft_override=None,
                     sampling=None, tau=None):
        """mtp.py:241-303 (fixed k; greedy, or sampled when sampling.temperature > 0).
        draft_override(cycle) -> list of k tokens or None replaces the drafts a cycle verifies (test
        hook for acceptance and rollback; the MTP caches still follow the computed drafts)."""
        cache, mcache, t, drafts = self.prefill(prompt_ids, k, sampling, tau)
        return self.decode(cache, mcache, t, drafts, max_tokens, eos, k, max_cycles, draft_override, sampling,
                           tau=tau)

    # -- mtp.py:136-140
    def restore(self, c: GDNCache, keep: int) -> None:
        win, mids = c.rollback
        n_keep = self.a.conv_k - 1
        c.conv = win[keep:keep + n_keep].copy()
        c.state = mids[keep - 1].copy() if keep - 1 < mids.shape[0] else c.state


def _sampled(sp) -> bool:
    return sp is not None and sp.temperature > 0


def sampling_k(sp) -> int:
    """lm_head2.py:32-36 k_for: head candidates for a sampling configuration."""
    if sp is None or sp.temperature <= 0 or 0 < sp.top_k <= 32:
        return 64
    return 256 if sp.top_k <= 0 else min(4 * sp.top_k, 2048)


# ------------------------------------------------------------------ synthetic weights
def synthetic_weights(args: ModelArgs, seed: int = 0, std: float = 0.02) -> dict:
    """Seeded random-init weights in numpy (small configs; the B200 engine makes full-size ones on
    the GPU and the oracle can be fed those instead).  Linear weights N(0, std) -> affine g64."""
    rng = np.random.default_rng(seed)

    def bf(shape, scale=std):
        return ops.f32_to_bf16(rng.standard_normal(shape, dtype=np.float32) * np.float32(scale))

    def lin(n, k):
        return ops.quantize_affine(bf((n, k)))

    ones = lambda n: ops.f32_to_bf16(np.ones(n, np.float32))
    a = args
    W = {}
    W["embed"] = lin(a.vocab, a.hidden)
    for i in range(a.layers):
        L = {"input_ln": ones(a.hidden), "post_ln": ones(a.hidden), "gate_up": lin(2 * a.intermediate, a.hidden),
             "down": lin(a.hidden, a.intermediate)}
        if a.is_linear(i):
            L.update(in_proj=lin(a.gdn_proj, a.hidden), conv1d=bf((a.conv_dim, a.conv_k), 1.0 / np.sqrt(a.conv_k)),
                     A_log=np.log(rng.uniform(1, 16, a.lin_hv)).astype(np.float32), dt_bias=bf((a.lin_hv,), 1.0),
                     norm=ones(a.lin_dv), out_proj=lin(a.hidden, a.lin_hv * a.lin_dv))
        else:
            L.update(qkv_proj=lin(a.attn_proj, a.hidden), q_norm=ones(a.head_dim), k_norm=ones(a.head_dim),
                     o_proj=lin(a.hidden, a.n_heads * a.head_dim))
        W[f"layers.{i}"] = L
    W["norm"] = ones(a.hidden)
    W["lm_head"] = bf((a.vocab, a.hidden))
    W["lm_head_q"] = ops.quantize_affine(W["lm_head"])
    W["mtp"] = {"pre_fc_norm_embedding": ones(a.hidden), "pre_fc_norm_hidden": ones(a.hidden),
                "fc": lin(a.hidden, 2 * a.hidden), "norm": ones(a.hidden),
                "layer": {"input_ln": ones(a.hidden), "post_ln": ones(a.hidden),
                          "qkv_proj": lin(a.attn_proj, a.hidden), "q_norm": ones(a.head_dim),
                          "k_norm": ones(a.head_dim), "o_proj": lin(a.hidden, a.n_heads * a.head_dim),
                          "gate_up": lin(2 * a.intermediate, a.hidden), "down": lin(a.hidden, a.intermediate)}}
    return W


def synthetic_weights_seeded(args: ModelArgs, seed: int = 0, std: float = 0.02, threads: int | None = None) -> dict:
    """Full-size seeded random-init weights, reproducible on any machine and generated in parallel:
    the tensors are listed in a fixed order and cut into chunks of at most 2^24 elements; chunk i of
    the list draws from np.random.default_rng(SeedSequence(seed).spawn(n)[i]).  Distributions as
    synthetic_weights (linear N(0, std) -> affine g64 by the oracle quantizer, norms 1, conv
    N(0, 1/KC), A_log = log U(1, 16), dt_bias N(0, 1)); the numbers differ from synthetic_weights'."""
    import os
    from concurrent.futures import ThreadPoolExecutor

    a = args
    specs = []  # (path, kind, shape, scale)
    ones = lambda n: ops.f32_to_bf16(np.ones(n, np.float32))

    def lin(path, n, k):
        specs.append((path, "lin", (n, k), std))

    def bf(path, shape, scale):
        specs.append((path, "bf", shape, scale))

    lin(("embed",), a.vocab, a.hidden)
    for i in range(a.layers):
        L = f"layers.{i}"
        lin((L, "gate_up"), 2 * a.intermediate, a.hidden)
        lin((L, "down"), a.hidden, a.intermediate)
        if a.is_linear(i):
            lin((L, "in_proj"), a.gdn_proj, a.hidden)
            bf((L, "conv1d"), (a.conv_dim, a.conv_k), 1.0 / np.sqrt(a.conv_k))
            specs.append(((L, "A_log"), "alog", (a.lin_hv,), 0.0))
            bf((L, "dt_bias"), (a.lin_hv,), 1.0)
            lin((L, "out_proj"), a.hidden, a.lin_hv * a.lin_dv)
        else:
            lin((L, "qkv_proj"), a.attn_proj, a.hidden)
            lin((L, "o_proj"), a.hidden, a.n_heads * a.head_dim)
    bf(("lm_head",), (a.vocab, a.hidden), std)
    lin(("mtp", "fc"), a.hidden, 2 * a.hidden)
    for name, n, k in (("qkv_proj", a.attn_proj, a.hidden), ("o_proj", a.hidden, a.n_heads * a.head_dim),
                       ("gate_up", 2 * a.intermediate, a.hidden), ("down", a.hidden, a.intermediate)):
        lin(("mtp", "layer", name), n, k)

    CH = 1 << 24
    chunks = []  # (spec index, flat start, flat end)
    for si, (_, _, shape, _) in enumerate(specs):
        n = int(np.prod(shape))
        chunks += [(si, o, min(o + CH, n)) for o in range(0, n, CH)]
    seeds = np.random.SeedSequence(seed).spawn(len(chunks))
    bufs = [np.empty(int(np.prod(sp[2])), np.uint16 if sp[1] != "alog" else np.float32) for sp in specs]

    def fill(ci):
        si, o0, o1 = chunks[ci]
        _, kind, _, scale = specs[si]
        rng = np.random.default_rng(seeds[ci])
        if kind == "alog":
            bufs[si][o0:o1] = np.log(rng.uniform(1, 16, o1 - o0)).astype(np.float32)
        else:
            bufs[si][o0:o1] = ops.f32_to_bf16(rng.standard_normal(o1 - o0, dtype=np.float32) * np.float32(scale))

    with ThreadPoolExecutor(threads or os.cpu_count()) as ex:
        list(ex.map(fill, range(len(chunks))))
    W = {"mtp": {"layer": {}}}
    for (path, kind, shape, _), buf in zip(specs, bufs):
        v = buf.reshape(shape)
        if kind == "lin":
            v = ops.quantize_affine(v)
        d = W
        for key in path[:-1]:
            d = d.setdefault(key, {})
        d[path[-1]] = v
    W["lm_head_q"] = ops.quantize_affine(W["lm_head"])
    W["norm"] = ones(a.hidden)
    for i in range(a.layers):
        L = W[f"layers.{i}"]
        L.update(input_ln=ones(a.hidden), post_ln=ones(a.hidden))
        if a.is_linear(i):
            L["norm"] = ones(a.lin_dv)
        else:
            L.update(q_norm=ones(a.head_dim), k_norm=ones(a.head_dim))
    M = W["mtp"]
    M.update(pre_fc_norm_embedding=ones(a.hidden), pre_fc_norm_hidden=ones(a.hidden), norm=ones(a.hidden))
    M["layer"].update(input_ln=ones(a.hidden), post_ln=ones(a.hidden), q_norm=ones(a.head_dim),
                      k_norm=ones(a.head_dim))
    return W


def synthetic_weights_fast(args: ModelArgs, seed: int = 0, std: float = 0.02) -> dict:
    """Full-size random weights for CPU timing runs: packed nibbles drawn uniformly and per-group
    scales / biases with the magnitudes an N(0, std) group quantizes to ((max-min)/15 ~ 0.3*std,
    min ~ -2.5*std); the bf16 lm_head is N(0, std) and its coarse copy is quantized from it.  Same
    shapes, formats and per-token work as synthetic_weights, generated in seconds."""
    rng = np.random.default_rng(seed)

    def lin(n, k):
        wq = rng.integers(0, 2 ** 32, (n, k // 8), dtype=np.uint32)
        s = ops.f32_to_bf16((0.3 * std + 0.03 * std * rng.standard_normal((n, k // 64))).astype(np.float32))
        b = ops.f32_to_bf16((-2.5 * std + 0.25 * std * rng.standard_normal((n, k // 64))).astype(np.float32))
        return wq, s, b

    ones = lambda n: ops.f32_to_bf16(np.ones(n, np.float32))
    bf = lambda shape, sc: ops.f32_to_bf16(rng.standard_normal(shape, dtype=np.float32) * np.float32(sc))
    a = args
    W = {"embed": lin(a.vocab, a.hidden)}
    for i in range(a.layers):
        L = {"input_ln": ones(a.hidden), "post_ln": ones(a.hidden), "gate_up": lin(2 * a.intermediate, a.hidden),
             "down": lin(a.hidden, a.intermediate)}
        if a.is_linear(i):
            L.update(in_proj=lin(a.gdn_proj, a.hidden), conv1d=bf((a.conv_dim, a.conv_k), 1.0 / np.sqrt(a.conv_k)),
                     A_log=np.log(rng.uniform(1, 16, a.lin_hv)).astype(np.float32), dt_bias=bf((a.lin_hv,), 1.0),
                     norm=ones(a.lin_dv), out_proj=lin(a.hidden, a.lin_hv * a.lin_dv))
        else:
            L.update(qkv_proj=lin(a.attn_proj, a.hidden), q_norm=ones(a.head_dim), k_norm=ones(a.head_dim),
                     o_proj=lin(a.hidden, a.n_heads * a.head_dim))
        W[f"layers.{i}"] = L
    W["norm"] = ones(a.hidden)
    W["lm_head"] = bf((a.vocab, a.hidden), std)
    W["lm_head_q"] = ops.quantize_affine(W["lm_head"])
    W["mtp"] = {"pre_fc_norm_embedding": ones(a.hidden), "pre_fc_norm_hidden": ones(a.hidden),
                "fc": lin(a.hidden, 2 * a.hidden), "norm": ones(a.hidden),
                "layer": {"input_ln": ones(a.hidden), "post_ln": ones(a.hidden),
                          "qkv_proj": lin(a.attn_proj, a.hidden), "q_norm": ones(a.head_dim),
                          "k_norm": ones(a.head_dim), "o_proj": lin(a.hidden, a.n_heads * a.head_dim),
                          "gate_up": lin(2 * a.intermediate, a.hidden), "down": lin(a.hidden, a.intermediate)}}
    return W
