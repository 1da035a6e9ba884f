"""Generation engine on B200 -- the engine.py surface of qwen-mtp-mac (the swap point the server uses).

Reference: engine.py:28-34 ``Sampling``, engine.py:37-213 ``Engine`` (``generate(ids, prefix_len,
max_tokens, sp, stats)``: a token iterator with the prompt-prefix state cache, greedy verification or
exact speculative sampling) and engine.py:216-274 ``Job`` / ``Worker`` (one thread owns the model).

The reference loads Qwen3.5 from Ollama blobs and patches MLX; here the engine takes a model handle
(``qmtp.model.Model``: configuration + device weights, synthetic or read by ``qmtp.loader``) and runs
every cycle as one replay of a captured CUDA graph (``MTPDecoder``).  The decoder keeps the prompt
prefix cache between requests, as the reference's snapshot does (engine.py:52-88).
"""
from __future__ import annotations

import queue
import threading
import time
from dataclasses import dataclass, field

from .mtp import MTPDecoder, Sampling
from .model import Model

PREFILL_CHUNK = 2048  # engine.py:25; the B200 prefill runs in verify-shaped chunks (MTPDecoder.prefill)

__all__ = ["Engine", "Job", "Worker", "Sampling", "PREFILL_CHUNK"]


class Engine:
    """engine.py:37-213 over a B200 decoder.  ``model``: a qmtp.model.Model; ``eos``: end-of-sequence
    token ids (the tokenizer's, engine.py:46); ``max_context``: prompt + generated tokens a request
    may hold (bounded by the model's KV-cache length)."""

    def __init__(self, model: Model, k: int = 2, eos=(), max_context: int | None = None, draft_vocab: int = 65536,
                 draft_counts=None):
        """draft_vocab / draft_counts: engine.py:38,46-48 -- with corpus counts (build_draft_vocab.py's
        file or array) the draft head scores the draft_vocab most frequent ids plus the EOS ids
        (load_draft_head(..., freq=True)); without, the full-vocabulary head."""
        from .mtp import load_draft_head

        self.lm = model
        self.k = k
        self.eos = set(int(t) for t in eos)
        self.max_context = min(max_context or model.args.max_pos, model.args.max_pos)
        head = None
        if draft_counts is not None:
            head = load_draft_head(draft_vocab, {"bits": 4, "group_size": 64}, True, sorted(self.eos), lm=model,
                                   counts=draft_counts)
        self.head = head
        self.dec = MTPDecoder(model.args, model.weights, k=k, max_tokens=self.max_context,
                              device=model.weights["norm"].device, draft_head=head)

    @classmethod
    def from_checkpoint(cls, path, k: int = 2, eos=(), mtp_files=(), max_pos: int = 4096, device="cuda"):
        """A model directory read by qmtp.loader (config.json + safetensors shards; the MTP tensors
        in the checkpoint or in mtp_files, as the reference's fetch_mtp.py writes them)."""
        from . import loader

        config, files = loader.checkpoint_dir(path)
        args, W = loader.load(files, config, mtp_files=mtp_files, max_pos=max_pos, device=device)
        return cls(Model(args, W), k=k, eos=eos)

    def generate(self, ids, prefix_len, max_tokens, sp: Sampling, stats: dict):
        """engine.py:155-213: yields the generated tokens of prompt `ids`.  prefix_len: tokens of the
        prompt before the generation prompt (the reusable snapshot point).  stats receives t_start,
        prompt_tokens, cached_tokens, t_first, then cycles, accepted and k (the reference's keys) and
        tps / tok_ciclo."""
        t0 = time.perf_counter()
        stats["t_start"] = t0
        ids = [int(t) for t in ids]
        if not ids:
            raise ValueError("empty prompt")
        if len(ids) + max_tokens + self.k + 1 > self.max_context:
            raise ValueError(f"prompt ({len(ids)}) + max_tokens ({max_tokens}) exceed the context of "
                             f"{self.max_context} tokens")
        dec = self.dec
        dec.set_sampling(sp if sp is not None and sp.temperature > 0 else None)
        prefix_len = min(int(prefix_len), len(ids) - 1)
        first = dec.prefill(ids, prefix_len)
        stats.update(prompt_tokens=len(ids), cached_tokens=dec.cached_tokens, t_first=time.perf_counter())
        n_out = 1
        yield first
        done = first in self.eos or n_out >= max_tokens
        cycles = 0
        acc0 = list(dec.ctrl.tolist()[10:10 + self.k])
        t1 = time.perf_counter()
        if not done:
            dec.ensure_graph()
        while not done:
            emitted = dec.run_cycle()
            cycles += 1
            for tok in emitted:
                n_out += 1
                yield tok
                if tok in self.eos or n_out >= max_tokens:
                    done = True
                    break
        acc = dec.ctrl.tolist()[10:10 + self.k]
        dt = time.perf_counter() - t1
        stats.update(cycles=cycles, accepted=int(sum(a - b for a, b in zip(acc, acc0))), k=self.k,
                     tps=(n_out - 1) / dt if dt > 0 else 0.0, tok_ciclo=(n_out - 1) / max(cycles, 1))


@dataclass
class Job:
    """engine.py:216-238: a request in flight; tokens() streams them and re-raises a worker error."""
    args: tuple
    out: queue.Queue = field(default_factory=queue.Queue)
    cancel: threading.Event = field(default_factory=threading.Event)
    stats: dict = field(default_factory=dict)
    error: Exception | None = None
    done: bool = False

    def tokens(self):
        while not self.done:
            t = self.out.get()
            if t is None:
                self.done = True
                break
            yield t
        if self.error:
            raise self.error


class Worker:
    """engine.py:241-274: one thread owns the engine (and its CUDA stream); requests queue up."""

    def __init__(self, engine_factory, **kw):
        self.jobs: queue.Queue = queue.Queue()
        self._ready = threading.Event()
        self._init_error = None
        self._thread = threading.Thread(target=self._loop, args=(engine_factory, kw), daemon=True)
        self._thread.start()
        self._ready.wait()
        if self._init_error:
            raise self._init_error

    def _loop(self, factory, kw):
        try:
            self.engine = factory(**kw)
        except Exception as e:  # noqa: BLE001 - re-raised in the submitting thread
            self._init_error = e
            self._ready.set()
            return
        self._ready.set()
        while True:
            job = self.jobs.get()
            if job is None:
                return
            try:
                for t in self.engine.generate(*job.args, job.stats):
                    if job.cancel.is_set():
                        break
                    job.out.put(t)
            except Exception as e:  # noqa: BLE001
                job.error = e
            finally:
                job.out.put(None)

    def submit(self, ids, prefix_len, max_tokens, sp) -> Job:
        job = Job((ids, prefix_len, max_tokens, sp))
        self.jobs.put(job)
        return job

    def close(self):
        self.jobs.put(None)
        self._thread.join(timeout=60)
