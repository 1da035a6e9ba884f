"""Checkpoint loading for the B200 decoder: safetensors files -> ``qmtp.model.Weights``.

What the reference does at load time, restated for this engine's weight layout:

* ``qwen_ollama.py:22-28``: an Ollama model is a manifest whose layers are blobs; JSON layers
  (config.json, tokenizer files) and tensor layers (one safetensors file per blob).
  ``ollama_checkpoint`` resolves the same manifest and returns the config and the tensor files.
* ``qwen_ollama.py:43-50``: tensors whose name starts with ``vision_tower`` are skipped and
  ``.weight.scale`` is renamed ``.scales`` (``sanitize_names``).
* ``mtp.py:61-66``: the MTP tensors come raw from the Hugging Face checkpoint, where Qwen3.5's
  zero-centred RMSNorms store ``w - 1``; every 1-D MTP tensor gets ``+ 1`` (``load_mtp_tensors``).
* ``mtp.py:35-57`` / mlx-lm ``qwen3_5``: the module names of the trunk and of the MTP layer.

The decoder serves two 4-bit linear formats: affine group 64 (the MLX ``quantize(w, 64, 4)``
format: uint32 words of 8 nibbles, bf16 scales and biases per 64 inputs) and NVFP4 (the same nibble
words holding e2m1 values, one e4m3 ``uint8`` scale per 16 inputs, no biases; the format of the Ollama
``qwen3.5:9b-mlx`` blobs, qwen_ollama.py:20).  A checkpoint linear in either format is used as stored;
a bf16 linear is quantized to affine g64 on the GPU at load time (the reference quantizes the MTP head
at load too, ``mtp.py:67-68``).  Other quantized formats are rejected with an error.

Projections that read the same input are concatenated along the output rows, as ``qmtp.model``
documents: GatedDeltaNet ``[in_proj_qkv | in_proj_z | in_proj_b | in_proj_a]``, attention
``[q_proj (per head: query, gate) | k_proj | v_proj]``, MLP ``[gate_proj | up_proj]``.  Per-row
quantization makes the concatenation exact.
"""
from __future__ import annotations

import json
import struct
from dataclasses import dataclass
from pathlib import Path
from typing import Iterable

import numpy as np

from .model import ModelArgs, Weights

# ----------------------------------------------------------------------------------- safetensors
_DTYPES = {"BF16": np.uint16, "F16": np.float16, "F32": np.float32, "F64": np.float64, "U8": np.uint8,
           "I8": np.int8, "U16": np.uint16, "I16": np.int16, "U32": np.uint32, "I32": np.int32,
           "U64": np.uint64, "I64": np.int64, "BOOL": np.bool_}
_NAMES = {np.dtype(np.float16): "F16", np.dtype(np.float32): "F32", np.dtype(np.float64): "F64",
          np.dtype(np.uint8): "U8", np.dtype(np.int8): "I8", np.dtype(np.int16): "I16",
          np.dtype(np.uint32): "U32", np.dtype(np.int32): "I32", np.dtype(np.uint64): "U64",
          np.dtype(np.int64): "I64", np.dtype(np.bool_): "BOOL"}


def read_safetensors(path) -> dict[str, np.ndarray]:
    """Tensors of one safetensors file (8-byte little-endian header length, JSON header, data).
    BF16 tensors come back as their uint16 bit patterns.  The file is memory-mapped."""
    path = Path(path)
    size = path.stat().st_size
    with open(path, "rb") as f:
        head = f.read(8)
        if len(head) != 8:
            raise ValueError(f"{path}: not a safetensors file (short header)")
        n = struct.unpack("<Q", head)[0]
        if n > size - 8:
            raise ValueError(f"{path}: header length {n} exceeds the file")
        header = json.loads(f.read(n))
    data = np.memmap(path, dtype=np.uint8, mode="r", offset=8 + n) if size > 8 + n else np.zeros(0, np.uint8)
    out = {}
    for name, meta in header.items():
        if name == "__metadata__":
            continue
        dt = meta["dtype"]
        if dt not in _DTYPES:
            raise ValueError(f"{path}: tensor {name} has unsupported dtype {dt}")
        a, b = meta["data_offsets"]
        shape = tuple(meta["shape"])
        item = np.dtype(_DTYPES[dt]).itemsize
        if not (0 <= a <= b <= data.size) or (b - a) != item * int(np.prod(shape, dtype=np.int64)):
            raise ValueError(f"{path}: tensor {name} has inconsistent offsets {a}..{b} for {dt}{list(shape)}")
        out[name] = np.frombuffer(data, dtype=_DTYPES[dt], count=(b - a) // item, offset=a).reshape(shape)
    return out


def write_safetensors(path, tensors: dict, bf16: Iterable[str] = ()) -> None:
    """Writes numpy arrays as one safetensors file; names in ``bf16`` (uint16 arrays) are tagged BF16."""
    bf16 = set(bf16)
    header, off, blobs = {}, 0, []
    for name, arr in tensors.items():
        arr = np.ascontiguousarray(arr)
        if name in bf16:
            if arr.dtype != np.uint16:
                raise ValueError(f"{name}: bf16 tensors are passed as uint16 bit patterns")
            dt = "BF16"
        elif arr.dtype == np.uint16:
            dt = "U16"
        else:
            dt = _NAMES[arr.dtype]
        raw = arr.tobytes()
        header[name] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    hj = json.dumps(header, separators=(",", ":")).encode()
    hj += b" " * ((8 - len(hj) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        for raw in blobs:
            f.write(raw)


# ----------------------------------------------------------------------------------- names
_PREFIXES = ("model.language_model.", "language_model.model.", "language_model.", "model.")


def sanitize_names(tensors: dict) -> dict:
    """qwen_ollama.py:45-50: drop vision tensors, ``.weight.scale`` -> ``.scales``; then strip the
    wrapper prefixes so trunk names read ``layers.{i}...``, ``embed_tokens...``, ``norm...``, ``lm_head...``."""
    out = {}
    for k, v in tensors.items():
        if k.startswith("vision_tower") or k.startswith("model.visual") or ".vision_tower." in k:
            continue
        k = k.replace(".weight.scale", ".scales")
        for p in _PREFIXES:
            if k.startswith(p):
                k = k[len(p):]
                break
        if k in out:
            raise ValueError(f"duplicate tensor after renaming: {k}")
        out[k] = v
    return out


def args_from_config(config: dict, max_pos: int = 1024) -> ModelArgs:
    """ModelArgs from a Qwen3.5 ``config.json`` (top level or its ``text_config``)."""
    c = config.get("text_config", config)
    rope = c.get("rope_parameters") or c.get("rope_scaling") or {}
    head_dim = int(c.get("head_dim", c["hidden_size"] // c["num_attention_heads"]))
    prf = float(c.get("partial_rotary_factor", rope.get("partial_rotary_factor", 0.25)))
    a = ModelArgs(hidden=int(c["hidden_size"]), layers=int(c["num_hidden_layers"]),
                  intermediate=int(c["intermediate_size"]), n_heads=int(c["num_attention_heads"]),
                  n_kv=int(c["num_key_value_heads"]), head_dim=head_dim, rotary_dim=int(head_dim * prf),
                  rope_theta=float(c.get("rope_theta", rope.get("rope_theta", 10_000_000.0))),
                  vocab=int(c["vocab_size"]), lin_hk=int(c["linear_num_key_heads"]),
                  lin_hv=int(c["linear_num_value_heads"]), lin_dk=int(c["linear_key_head_dim"]),
                  lin_dv=int(c["linear_value_head_dim"]), conv_k=int(c["linear_conv_kernel_dim"]),
                  eps=float(c["rms_norm_eps"]), full_attention_interval=int(c.get("full_attention_interval", 4)),
                  max_pos=int(max_pos))
    types = c.get("layer_types")
    if types is not None:
        want = ["linear_attention" if a.is_linear(i) else "full_attention" for i in range(a.layers)]
        if list(types) != want:
            raise NotImplementedError("layer_types is not the fixed every-Nth-layer attention pattern this "
                                      "decoder implements")
    return a


# ----------------------------------------------------------------------------------- layout
@dataclass
class Bf16Linear:
    """A bf16 [N, K] linear (uint16 bits) still to be quantized to affine g64 on the GPU."""
    w: np.ndarray


def _bf16_array(v: np.ndarray, name: str) -> np.ndarray:
    if v.dtype == np.uint16:
        return v
    if v.dtype == np.float32:  # exact bf16 values stored as f32 are accepted; anything else rounds
        u = v.view(np.uint32)
        return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    raise ValueError(f"{name}: expected bf16 (or f32) values, got {v.dtype}")


def _linear(t: dict, name: str, n: int, k: int):
    """(wq, scales, biases) for an affine-g64 linear, (wq, scales) for an NVFP4 one, or Bf16Linear."""
    w = t.get(name + ".weight")
    if w is None:
        raise KeyError(f"missing tensor {name}.weight")
    s, b = t.get(name + ".scales"), t.get(name + ".biases")
    if s is None:
        w = _bf16_array(w, name)
        if w.shape != (n, k):
            raise ValueError(f"{name}.weight: shape {w.shape}, expected {(n, k)}")
        return Bf16Linear(w)
    w = w.view(np.uint32) if w.dtype in (np.int32, np.uint32) else None
    if b is None and s.dtype == np.uint8 and s.shape == (n, k // 16):
        if w is None or w.shape != (n, k // 8):
            raise ValueError(f"{name}: NVFP4 nibbles must be uint32 [{n}, {k // 8}]")
        return (w, s)
    if b is None or s.dtype != np.uint16 or b.dtype != np.uint16:
        raise NotImplementedError(f"{name}: quantized with a format other than affine 4-bit group 64 or "
                                  "NVFP4 group 16")
    if w is None or w.shape != (n, k // 8) or s.shape != (n, k // 64) or b.shape != (n, k // 64):
        raise ValueError(f"{name}: affine g64 tensors must be uint32 [{n}, {k // 8}] and bf16 [{n}, {k // 64}]")
    return (w, s, b)


def _concat(parts, name):
    """Row-wise concatenation of linears of one input (all quantized or all bf16)."""
    if all(isinstance(p, tuple) for p in parts) and len({len(p) for p in parts}) == 1:
        return tuple(np.concatenate([p[i] for p in parts], axis=0) for i in range(len(parts[0])))
    if all(isinstance(p, Bf16Linear) for p in parts):
        return Bf16Linear(np.concatenate([p.w for p in parts], axis=0))
    raise NotImplementedError(f"{name}: projections of one input in different formats")


def _vec(t: dict, name: str, n: int, plus_one: bool = False, dtype=np.uint16) -> np.ndarray:
    v = t.get(name)
    if v is None:
        raise KeyError(f"missing tensor {name}")
    if dtype == np.uint16:
        v = _bf16_array(np.asarray(v), name).reshape(-1)
        if plus_one:
            v = _bf16_add_one(v)
    else:
        v = np.asarray(v)
        if v.dtype == np.uint16:  # bf16 bits
            v = (v.astype(np.uint32) << 16).view(np.float32)
        v = v.astype(dtype).reshape(-1)
    if v.size != n:
        raise ValueError(f"{name}: {v.size} values, expected {n}")
    return np.ascontiguousarray(v)


def _bf16_add_one(v: np.ndarray) -> np.ndarray:
    """bf16(x + 1) for bf16 bit patterns x: the sum in fp32 (exact for bf16 inputs), rounded to
    nearest-even bf16, as the reference's ``v + 1.0`` on a bf16 array does."""
    f = (v.astype(np.uint32) << 16).view(np.float32) + np.float32(1.0)
    u = f.view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def _attn(t, p, a: ModelArgs, hf_norms: bool):
    H, D = a.hidden, a.head_dim
    q = _linear(t, p + "self_attn.q_proj", 2 * a.n_heads * D, H)
    kk = _linear(t, p + "self_attn.k_proj", a.n_kv * D, H)
    v = _linear(t, p + "self_attn.v_proj", a.n_kv * D, H)
    return {"qkv_proj": _concat([q, kk, v], p + "self_attn"),
            "q_norm": _vec(t, p + "self_attn.q_norm.weight", D, hf_norms),
            "k_norm": _vec(t, p + "self_attn.k_norm.weight", D, hf_norms),
            "o_proj": _linear(t, p + "self_attn.o_proj", H, a.n_heads * D)}


def _mlp(t, p, a: ModelArgs, hf_norms: bool):
    H, I = a.hidden, a.intermediate
    g = _linear(t, p + "mlp.gate_proj", I, H)
    u = _linear(t, p + "mlp.up_proj", I, H)
    return {"input_ln": _vec(t, p + "input_layernorm.weight", H, hf_norms),
            "post_ln": _vec(t, p + "post_attention_layernorm.weight", H, hf_norms),
            "gate_up": _concat([g, u], p + "mlp"), "down": _linear(t, p + "mlp.down_proj", H, I)}


def trunk_layout(tensors: dict, a: ModelArgs, hf_norms: bool = False) -> dict:
    """Numpy weights of the trunk in this engine's layout (the oracle's key names).  ``tensors`` are
    sanitized names.  hf_norms: the zero-centred RMSNorm weights are stored as ``w - 1`` (raw Hugging
    Face tensors) and get ``+ 1``; MLX-converted checkpoints already store ``w``."""
    t = tensors
    H = a.hidden
    W = {"embed": _linear(t, "embed_tokens", a.vocab, H)}
    for i in range(a.layers):
        p = f"layers.{i}."
        L = _mlp(t, p, a, hf_norms)
        if a.is_linear(i):
            la = p + "linear_attn."
            Z = a.lin_hv * a.lin_dv
            parts = [_linear(t, la + "in_proj_qkv", a.conv_dim, H), _linear(t, la + "in_proj_z", Z, H),
                     _linear(t, la + "in_proj_b", a.lin_hv, H), _linear(t, la + "in_proj_a", a.lin_hv, H)]
            conv = t.get(la + "conv1d.weight")
            if conv is None:
                raise KeyError(f"missing tensor {la}conv1d.weight")
            conv = _bf16_array(np.asarray(conv), la + "conv1d.weight")
            if conv.size != a.conv_dim * a.conv_k:
                raise ValueError(f"{la}conv1d.weight: {conv.shape}, expected {a.conv_dim} x {a.conv_k}")
            L.update(in_proj=_concat(parts, la + "in_proj"),
                     conv1d=np.ascontiguousarray(conv.reshape(a.conv_dim, a.conv_k)),
                     A_log=_vec(t, la + "A_log", a.lin_hv, dtype=np.float32),
                     dt_bias=_vec(t, la + "dt_bias", a.lin_hv),
                     norm=_vec(t, la + "norm.weight", a.lin_dv),  # gated norm: weight as stored
                     out_proj=_linear(t, la + "out_proj", H, Z))
        else:
            L.update(_attn(t, p, a, hf_norms))
        W[f"layers.{i}"] = L
    W["norm"] = _vec(t, "norm.weight", H, hf_norms)
    lm = t.get("lm_head.weight")
    if lm is None:
        raise KeyError("missing tensor lm_head.weight (tied embeddings are not supported)")
    if t.get("lm_head.scales") is not None:
        raise NotImplementedError("lm_head must be bf16: the two-stage head rescoring reads the bf16 rows")
    lm = _bf16_array(np.asarray(lm), "lm_head.weight")
    if lm.shape != (a.vocab, H):
        raise ValueError(f"lm_head.weight: {lm.shape}, expected {(a.vocab, H)}")
    W["lm_head"] = np.ascontiguousarray(lm)
    W["lm_head_q"] = Bf16Linear(W["lm_head"])  # coarse stage and draft head (lm_head2.py:17)
    return W


def load_mtp_tensors(tensors: dict) -> dict:
    """mtp.py:61-66: ``mtp.*`` tensors with the prefix removed and ``+ 1`` on every 1-D tensor
    (``.weight.scale`` is renamed ``.scales`` as for the trunk)."""
    out = {}
    for k, v in tensors.items():
        if not k.startswith("mtp."):
            continue
        v = np.asarray(v)
        if v.ndim == 1:
            v = _bf16_add_one(_bf16_array(v, k))
        out[k[len("mtp."):].replace(".weight.scale", ".scales")] = v
    if not out:
        raise KeyError("no mtp.* tensors")
    return out


def mtp_layout(t: dict, a: ModelArgs) -> dict:
    """The MTP head (mtp.py:48-57) in this engine's layout; ``t`` from ``load_mtp_tensors`` (norms
    already offset)."""
    H = a.hidden
    layer = _mlp(t, "layers.0.", a, False)
    layer.update(_attn(t, "layers.0.", a, False))
    return {"pre_fc_norm_embedding": _vec(t, "pre_fc_norm_embedding.weight", H),
            "pre_fc_norm_hidden": _vec(t, "pre_fc_norm_hidden.weight", H),
            "fc": _linear(t, "fc", H, 2 * H), "norm": _vec(t, "norm.weight", H), "layer": layer}


def to_device(Wn: dict, device="cuda") -> Weights:
    """Device weights: quantized triples and bf16 vectors are moved, bf16 linears are quantized on the
    GPU (libqmtp quantizer, the ``mx.quantize(w, 64, 4)`` format)."""
    import torch

    from .model import from_numpy
    from .qmv_kernel import QuantizedLinear

    device = torch.device(device)

    # memory-mapped tensors are read-only; torch wants writable host buffers
    host = lambda x: np.require(x, requirements=["C", "W"])

    def conv(v):
        if isinstance(v, dict):
            return {k: conv(x) for k, x in v.items()}
        if isinstance(v, Bf16Linear):
            w = torch.from_numpy(host(v.w).view(np.int16)).view(torch.bfloat16).to(device)
            q = QuantizedLinear.from_linear(w)
            del w
            return q
        if isinstance(v, tuple):
            v = tuple(host(x) for x in v)
        else:
            v = host(v)
        return from_numpy({"_": v}, device)["_"]

    return Weights({k: conv(v) for k, v in Wn.items()})


def load(files: Iterable, config: dict, mtp_files: Iterable = (), hf_norms: bool = False, max_pos: int = 1024,
         device="cuda"):
    """(ModelArgs, Weights) from trunk safetensors files (+ the MTP tensors, e.g. the file the
    reference's fetch_mtp.py writes).  Without MTP files the checkpoint itself must hold ``mtp.*``."""
    a = args_from_config(config, max_pos)
    raw = {}
    for f in files:
        raw.update(read_safetensors(f))
    mraw = dict(raw)
    for f in mtp_files:
        mraw.update(read_safetensors(f))
    Wn = trunk_layout(sanitize_names({k: v for k, v in raw.items() if not k.startswith("mtp.")}), a, hf_norms)
    Wn["mtp"] = mtp_layout(load_mtp_tensors(mraw), a)
    return a, to_device(Wn, device)


def checkpoint_dir(path):
    """(config dict, safetensors files) of a Hugging Face / MLX model directory: the shards named by
    model.safetensors.index.json (weight_map), else every *.safetensors file in the directory."""
    d = Path(path).expanduser()
    config = json.loads((d / "config.json").read_text())
    index = d / "model.safetensors.index.json"
    if index.exists():
        shards = sorted(set(json.loads(index.read_text())["weight_map"].values()))
        files = [d / f for f in shards]
        missing = [str(f) for f in files if not f.exists()]
        if missing:
            raise FileNotFoundError(f"shards named by the index are missing: {missing}")
    else:
        files = sorted(d.glob("*.safetensors"))
    if not files:
        raise FileNotFoundError(f"{d}: no safetensors files")
    return config, files


# ----------------------------------------------------------------------------------- Ollama
def ollama_checkpoint(tag: str = "9b-mlx", root="~/.ollama/models", model: str = "qwen3.5"):
    """qwen_ollama.py:22-28: (config dict, tensor blob paths, {json name: path}) of an Ollama model."""
    root = Path(root).expanduser()
    m = json.loads((root / "manifests/registry.ollama.ai/library" / model / tag).read_text())
    blob = lambda layer: root / "blobs" / layer["digest"].replace(":", "-")
    jsons = {layer["name"]: blob(layer) for layer in m["layers"] if layer["mediaType"].endswith("image.json")}
    tensors = [blob(layer) for layer in m["layers"] if layer["mediaType"].endswith("image.tensor")]
    if "config.json" not in jsons:
        raise KeyError(f"{model}:{tag}: manifest has no config.json layer")
    return json.loads(Path(jsons["config.json"]).read_text()), tensors, jsons
