"""Test helper: the oracle's numpy weights written back as a Qwen3.5 checkpoint (Hugging Face / MLX
module names, split projections), the input of qmtp.loader."""
import numpy as np

from oracle import ops


def config_dict(a):
    """config.json of a Qwen3.5-shaped model with the oracle's ModelArgs (nested text_config)."""
    types = ["linear_attention" if a.is_linear(i) else "full_attention" for i in range(a.layers)]
    return {"model_type": "qwen3_5", "text_config": {
        "hidden_size": a.hidden, "num_hidden_layers": a.layers, "intermediate_size": a.intermediate,
        "num_attention_heads": a.n_heads, "num_key_value_heads": a.n_kv, "head_dim": a.head_dim,
        "vocab_size": a.vocab, "linear_num_key_heads": a.lin_hk, "linear_num_value_heads": a.lin_hv,
        "linear_key_head_dim": a.lin_dk, "linear_value_head_dim": a.lin_dv, "linear_conv_kernel_dim": a.conv_k,
        "rms_norm_eps": a.eps, "full_attention_interval": 4, "layer_types": types,
        "rope_parameters": {"rope_theta": a.rope_theta, "partial_rotary_factor": a.rotary_dim / a.head_dim}}}


def minus_one(w):
    """bf16 bits of w - 1 for the oracle's unit norm weights (exact: 1 - 1 = 0)."""
    f = ops.bf16_to_f32(w) - np.float32(1.0)
    return ops.f32_to_bf16(f.astype(np.float32))


def checkpoint(Wn, a, hf_norms=True, prefix="model.language_model.", scale_suffix=".scales"):
    """(trunk tensors, mtp tensors, names of bf16 tensors).  Quantized linears keep their triples
    (``.weight`` uint32, ``.scales`` / ``.biases`` bf16); the MTP tensors carry raw-HF norms (w - 1)."""
    T, M, bf = {}, {}, set()

    def put(d, name, v, is_bf16):
        d[name] = np.ascontiguousarray(v)
        if is_bf16:
            bf.add(name)

    def lin(d, name, trip, r0=None, r1=None):
        sl = slice(r0, r1)
        if len(trip) == 2:  # NVFP4 (Ollama blobs name the scales ".weight.scale")
            put(d, name + ".weight", trip[0][sl], False)
            put(d, name + (".weight.scale" if scale_suffix != ".scales" else ".scales"), trip[1][sl], False)
            return
        w, s, b = trip
        put(d, name + ".weight", w[sl], False)
        put(d, name + ".scales", s[sl], True)
        put(d, name + ".biases", b[sl], True)

    def norm(d, name, w, raw):
        put(d, name, minus_one(w) if raw else w, True)

    def block(d, p, L, raw):
        norm(d, p + "input_layernorm.weight", L["input_ln"], raw)
        norm(d, p + "post_attention_layernorm.weight", L["post_ln"], raw)
        I = a.intermediate
        lin(d, p + "mlp.gate_proj", L["gate_up"], 0, I)
        lin(d, p + "mlp.up_proj", L["gate_up"], I, 2 * I)
        lin(d, p + "mlp.down_proj", L["down"])
        if "qkv_proj" in L:
            q = 2 * a.n_heads * a.head_dim
            kv = a.n_kv * a.head_dim
            lin(d, p + "self_attn.q_proj", L["qkv_proj"], 0, q)
            lin(d, p + "self_attn.k_proj", L["qkv_proj"], q, q + kv)
            lin(d, p + "self_attn.v_proj", L["qkv_proj"], q + kv, q + 2 * kv)
            norm(d, p + "self_attn.q_norm.weight", L["q_norm"], raw)
            norm(d, p + "self_attn.k_norm.weight", L["k_norm"], raw)
            lin(d, p + "self_attn.o_proj", L["o_proj"])

    lin(T, prefix + "embed_tokens", Wn["embed"])
    for i in range(a.layers):
        L = Wn[f"layers.{i}"]
        p = f"{prefix}layers.{i}."
        block(T, p, L, hf_norms)
        if a.is_linear(i):
            la = p + "linear_attn."
            c, z = a.conv_dim, a.lin_hv * a.lin_dv
            lin(T, la + "in_proj_qkv", L["in_proj"], 0, c)
            lin(T, la + "in_proj_z", L["in_proj"], c, c + z)
            lin(T, la + "in_proj_b", L["in_proj"], c + z, c + z + a.lin_hv)
            lin(T, la + "in_proj_a", L["in_proj"], c + z + a.lin_hv, c + z + 2 * a.lin_hv)
            put(T, la + "conv1d.weight", L["conv1d"].reshape(c, 1, a.conv_k), True)  # PyTorch Conv1d layout
            put(T, la + "A_log", L["A_log"], False)
            put(T, la + "dt_bias", L["dt_bias"], True)
            put(T, la + "norm.weight", L["norm"], True)
            lin(T, la + "out_proj", L["out_proj"])
    norm(T, prefix + "norm.weight", Wn["norm"], hf_norms)
    put(T, "lm_head.weight", Wn["lm_head"], True)
    put(T, "model.visual.blocks.0.weight", np.zeros(4, np.uint16), True)  # skipped by the loader
    m = Wn["mtp"]
    for n in ("pre_fc_norm_embedding", "pre_fc_norm_hidden", "norm"):
        norm(M, f"mtp.{n}.weight", m[n], True)
    lin(M, "mtp.fc", m["fc"])
    block(M, "mtp.layers.0.", m["layer"], True)
    return T, M, bf


def dequant(trip):
    """bf16 bits of s * q + b for an affine-g64 triple (the dense weight a bf16 checkpoint holds)."""
    wq, s, b = trip
    n, k8 = wq.shape
    q = ((wq[:, :, None] >> (4 * np.arange(8, dtype=np.uint32))) & 15).reshape(n, 8 * k8).astype(np.float32)
    sf = np.repeat(ops.bf16_to_f32(s), 64, axis=1)
    bf = np.repeat(ops.bf16_to_f32(b), 64, axis=1)
    return ops.f32_to_bf16((sf * q + bf).astype(np.float32))


def to_nvfp4(Wn):
    """The oracle weights with every linear except the lm_head copies re-quantized to NVFP4 g16."""
    def conv(k, v):
        if isinstance(v, dict):
            return {kk: conv(kk, x) for kk, x in v.items()}
        if isinstance(v, tuple) and k != "lm_head_q":
            return ops.quantize_fp4(dequant(v), "nvfp4")
        return v
    return {k: conv(k, v) for k, v in Wn.items()}
