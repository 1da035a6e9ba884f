"""Checkpoint loading (qmtp.loader) on the CPU: safetensors format, name sanitising, config mapping,
the projection concatenations, the MTP norm offset (mtp.py:61-66) and the Ollama manifest lookup."""
import json

import numpy as np
import pytest

from oracle import model as om
from oracle import ops
from tests import _ckpt


def _loader():
    from qmtp import loader

    return loader


def test_safetensors_round_trip(tmp_path):
    L = _loader()
    r = np.random.default_rng(0)
    t = {"a.bf16": ops.f32_to_bf16(r.standard_normal((3, 5)).astype(np.float32)),
         "b.f32": r.standard_normal((2, 3, 4)).astype(np.float32),
         "c.u32": r.integers(0, 2 ** 32, (7,), dtype=np.uint64).astype(np.uint32),
         "d.i64": np.arange(5, dtype=np.int64), "e.u8": np.arange(3, dtype=np.uint8),
         "f.empty": np.zeros((0, 4), np.float32)}
    L.write_safetensors(tmp_path / "x.safetensors", t, bf16=["a.bf16"])
    back = L.read_safetensors(tmp_path / "x.safetensors")
    assert set(back) == set(t)
    for k, v in t.items():
        assert back[k].dtype == v.dtype and back[k].shape == v.shape and np.array_equal(back[k], v), k
    raw = (tmp_path / "x.safetensors").read_bytes()
    n = int.from_bytes(raw[:8], "little")
    assert json.loads(raw[8:8 + n])["a.bf16"]["dtype"] == "BF16"


def test_safetensors_rejects_bad_files(tmp_path):
    L = _loader()
    (tmp_path / "short").write_bytes(b"\x01\x02")
    with pytest.raises(ValueError):
        L.read_safetensors(tmp_path / "short")
    (tmp_path / "long").write_bytes((10 ** 6).to_bytes(8, "little") + b"{}")
    with pytest.raises(ValueError):
        L.read_safetensors(tmp_path / "long")
    hdr = json.dumps({"t": {"dtype": "F32", "shape": [4], "data_offsets": [0, 12]}}).encode()
    (tmp_path / "bad").write_bytes(len(hdr).to_bytes(8, "little") + hdr + bytes(16))
    with pytest.raises(ValueError):
        L.read_safetensors(tmp_path / "bad")


def test_sanitize_names():
    L = _loader()
    t = {"language_model.model.layers.0.mlp.gate_proj.weight": 1, "language_model.lm_head.weight": 2,
         "model.language_model.embed_tokens.weight.scale": 3, "vision_tower.blocks.0.w": 4,
         "model.visual.patch.weight": 5, "model.norm.weight": 6}
    assert L.sanitize_names(t) == {"layers.0.mlp.gate_proj.weight": 1, "lm_head.weight": 2,
                                   "embed_tokens.scales": 3, "norm.weight": 6}
    with pytest.raises(ValueError):
        L.sanitize_names({"model.norm.weight": 1, "language_model.norm.weight": 2})


def test_args_from_config():
    L = _loader()
    from qmtp import model as qm

    a = L.args_from_config(_ckpt.config_dict(om.SMALL), max_pos=1024)
    assert a == qm.SMALL
    c = _ckpt.config_dict(om.CONFIG4)
    assert L.args_from_config(c, max_pos=1024) == qm.CONFIG4
    c["text_config"]["layer_types"][0] = "full_attention"
    with pytest.raises(NotImplementedError):
        L.args_from_config(c)


def test_bf16_add_one_matches_rounding():
    L = _loader()
    x = np.arange(0, 65536, 7, dtype=np.uint32).astype(np.uint16)
    x = x[(x & 0x7F80) != 0x7F80]  # finite values only
    f = ops.bf16_to_f32(x).astype(np.float64) + 1.0
    want = ops.f32_to_bf16(f.astype(np.float32))  # the fp32 sum is exact for bf16 inputs of this range
    assert np.array_equal(L._bf16_add_one(x), want)


@pytest.fixture(scope="module")
def small_weights():
    return om.synthetic_weights(om.SMALL, seed=3)


def _eq(got, want, path="W"):
    if isinstance(want, dict):
        assert set(got) == set(want), path
        for k in want:
            _eq(got[k], want[k], f"{path}.{k}")
    elif isinstance(want, tuple):
        assert isinstance(got, tuple) and len(got) == len(want), path
        for g, w in zip(got, want):
            assert g.dtype == w.dtype and np.array_equal(g, w), path
    else:
        assert np.array_equal(np.asarray(got), want), path


@pytest.mark.parametrize("hf_norms", [True, False])
def test_layout_reassembles_the_oracle_weights(tmp_path, small_weights, hf_norms):
    L = _loader()
    a = om.SMALL
    T, M, bf = _ckpt.checkpoint(small_weights, a, hf_norms=hf_norms)
    L.write_safetensors(tmp_path / "trunk.safetensors", T, bf16=[k for k in T if k in bf])
    L.write_safetensors(tmp_path / "mtp.safetensors", M, bf16=[k for k in M if k in bf])
    raw = L.read_safetensors(tmp_path / "trunk.safetensors")
    args = L.args_from_config(_ckpt.config_dict(a))
    W = L.trunk_layout(L.sanitize_names(raw), args, hf_norms=hf_norms)
    W["mtp"] = L.mtp_layout(L.load_mtp_tensors(L.read_safetensors(tmp_path / "mtp.safetensors")), args)
    assert isinstance(W["lm_head_q"], L.Bf16Linear)
    assert np.array_equal(W["lm_head_q"].w, small_weights["lm_head"])
    want = dict(small_weights)
    del want["lm_head_q"]
    del W["lm_head_q"]
    _eq(W, want)


def test_bf16_linears_are_marked_for_quantization(small_weights):
    L = _loader()
    a = om.SMALL
    T, M, _ = _ckpt.checkpoint(small_weights, a)
    wq, s, b = small_weights["mtp"]["fc"]
    dense = ops.f32_to_bf16(np.zeros((a.hidden, 2 * a.hidden), np.float32))
    for k in ("mtp.fc.scales", "mtp.fc.biases"):
        del M[k]
    M["mtp.fc.weight"] = dense
    m = L.mtp_layout(L.load_mtp_tensors(M), L.args_from_config(_ckpt.config_dict(a)))
    assert isinstance(m["fc"], L.Bf16Linear) and np.array_equal(m["fc"].w, dense)


def test_rejects_other_quantized_formats(small_weights):
    L = _loader()
    a = om.SMALL
    T, _, _ = _ckpt.checkpoint(small_weights, a)
    T = L.sanitize_names(T)
    n = "layers.0.mlp.down_proj"
    T[n + ".scales"] = np.zeros((a.hidden, a.intermediate // 32), np.uint8)  # MXFP4-shaped scales: not served
    del T[n + ".biases"]
    with pytest.raises(NotImplementedError):
        L.trunk_layout(T, L.args_from_config(_ckpt.config_dict(a)))


def test_nvfp4_checkpoint_layout(tmp_path, small_weights):
    """An NVFP4 checkpoint (Ollama scale names) reassembles into (nibbles, scales) pairs."""
    L = _loader()
    a = om.SMALL
    Wq = _ckpt.to_nvfp4(small_weights)
    T, M, bf = _ckpt.checkpoint(Wq, a, scale_suffix=".weight.scale")
    assert any(k.endswith(".weight.scale") for k in T)
    L.write_safetensors(tmp_path / "t.safetensors", T, bf16=[k for k in T if k in bf])
    args = L.args_from_config(_ckpt.config_dict(a))
    W = L.trunk_layout(L.sanitize_names(L.read_safetensors(tmp_path / "t.safetensors")), args, hf_norms=True)
    W["mtp"] = L.mtp_layout(L.load_mtp_tensors(M), args)
    del W["lm_head_q"]
    want = dict(Wq)
    del want["lm_head_q"]
    _eq(W, want)


def test_ollama_manifest(tmp_path):
    L = _loader()
    root = tmp_path / "models"
    (root / "blobs").mkdir(parents=True)
    man = root / "manifests/registry.ollama.ai/library/qwen3.5"
    man.mkdir(parents=True)
    cfg = _ckpt.config_dict(om.SMALL)
    layers = []
    for i, (name, media, data) in enumerate([("config.json", "application/vnd.ollama.image.json", json.dumps(cfg)),
                                             ("tok.json", "application/vnd.ollama.image.json", "{}"),
                                             (None, "application/vnd.ollama.image.tensor", "x"),
                                             (None, "application/vnd.ollama.image.tensor", "y")]):
        digest = f"sha256:{i:064x}"
        (root / "blobs" / digest.replace(":", "-")).write_text(data)
        layers.append({"mediaType": media, "digest": digest, **({"name": name} if name else {})})
    (man / "9b-mlx").write_text(json.dumps({"layers": layers}))
    c, tensors, jsons = L.ollama_checkpoint("9b-mlx", root)
    assert c == cfg and len(tensors) == 2 and set(jsons) == {"config.json", "tok.json"}
    assert all(p.read_text() in ("x", "y") for p in tensors)


def test_oracle_nvfp4_embedding():
    """qo_embed_nvfp4 = bf16(e2m1(q) * e4m3(s)) with the reference's decoders (qmv_kernel.py:16-29)."""
    r = np.random.default_rng(9)
    V, D = 50, 128
    wq = r.integers(0, 2 ** 32, (V, D // 8), dtype=np.uint64).astype(np.uint32)
    sc = r.integers(0, 256, (V, D // 16), dtype=np.int64).astype(np.uint8)
    tok = np.int32([3, 0, 49, 3])
    e2m1, e4m3, _ = ops.decode_tables()
    q = ((wq[:, :, None] >> (4 * np.arange(8, dtype=np.uint32))) & 15).reshape(V, D)
    want = ops.f32_to_bf16((e2m1[q] * np.repeat(e4m3[sc], 16, axis=1)).astype(np.float32))[tok]
    assert np.array_equal(om.embed(tok, wq, sc, D), want)


def test_loader_error_paths(small_weights):
    """Missing or unusable tensors fail with a clear error instead of loading something else."""
    L = _loader()
    a = om.SMALL
    args = L.args_from_config(_ckpt.config_dict(a))
    T, _, _ = _ckpt.checkpoint(small_weights, a)
    T = L.sanitize_names(T)
    for mutate, exc in [(lambda t: t.pop("lm_head.weight"), KeyError),                  # tied embeddings
                        (lambda t: t.update({"lm_head.scales": np.zeros(1, np.uint16)}), NotImplementedError),
                        (lambda t: t.pop("layers.0.linear_attn.A_log"), KeyError),
                        (lambda t: t.update({"layers.0.linear_attn.conv1d.weight": np.zeros((3, 4), np.uint16)}),
                         ValueError),
                        (lambda t: t.update({"layers.3.self_attn.k_proj.weight":
                                             np.zeros((7, a.hidden // 8), np.uint32)}), ValueError)]:
        t = dict(T)
        mutate(t)
        with pytest.raises(exc):
            L.trunk_layout(t, args)


def test_config_variants():
    """Top-level config (no text_config), rope_scaling instead of rope_parameters, no layer_types."""
    L = _loader()
    from qmtp import model as qm

    c = dict(_ckpt.config_dict(om.SMALL)["text_config"])
    rope = c.pop("rope_parameters")
    c.pop("layer_types")
    c["rope_scaling"] = rope
    assert L.args_from_config(c, max_pos=1024) == qm.SMALL
    c.pop("rope_scaling")
    c["rope_theta"], c["partial_rotary_factor"] = om.SMALL.rope_theta, 0.25
    assert L.args_from_config(c, max_pos=1024) == qm.SMALL


def test_checkpoint_dir(tmp_path):
    L = _loader()
    cfg = _ckpt.config_dict(om.SMALL)
    (tmp_path / "config.json").write_text(json.dumps(cfg))
    for n in ("b.safetensors", "a.safetensors"):
        L.write_safetensors(tmp_path / n, {"x": np.zeros(2, np.float32)})
    c, files = L.checkpoint_dir(tmp_path)
    assert c == cfg and [f.name for f in files] == ["a.safetensors", "b.safetensors"]
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps({"weight_map": {"x": "b.safetensors"}}))
    assert [f.name for f in L.checkpoint_dir(tmp_path)[1]] == ["b.safetensors"]
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps({"weight_map": {"x": "c.safetensors"}}))
    with pytest.raises(FileNotFoundError):
        L.checkpoint_dir(tmp_path)
