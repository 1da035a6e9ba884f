"""A checkpoint written from the oracle's weights, loaded by qmtp.loader (bf16 MTP projection
quantized on the GPU), decodes the same greedy MTP stream as the oracle (GPU)."""
import numpy as np
import pytest

from oracle import model as om
from oracle import ops
from tests import _ckpt
from tests.test_model_oracle import prompt

pytestmark = pytest.mark.gpu


_dequant = _ckpt.dequant


def test_loaded_checkpoint_decodes_like_the_oracle(tmp_path, dev):
    from qmtp import loader
    from qmtp.mtp import MTPDecoder, decode_mtp

    a = om.SMALL
    Wn = om.synthetic_weights(a, seed=3)
    T, M, bf = _ckpt.checkpoint(Wn, a, hf_norms=True)
    dense = _dequant(Wn["mtp"]["fc"])  # the MTP fc as a bf16 tensor, quantized again at load time
    for k in ("mtp.fc.scales", "mtp.fc.biases"):
        del M[k]
    M["mtp.fc.weight"] = dense
    bf.add("mtp.fc.weight")
    loader.write_safetensors(tmp_path / "trunk.safetensors", T, bf16=[k for k in T if k in bf])
    loader.write_safetensors(tmp_path / "mtp.safetensors", M, bf16=[k for k in M if k in bf])
    args, W = loader.load([tmp_path / "trunk.safetensors"], _ckpt.config_dict(a), [tmp_path / "mtp.safetensors"],
                          hf_norms=True, max_pos=1024, device=dev)
    want = dict(Wn)
    want["mtp"] = dict(Wn["mtp"], fc=ops.quantize_affine(dense))
    p = prompt(40, seed=7)
    ref, _ = om.OracleModel(a, want).generate_mtp(p, 30)
    out, st = decode_mtp(MTPDecoder(args, W, k=2, max_tokens=300), p, 30)
    assert out == ref


def test_nvfp4_checkpoint_decodes_like_the_oracle(tmp_path, dev):
    """Every linear (and the embedding) in NVFP4, written with Ollama's scale names, loaded and decoded."""
    from qmtp import loader
    from qmtp.mtp import MTPDecoder, decode_mtp

    a = om.SMALL
    Wq = _ckpt.to_nvfp4(om.synthetic_weights(a, seed=3))
    T, M, bf = _ckpt.checkpoint(Wq, a, hf_norms=True, scale_suffix=".weight.scale")
    loader.write_safetensors(tmp_path / "trunk.safetensors", T, bf16=[k for k in T if k in bf])
    loader.write_safetensors(tmp_path / "mtp.safetensors", M, bf16=[k for k in M if k in bf])
    args, W = loader.load([tmp_path / "trunk.safetensors"], _ckpt.config_dict(a), [tmp_path / "mtp.safetensors"],
                          hf_norms=True, max_pos=1024, device=dev)
    assert W["embed"].mode == "nvfp4" and W["layers.0"]["in_proj"].mode == "nvfp4"
    p = prompt(40, seed=8)
    ref, _ = om.OracleModel(a, Wq).generate_mtp(p, 16)
    out, _ = decode_mtp(MTPDecoder(args, W, k=2, max_tokens=300), p, 16)
    assert out == ref


def test_nvfp4_embed_and_residual_gemv(dev):
    """qmtp_embed_nvfp4 and qmtp_qmv_nvfp4_g16_res against the oracle, bit-exact."""
    import torch

    from oracle import model as omod
    from qmtp import _lib
    from tests._util import randn_bf16, to_np, to_torch

    r = np.random.default_rng(4)
    V, D = 700, 2048
    wq = r.integers(0, 2 ** 32, (V, D // 8), dtype=np.uint64).astype(np.uint32)
    sc = r.integers(0, 256, (V, D // 16), dtype=np.int64).astype(np.uint8)
    tok = np.int32([0, 699, 5, 5, 123])
    out = torch.empty((5, D), dtype=torch.bfloat16, device=dev)
    tk, wt, st = torch.from_numpy(tok).to(dev), to_torch(wq, dev), to_torch(sc, dev)  # kept alive over the call
    _lib.check(_lib.lib().qmtp_embed_nvfp4(tk.data_ptr(), 5, wt.data_ptr(), st.data_ptr(), V, D, out.data_ptr(), D,
                                           _lib.stream()), "embed_nvfp4")
    torch.cuda.synchronize()
    assert np.array_equal(to_np(out), omod.embed(tok, wq, sc, D))
    N, K, Mr = 300, 4096, 3
    nq = r.integers(0, 2 ** 32, (N, K // 8), dtype=np.uint64).astype(np.uint32)
    ns = r.integers(54, 70, (N, K // 16), dtype=np.int64).astype(np.uint8)
    x, res = randn_bf16((Mr, K), 1), randn_bf16((Mr, N), 2)
    y = to_torch(res, dev).clone()
    xt, qt, nt = to_torch(x, dev), to_torch(nq, dev), to_torch(ns, dev)
    _lib.check(_lib.lib().qmtp_qmv_nvfp4_g16_res(xt.data_ptr(), qt.data_ptr(), nt.data_ptr(), y.data_ptr(),
                                                 y.data_ptr(), Mr, N, K, N, _lib.stream()), "qmv_nvfp4_res")
    torch.cuda.synchronize()
    assert np.array_equal(to_np(y), omod.add(res, ops.qmv_nvfp4(x, nq, ns)))
