"""A checkpoint written from the oracle's weights, loaded by qmtp.loader (bf16 MTP projection
quantized on the GPU), decodes the same greedy MTP stream as the oracle (GPU)."""
import numpy as np
import pytest

from oracle import model as om
from oracle import ops
from tests import _ckpt
from tests.test_model_oracle import prompt

pytestmark = pytest.mark.gpu


def _dequant(trip):
    """bf16 bits of s * q + b for an affine-g64 triple (the dense weight a bf16 checkpoint holds)."""
    wq, s, b = trip
    n, k8 = wq.shape
    q = ((wq[:, :, None] >> (4 * np.arange(8, dtype=np.uint32))) & 15).reshape(n, 8 * k8).astype(np.float32)
    sf = np.repeat(ops.bf16_to_f32(s), 64, axis=1)
    bf = np.repeat(ops.bf16_to_f32(b), 64, axis=1)
    return ops.f32_to_bf16((sf * q + bf).astype(np.float32))


def test_loaded_checkpoint_decodes_like_the_oracle(tmp_path, dev):
    from qmtp import loader
    from qmtp.mtp import MTPDecoder, generate_mtp

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
    out, st = generate_mtp(MTPDecoder(args, W, k=2, max_tokens=300), p, 30)
    assert out == ref
