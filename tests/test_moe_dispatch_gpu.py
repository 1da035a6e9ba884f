"""qmtp_moe_dispatch (fixed-capacity expert-parallel dispatch) against its plain-torch restatement,
exactly (GPU, one device): slot layout, expert ids, position table, counts and copied rows, for 1-8
ranks, with and without capacity overflow."""
import pytest
import torch

from tests._moe_dispatch_ref import ref_dispatch

pytestmark = pytest.mark.gpu

E_R, N_SH, H, T, TOPK = 64, 2, 256, 96, 6


def _bufs(world, cap, n, dev):
    return dict(send_x=torch.zeros((world * cap, H), dtype=torch.bfloat16, device=dev),
                send_e=torch.zeros((world * cap,), dtype=torch.int32, device=dev),
                sh_x=torch.zeros((n, H), dtype=torch.bfloat16, device=dev),
                sh_e=torch.zeros((n,), dtype=torch.int32, device=dev),
                pos=torch.zeros((n,), dtype=torch.int32, device=dev),
                counts=torch.zeros((world + 1,), dtype=torch.int32, device=dev))


@pytest.mark.parametrize("world,cap_kind", [(1, "full"), (2, "full"), (4, "full"), (8, "full"), (2, "tight"),
                                            (8, "overflow")])
def test_dispatch_matches_restatement(world, cap_kind, dev):
    from qmtp import _lib, moe

    g = torch.Generator(device=dev)
    g.manual_seed(world)
    x = torch.randn((T, H), generator=g, device=dev).to(torch.bfloat16)
    idx, _ = moe.route(torch.randn((T, E_R), generator=g, device=dev), TOPK, N_SH)
    S = idx.shape[1]
    per_rank = torch.bincount((idx[idx < E_R] // (E_R // world)).reshape(-1).long(), minlength=world)
    cap = {"full": T * S, "tight": int(per_rank.max()), "overflow": max(1, int(per_rank.max()) - 5)}[cap_kind]
    got = _bufs(world, cap, T * S, dev)
    _lib.device_error()  # clear
    moe.dispatch(idx, x, E_R, N_SH, world, cap, **got)
    torch.cuda.synchronize()
    err = _lib.device_error()
    want = _bufs(world, cap, T * S, torch.device("cpu"))
    ref_dispatch(idx.cpu(), x.cpu(), E_R, N_SH, world, cap, **want)
    for k in ("send_e", "sh_e", "pos", "counts"):
        assert torch.equal(got[k].cpu(), want[k]), k
    ok = want["send_e"] >= 0
    assert torch.equal(got["send_x"].cpu()[ok].view(torch.int16), want["send_x"][ok].view(torch.int16))
    ok = want["sh_e"] >= 0
    assert torch.equal(got["sh_x"].cpu()[ok].view(torch.int16), want["sh_x"][ok].view(torch.int16))
    assert (err != 0) == (cap_kind == "overflow")
