"""Plain-torch restatement of qmtp_moe_dispatch (test infrastructure): the fixed-capacity layout of an
expert-parallel MoE layer, used as the expected output of the CUDA kernel and as the dispatch of the
gloo (CPU) expert-parallel test."""
import torch


def ref_dispatch(idx, x, n_routed, n_shared, world, cap, send_x, send_e, sh_x, sh_e, pos, counts):
    T, S = idx.shape
    per = n_routed // world
    flat = idx.reshape(-1).tolist()
    send_e.fill_(-1)
    sh_e.fill_(-1)
    pos.fill_(-1)
    fill = [0] * (world + 1)
    for i, e in enumerate(flat):  # (t, j) order
        t = i // S
        if e < 0 or e >= n_routed + n_shared:
            continue
        if e < n_routed:
            d = e // per
            p = fill[d]
            fill[d] += 1
            if p >= cap:
                continue
            send_e[d * cap + p] = e - d * per
            send_x[d * cap + p] = x[t]
            pos[i] = d * cap + p
        else:
            q = fill[world]
            fill[world] += 1
            sh_e[q] = per + e - n_routed
            sh_x[q] = x[t]
            pos[i] = 2 * world * cap + q
    counts.copy_(torch.tensor(fill, dtype=counts.dtype))
