"""CPU restatement of the identity phase's batched GEMMs (reference train/speedrun/id_kernels.py) — test
infrastructure only: the checker of noise_b200.id_kernels, never called by the product path.

Products accumulate in fp64 and are rounded to bf16 once, where the reference's Triton kernels accumulate in fp32 (so
single outputs may differ from both by one bf16 ulp); the slope epilogue is fp32 as there."""
import torch


def _bf(x):
    return x.to(torch.bfloat16)


def hidden_credits(us, steps, credb, w_out_t):
    """out[l] = bf16(slope(U_l, step_l) * float(bf16(credb[l] @ w_out_t[l]))), slope = (max(u + s, 0)^2 -
    max(u - s, 0)^2) / (2 s) (id_kernels.py:40-57)."""
    layers, m, _ = credb.shape
    n = w_out_t.shape[-1]
    read = _bf((credb.double() @ w_out_t.double()).float()).float()
    u = torch.stack([x.reshape(m, n) for x in us]).float()
    step = steps.float()[:, :, None]
    up = torch.clamp(u + step, min=0.0)
    down = torch.clamp(u - step, min=0.0)
    slope = (up * up - down * down) / (2 * step)
    return _bf(slope * read)


def at_b_layers(As, Bs):
    """out[l] = bf16(As[l]^T @ Bs[l]), each flattened to (K, .) rows (id_kernels.py:141-170)."""
    outs = []
    for a, b in zip(As, Bs):
        a2, b2 = a.reshape(-1, a.shape[-1]).double(), b.reshape(-1, b.shape[-1]).double()
        outs.append(_bf((a2.T @ b2).float()))
    return torch.stack(outs)


def square_credit_grads(n1s, got2):
    """out[j L + l] = bf16(n1s[l]^T @ B_jl), B_jl[tok, w HD + d] = got2[w, l, j, tok, d] (id_kernels.py:90-133)."""
    world, layers, three, m, hd = got2.shape
    outs = []
    for j in range(three):
        for l in range(layers):
            b = got2[:, l, j].permute(1, 0, 2).reshape(m, world * hd).double()
            outs.append(_bf((n1s[l].double().T @ b).float()))
    return torch.stack(outs)
