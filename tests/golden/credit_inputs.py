"""Inputs of the credit-kernel fixtures (tests/golden/credit_kernels.pt), regenerated from a CPU generator seed.

Shaped like the Cut phase's (reference train/speedrun/run.py:1749-1802): RoPE'd + RMS-normed fp32 queries / keys
(unit RMS) whose bf16 copies feed the bf16 kernels, raw queries / keys, values, hubs and the bf16-rounded RoPE tables
[T, 32] as fp32."""
import torch


def credit_inputs(rows=2, t=256, seed=7):
    g = torch.Generator().manual_seed(seed)

    def unit():
        return torch.nn.functional.rms_norm(torch.randn(rows, t, 64, generator=g), (64,))

    qp, kp = unit(), unit()
    values = torch.randn(rows, t, 64, generator=g) * 0.5
    hub = torch.randn(rows, t, 64, generator=g) * 0.1
    q_raw = torch.randn(rows, t, 64, generator=g) * 0.7
    k_raw = torch.randn(rows, t, 64, generator=g) * 0.7
    inv = 1.0 / 10000 ** (torch.arange(0, 64, 2, dtype=torch.float32) / 64)
    freqs = torch.outer(torch.arange(t, dtype=torch.float32), inv)
    cos, sin = freqs.cos().bfloat16().float(), freqs.sin().bfloat16().float()
    return dict(qp=qp, kp=kp, values=values, hub=hub, q_raw=q_raw, k_raw=k_raw, cos=cos, sin=sin)
