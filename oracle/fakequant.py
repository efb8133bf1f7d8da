"""TEST INFRASTRUCTURE ONLY: the reference's CPU path for one linear layer, restated.

rtx527896828/webyIQ tools/reference.py runs the model in fp32 torch on the CPU with
  - every linear weight replaced by its int4 dequantization (reference.py:35-40),
    done once, outside the forward pass;
  - every linear input fake-quantized to int8 (reference.py:42-52): per group of 32
    dx = amax/127, q = round(x/dx) (0 where dx = 0), x <- q*dx;
  - then F.linear in fp32.
`fake_quant_linear` is that per-layer computation; `fq_token` is the per-token
(per-row absmax) variant used by the BASELINE configs.  bench.py times this on the
host cores as the CPU baseline.
"""

import torch


def fq_group32(x):
    """reference.py:43-48 restated: int8 fake-quant per group of 32 along the last dim."""
    g = x.reshape(*x.shape[:-1], -1, 32)
    dx = g.abs().amax(-1, keepdim=True) / 127.0
    q = torch.where(dx > 0, torch.round(g / torch.where(dx > 0, dx, 1.0)), 0.0)
    return (q * dx).reshape(x.shape)


def fq_token(x):
    """Per-token variant: one dx per row."""
    dx = x.abs().amax(-1, keepdim=True) / 127.0
    q = torch.where(dx > 0, torch.round(x / torch.where(dx > 0, dx, 1.0)), 0.0)
    return q * dx


def fake_quant_linear(x, w_deq, per_token=False):
    """y = F.linear(fq(x), W_deq) in fp32 (reference.py:35-52, 63-64)."""
    xf = fq_token(x) if per_token else fq_group32(x)
    return torch.nn.functional.linear(xf, w_deq)
