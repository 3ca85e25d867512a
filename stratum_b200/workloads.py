"""Seeded synthetic inputs with the shapes and distributions of the benchmark configs.

The reference's benchmark configs use random init and
uniform token ids, so everything here is generated, never loaded.
"""

from __future__ import annotations

import torch

# Config 2: NF4 codec bandwidth sweep.
CODEC_SHAPES = ((2048, 2048), (4096, 4096), (14336, 4096), (4096, 14336))
OUTLIER_FRACTION = 1e-3
OUTLIER_SCALE = 20.0

# Config 1: a single NF4Linear (weight [out, in]).
LINEAR1_WEIGHT = (5632, 2048)
LINEAR1_X = (2, 512, 2048)
LINEAR1_RANK = 16
LINEAR1_ALPHA = 32


def codec_weight(shape, seed: int = 0, device="cuda", dtype=torch.float16) -> torch.Tensor:
    """fp16 ~N(0, 0.02) with 0.1% of entries (fixed random positions) scaled x20."""
    g = torch.Generator(device=device).manual_seed(seed)
    w = torch.randn(shape, generator=g, device=device, dtype=torch.float32) * 0.02
    n = w.numel()
    k = max(1, int(n * OUTLIER_FRACTION))
    idx = torch.randint(0, n, (k,), generator=g, device=device)
    w.view(-1)[idx] *= OUTLIER_SCALE
    return w.to(dtype)


def linear_inputs(weight_shape=LINEAR1_WEIGHT, x_shape=LINEAR1_X, rank=LINEAR1_RANK, seed: int = 0,
                  device="cuda", weight_dtype=torch.float16, act_dtype=torch.bfloat16):
    """Config-1 style NF4Linear inputs: W ~N(0,0.02), LoRA A kaiming-uniform(a=sqrt 5), B ~N(0,0.01),
    x ~N(0,1), dY ~N(0,1)."""
    import math

    g = torch.Generator(device=device).manual_seed(seed)
    out_f, in_f = weight_shape
    w = (torch.randn(weight_shape, generator=g, device=device) * 0.02).to(weight_dtype)
    bound = 1.0 / math.sqrt(in_f)  # kaiming_uniform(a=sqrt(5)) on [rank, in] -> U(-1/sqrt(in), 1/sqrt(in))
    lora_a = ((torch.rand((rank, in_f), generator=g, device=device) * 2 - 1) * bound).to(act_dtype)
    lora_b = (torch.randn((out_f, rank), generator=g, device=device) * 0.01).to(act_dtype)
    x = torch.randn(x_shape, generator=g, device=device).to(act_dtype)
    dy = torch.randn((*x_shape[:-1], out_f), generator=g, device=device).to(act_dtype)
    return w, lora_a, lora_b, x, dy
