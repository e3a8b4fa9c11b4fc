"""Seeded synthetic inputs with the benchmark's value distribution.

The reference evaluates this path on no public dataset; its workloads are DiT
activations.  These inputs stand in for them: Q/K/V ~ N(0, 1) in fp32, then for each
head 4 outlier channels (drawn with ``randperm(D)[:4]`` from the same generator,
independently per tensor and per head) scaled by 8, cast to bf16.  Text: one valid
token per chunk unless a test asks for more.
"""
from __future__ import annotations

import torch

OUTLIER_CHANNELS = 4
OUTLIER_SCALE = 8.0


def seeded_kv(shape, generator: torch.Generator, device="cpu", dtype=torch.bfloat16) -> torch.Tensor:
    """[B, L, H, D] tensor: N(0, 1) with 4 outlier channels per head scaled x8."""
    B, L, H, D = shape
    gen_dev = generator.device if hasattr(generator, "device") else torch.device("cpu")
    x = torch.randn((B, L, H, D), generator=generator, device=gen_dev, dtype=torch.float32)
    scale = torch.ones((H, D), dtype=torch.float32, device=gen_dev)
    for h in range(H):
        idx = torch.randperm(D, generator=generator, device=gen_dev)[:OUTLIER_CHANNELS]
        scale[h, idx] = OUTLIER_SCALE
    x.mul_(scale)
    return x.to(dtype=dtype, device=device)


def make_generator(seed: int, device="cpu") -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def config_seed(config_index: int) -> int:
    """Seed of BASELINE config ``config_index`` (1-based)."""
    return 1234 + config_index
