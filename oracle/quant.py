"""Quantise / decode restatements (CPU, torch fp32) — test infrastructure only.

INT8 follows the CPU branch of ``quantize_kv_into``
(hymm/models/dit/modules/int8_kv_cache.py:149-158) line for line; E4M3 is the same
rule with a 448 denominator and an RNE cast to float8_e4m3fn after clamping to
+-448 (the extension this build adds; the reference has no FP8 KV format).  Decode
follows ``dequantize_kv``'s CPU branch (:202-204).
"""
from __future__ import annotations

import torch


def quantize_int8(values: torch.Tensor):
    """bf16 [B, L, H, D] -> (int8 codes, fp32 scale [B, L, H, 1]); int8_kv_cache.py:150-157."""
    src = values.float()
    peak = src.abs().amax(dim=-1, keepdim=True)
    s = torch.where(peak > 0, peak / 127.0, torch.ones_like(peak))
    scaled = src / s
    rounded = torch.where(scaled >= 0, torch.floor(scaled + 0.5), torch.ceil(scaled - 0.5))
    return rounded.clamp(-127, 127).to(torch.int8), s


def quantize_e4m3(values: torch.Tensor):
    """bf16 [B, L, H, D] -> (float8_e4m3fn codes, fp32 scale [B, L, H, 1]).

    Same lines as int8_kv_cache.py:150-153 with 127 -> 448; the cast is RNE after a
    clamp to +-448 (so torch's non-saturating cast never sees an out-of-range value)."""
    src = values.float()
    peak = src.abs().amax(dim=-1, keepdim=True)
    s = torch.where(peak > 0, peak / 448.0, torch.ones_like(peak))
    scaled = src / s
    return scaled.clamp(-448.0, 448.0).to(torch.float8_e4m3fn), s


def quantize(values: torch.Tensor, fmt: str):
    if fmt == "int8":
        return quantize_int8(values)
    if fmt == "fp8_e4m3":
        return quantize_e4m3(values)
    raise ValueError(fmt)


def dequantize(codes: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """bf16(code * scale), one fp32 multiply and one rounding (int8_kv_cache.py:202-204)."""
    return (codes.float() * scale).to(torch.bfloat16)
