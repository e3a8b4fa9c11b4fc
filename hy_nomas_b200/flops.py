"""Algorithmic work of one cached-attention call (the benchmark's unit).

FLOPs = 4 * H * D * (visible query-key pairs): two GEMMs (QK^T and PV) of 2 FLOPs per
multiply-add.  Only pairs that the mask leaves visible count, so skipped tiles are
never credited.  Pairs are counted in closed form from the chunk geometry.
"""
from __future__ import annotations


def visible_pairs(Lh: int, Li: int, Lt: int, attend_txt: bool = True, group_tokens: int = 0,
                  text_valid: int | None = None) -> int:
    """Visible (query, key) pairs for history Lh, image Li, text Lt (text_valid valid)."""
    tv = Lt if text_valid is None else text_valid
    lt_keys = tv if attend_txt else 0
    if group_tokens and Li > 0:
        img_pairs = 0
        for start in range(0, Li, group_tokens):
            rows = min(group_tokens, Li - start)
            img_pairs += rows * min(start + group_tokens, Li)
    else:
        img_pairs = Li * Li
    return Li * (Lh + lt_keys) + img_pairs + tv * (Lh + Li + lt_keys)


def attention_flops(Lh: int, Li: int, Lt: int, H: int, D: int = 128, attend_txt: bool = True,
                    group_tokens: int = 0, batch: int = 1, text_valid: int | None = None) -> float:
    return 4.0 * H * D * batch * visible_pairs(Lh, Li, Lt, attend_txt, group_tokens, text_valid)


def append_bytes(L: int, H: int, D: int = 128, batch: int = 1) -> int:
    """HBM bytes of one K/V pair quantise-on-write: read bf16, write codes + fp32 scales."""
    return batch * 2 * (L * H * D * 2 + L * H * D + L * H * 4)
