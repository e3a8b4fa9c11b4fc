"""Sequence-parallel layouts and the ring merge, restated on the CPU — test infrastructure only.

* ``pack_seq_to_heads`` / ``simulate_all_to_all`` / ``unpack_seq_to_heads`` restate
  ``_all_to_all_4D(scatter_idx=2, gather_idx=1)`` with the batch packing of
  ``all_to_all_qkv`` (hymm/distributed/communications.py:101-141, :270-280).
* ``pack_heads_to_seq`` / ``unpack_heads_to_seq`` restate scatter_idx=1, gather_idx=2
  (:143-198).
* ``lse_merge`` restates flash_attn_fwd_softmax_lse_correction and
  flash_attn_fwd_out_correction (attention/dynamic_ring_attention.py:86-105).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def pack_seq_to_heads(tensors, P: int, Ls_max: int) -> torch.Tensor:
    """[B, Ls, H, D] x n -> send buffer [P, Ls_max, n*B, H/P, D] (padding zero)."""
    x = torch.cat(tensors, dim=0)                      # [nB, Ls, H, D]
    nB, Ls, H, D = x.shape
    if Ls < Ls_max:
        x = F.pad(x, (0, 0, 0, 0, 0, Ls_max - Ls))
    # (nB, Ls, P, H/P, D) -> (P, Ls, nB, H/P, D), communications.py:113-124
    return x.reshape(nB, Ls_max, P, H // P, D).permute(2, 1, 0, 3, 4).contiguous()


def simulate_all_to_all(sends):
    """Rank r receives block r of every sender, stacked by sender."""
    P = len(sends)
    return [torch.stack([sends[src][r] for src in range(P)], dim=0) for r in range(P)]


def unpack_seq_to_heads(recv: torch.Tensor, lens, n: int):
    """[P, Ls_max, nB, Hp, D] -> n tensors [B, L, Hp, D] (padding removed)."""
    P, Ls_max, nB, Hp, D = recv.shape
    rows = torch.cat([recv[src, :lens[src]] for src in range(P)], dim=0)   # [L, nB, Hp, D]
    full = rows.permute(1, 0, 2, 3)
    B = nB // n
    return [full[i * B:(i + 1) * B].contiguous() for i in range(n)]


def pack_heads_to_seq(x: torch.Tensor, lens) -> torch.Tensor:
    """[B, L, Hp, D] -> send buffer [P, Hp, Ls_max, B, D] (each rank's rows, padded)."""
    B, L, Hp, D = x.shape
    P = len(lens)
    Ls_max = max(lens)
    chunks = []
    for c in x.split(list(lens), dim=1):
        chunks.append(F.pad(c, (0, 0, 0, 0, 0, Ls_max - c.shape[1])))
    y = torch.stack(chunks, dim=0)                      # [P, B, Ls_max, Hp, D]
    return y.permute(0, 3, 2, 1, 4).contiguous()


def unpack_heads_to_seq(recv: torch.Tensor, Ls: int) -> torch.Tensor:
    """[P, Hp, Ls_max, B, D] -> [B, Ls, H, D]."""
    P, Hp, Ls_max, B, D = recv.shape
    y = recv[:, :, :Ls].reshape(P * Hp, Ls, B, D)
    return y.permute(2, 1, 0, 3).contiguous()


def lse_merge(out_acc, lse_acc, out_b, lse_b):
    """Merge (out_b, lse_b) into (out_acc, lse_acc); out [..., S, H, D], lse [H, S].

    Equivalent to the reference's final-lse rescaling of every step's output."""
    mx = torch.maximum(lse_acc, lse_b)
    mn = torch.minimum(lse_acc, lse_b)
    finite = torch.isfinite(mx)
    safe_mx = torch.where(finite, mx, torch.zeros_like(mx))
    lse = torch.where(finite, safe_mx + torch.log1p(torch.exp(mn - safe_mx)), mx)
    wa = torch.where(finite, torch.exp(lse_acc - lse), torch.zeros_like(lse))
    wb = torch.where(finite, torch.exp(lse_b - lse), torch.zeros_like(lse))
    wa = wa.transpose(0, 1)[..., None]                  # [S, H, 1]
    wb = wb.transpose(0, 1)[..., None]
    return out_acc * wa + out_b * wb, lse
