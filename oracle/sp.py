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


def partial_attention(q, k, v, scale=None):
    """Softmax attention of q [B, Lq, H, D] over k/v [B, Lk, H, D] in float64: returns the
    normalised rows O [B, Lq, H, D] and their natural-log LSE [B, H, Lq] (-inf and zero rows
    when there is no key), the partial result one rank contributes for its keys."""
    B, Lq, H, D = q.shape
    scale = scale or D ** -0.5
    if k.shape[1] == 0:
        return torch.zeros(B, Lq, H, D, dtype=torch.float64), torch.full((B, H, Lq), float("-inf"), dtype=torch.float64)
    s = torch.einsum("bqhd,bkhd->bhqk", q.double(), k.double()) * scale
    lse = torch.logsumexp(s, dim=-1)
    p = torch.exp(s - lse[..., None])
    return torch.einsum("bhqk,bkhd->bqhd", p, v.double()), lse


def kv_stationary_step(q_slice, k_slice, v_slice, txt_q, txt_k, txt_v, hist_k, hist_v, group=None):
    """One step of the KV-stationary schedule restated on CPU with torch.distributed collectives
    (the protocol of hy_nomas_b200/kv_stationary.py; no reference counterpart in code, whose ring
    passes K/V instead, dynamic_ring_attention.py:115-286).  Rank r holds its slice of the frame
    (q/k/v_slice [B, Ls, H, D]), its history keys hist_k/hist_v [B, Lh_r, H, D] and the text
    tokens (the same on every rank).  Q is all-gathered; each rank attends every query to its
    keys (text keys on rank 0 only); the partial rows of image query q go to rank q // Ls and the
    text rows to every rank; the owner merges them (lse_merge).  Returns this rank's image rows
    [B, Ls, H, D] and the text rows [B, Lt, H, D] in float64."""
    import torch.distributed as dist
    P, r = dist.get_world_size(group), dist.get_rank(group)
    B, Ls, H, D = q_slice.shape
    Lt = txt_q.shape[1]
    gathered = [torch.empty_like(q_slice) for _ in range(P)]
    dist.all_gather(gathered, q_slice.contiguous(), group=group)
    q_all = torch.cat(gathered + [txt_q], dim=1)                 # [B, P*Ls + Lt, H, D]
    keys = [hist_k, k_slice] + ([txt_k] if r == 0 else [])
    vals = [hist_v, v_slice] + ([txt_v] if r == 0 else [])
    o, lse = partial_attention(q_all, torch.cat(keys, 1), torch.cat(vals, 1))
    # every rank's partials reach every rank (all_gather stands in for the scatter to owners);
    # the owner keeps its rows
    o_all = [torch.empty_like(o) for _ in range(P)]
    lse_all = [torch.empty_like(lse) for _ in range(P)]
    dist.all_gather(o_all, o, group=group)
    dist.all_gather(lse_all, lse, group=group)
    rows = list(range(r * Ls, (r + 1) * Ls)) + list(range(P * Ls, P * Ls + Lt))
    acc_o = o_all[0][:, rows][0]                                 # [S, H, D] (B = 1)
    acc_lse = lse_all[0][0][:, rows]                             # [H, S]
    for s in range(1, P):
        acc_o, acc_lse = lse_merge(acc_o, acc_lse, o_all[s][:, rows][0], lse_all[s][0][:, rows])
    return acc_o[None, :Ls], acc_o[None, Ls:]
