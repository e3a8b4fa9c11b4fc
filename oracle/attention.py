"""Cached chunk attention restated on the CPU in fp32 — test infrastructure only.

Semantics of ``causal_attention_with_cache_mp`` (hymm/models/dit/nomas_cpt.py):
  * keys  = [history | current image | current text]          (:608-649)
    text keys are present iff ``cache_txt or update_cache``    (:613-649)
  * key mask = [cache_mask[:, :valid] | ones | text_mask]      (:651-685)
  * queries = [current image | current text]                   (:687-690)
  * flash3 path: masked (padded) text queries produce zero rows (unpad/pad, :807-829)
  * history with batch 1 broadcasts over a larger current batch (:547-567)
Frame-level block-causal extension: image query i sees image key j iff
j // G <= i // G with G = chunk_causal_frames * tokens_per_frame, the chunk-causal
ranges of ``create_magi_mp_causal_ranges`` (attention/magi_attn.py:290-309, chunk c:
q [cT, (c+1)T) -> k [0, (c+1)T)); text queries see every visible key.
The softmax is computed exactly (fp32 scores, max-subtracted exp, fp32 sum).
"""
from __future__ import annotations

import math

import torch


def visibility(Lh: int, Li: int, Lt: int, attend_txt: bool, group_tokens: int,
               history_mask=None, text_mask=None, batch: int = 1) -> torch.Tensor:
    """bool [B, Lq, Lk] visibility of key j for query i."""
    Lk = Lh + Li + (Lt if attend_txt else 0)
    Lq = Li + Lt
    vis = torch.ones(batch, Lq, Lk, dtype=torch.bool)
    if history_mask is not None and Lh > 0:
        hm = history_mask[:, :Lh].to(torch.bool)
        if hm.shape[0] != batch:
            hm = hm.expand(batch, -1)
        vis[:, :, :Lh] &= hm[:, None, :]
    if attend_txt and Lt > 0 and text_mask is not None:
        vis[:, :, Lh + Li:] &= text_mask.to(torch.bool)[:, None, :]
    if group_tokens and Li > 0:
        qb = torch.arange(Li) // group_tokens
        kb = torch.arange(Li) // group_tokens
        vis[:, :Li, Lh:Lh + Li] &= (kb[None, :] <= qb[:, None])[None]
    return vis


def cached_attention(img_q, img_k, img_v, txt_q, txt_k, txt_v, hist_k, hist_v, *,
                     history_mask=None, text_mask=None, attend_txt=True, group_tokens=0,
                     softmax_scale=None, return_lse=False, return_magnitude=False):
    """Reference output of one rank's cached attention, fp32 [B, Li, H, D] / [B, Lt, H, D].

    ``hist_k`` / ``hist_v`` are the bf16 history (already decoded), batch B or 1.
    ``return_magnitude`` also returns softmax(S) @ |V| (the weighted magnitude of the values
    each output element sums, which scales the rounding error of a bf16 P)."""
    B, Li, H, D = img_q.shape
    Lt = txt_q.shape[1]
    Lh = hist_k.shape[1]
    if hist_k.shape[0] != B:
        hist_k = hist_k.expand(B, -1, -1, -1)
        hist_v = hist_v.expand(B, -1, -1, -1)
    parts_k = [hist_k, img_k] + ([txt_k] if attend_txt else [])
    parts_v = [hist_v, img_v] + ([txt_v] if attend_txt else [])
    k = torch.cat([p.float() for p in parts_k], dim=1)
    v = torch.cat([p.float() for p in parts_v], dim=1)
    q = torch.cat([img_q.float(), txt_q.float()], dim=1)
    vis = visibility(Lh, Li, Lt, attend_txt, group_tokens, history_mask, text_mask, B)
    qvalid = torch.ones(B, Li + Lt, dtype=torch.bool)
    if text_mask is not None and Lt > 0:
        qvalid[:, Li:] = text_mask.to(torch.bool)
    return _masked_attention(q, k, v, vis, qvalid, Li, softmax_scale, return_lse, return_magnitude)


def _masked_attention(q, k, v, vis, qvalid, Li, softmax_scale=None, return_lse=False, return_magnitude=False):
    """Exact softmax attention of fp32 q [B, Lq, H, D] over k/v [B, Lk, H, D] with the
    visibility ``vis`` [B, Lq, Lk]; rows where ``qvalid`` [B, Lq] is false are zero (LSE -inf).
    Returns the image rows [:Li] and the text rows [Li:] (plus LSE / magnitude on request)."""
    D = q.shape[-1]
    scale = softmax_scale if softmax_scale else 1.0 / math.sqrt(D)
    qh = q.permute(0, 2, 1, 3)                        # [B, H, Lq, D]
    kh = k.permute(0, 2, 1, 3)
    vh = v.permute(0, 2, 1, 3)
    s = torch.matmul(qh, kh.transpose(-1, -2)) * scale
    s = s.masked_fill(~vis[:, None], float("-inf"))
    m = s.amax(dim=-1, keepdim=True)
    m = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
    p = torch.exp(s - m)
    l = p.sum(dim=-1, keepdim=True)
    o = torch.matmul(p, vh) / torch.where(l > 0, l, torch.ones_like(l))
    mag = torch.matmul(p, vh.abs()) / torch.where(l > 0, l, torch.ones_like(l)) if return_magnitude else None
    lse = (m + torch.log(l)).squeeze(-1)               # [B, H, Lq]
    o = o.permute(0, 2, 1, 3)                          # [B, Lq, H, D]
    o = o * qvalid[:, :, None, None]
    lse = torch.where(qvalid[:, None, :] & (l.squeeze(-1) > 0), lse, torch.full_like(lse, float("-inf")))
    out = (o[:, :Li], o[:, Li:])
    if return_lse:
        out = out + (lse,)
    if return_magnitude:
        mag = mag.permute(0, 2, 1, 3)
        out = out + ((mag[:, :Li], mag[:, Li:]),)
    return out


def reference_sdpa_path(img_q, img_k, img_v, txt_q, txt_k, txt_v, hist_k, hist_v, *,
                        history_mask=None, text_mask=None, attend_txt=True, group_tokens=0):
    """The reference's CPU path restated (nomas_cpt.py:608-685 compose, :771-781 SDPA with
    ``attn_mask``), in the input dtype, with the chunk-causal ranges folded into the mask.

    This is what ``bench.py`` times as the CPU baseline: decoded bf16 history, torch.cat
    of [history | image | text], one F.scaled_dot_product_attention call."""
    import torch.nn.functional as F
    B, Li, H, D = img_q.shape
    Lt = txt_q.shape[1]
    Lh = hist_k.shape[1]
    if hist_k.shape[0] != B:
        hist_k = hist_k.expand(B, -1, -1, -1)
        hist_v = hist_v.expand(B, -1, -1, -1)
    full_k = torch.cat([hist_k, img_k] + ([txt_k] if attend_txt else []), dim=1)
    full_v = torch.cat([hist_v, img_v] + ([txt_v] if attend_txt else []), dim=1)
    q_full = torch.cat([img_q, txt_q], dim=1)
    vis = visibility(Lh, Li, Lt, attend_txt, group_tokens, history_mask, text_mask, B)
    hidden = F.scaled_dot_product_attention(
        q_full.transpose(1, 2), full_k.transpose(1, 2), full_v.transpose(1, 2),
        attn_mask=vis[:, None], dropout_p=0.0, is_causal=False)
    return hidden.transpose(1, 2)


def intra_segment_rows(Li: int, Lt: int, offsets, windows_tok, text_mask=None):
    """Per-row key classes of the intra-segment action mask for one sample.

    ``offsets`` is ``[o_0, ..., o_A]`` counted over the sample's valid text tokens (head text
    [0, o_0), action a [o_a, o_{a+1})); ``windows_tok`` lists ``[start, end, action]`` image
    token windows (action -1 = a gap).  Follows ``_build_intra_seg_cache_ranges`` /
    ``_emit`` (hymm/models/dit/nomas_cpt.py:107-193) and the per-sample compaction of
    ``_intra_seg_cache_forward`` (:198-332).  Returns ``row_action`` int [Li + Lt] (-2: the
    row has no ranges and stays zero; -1: common keys only; a >= 0: common keys + action a's
    text) and the text-key masks ``head`` bool [Lt] and ``actions`` bool [A, Lt]."""
    offs = [int(o) for o in offsets]
    if any(o < 0 for o in offs) or any(b < a for a, b in zip(offs, offs[1:])):
        raise ValueError("intra-segment text offsets must be nonnegative and nondecreasing")
    tm = torch.ones(Lt, dtype=torch.bool) if text_mask is None else text_mask.to(torch.bool).reshape(Lt)
    rank = torch.cumsum(tm.to(torch.int64), 0) - 1          # compact index of each valid text token
    A = len(offs) - 1
    head = tm & (rank < offs[0])
    actions = torch.stack([tm & (rank >= offs[a]) & (rank < offs[a + 1]) for a in range(A)]) if A > 0 \
        else torch.zeros(0, Lt, dtype=torch.bool)
    row_action = torch.full((Li + Lt,), -2, dtype=torch.int64)
    covered = torch.zeros(Li, dtype=torch.bool)
    for ws, we, aidx in windows_tok:
        ws, we = max(0, min(int(ws), Li)), max(0, min(int(we), Li))
        if we <= ws:
            continue
        if covered[ws:we].any():
            raise ValueError("intra-segment video windows overlap")
        covered[ws:we] = True
        row_action[ws:we] = int(aidx) if 0 <= int(aidx) < A else -1
    txt_rows = row_action[Li:]
    txt_rows[head] = -1
    for a in range(A):
        txt_rows[actions[a]] = a
    return row_action, head, actions


def intra_segment_visibility(Lh: int, Li: int, Lt: int, offsets_per_sample, windows_tok, *,
                             history_mask=None, text_mask=None, group_tokens=0, batch=1):
    """bool visibility [B, Lq, Lk] and query validity [B, Lq] of the cached path with
    intra-segment action masks (nomas_cpt.py:691-770).  A sample whose offsets are None (or
    missing) keeps full attention over its visible tokens (:307-313)."""
    vis = visibility(Lh, Li, Lt, True, group_tokens, history_mask, text_mask, batch)
    qvalid = torch.ones(batch, Li + Lt, dtype=torch.bool)
    if text_mask is not None and Lt > 0:
        qvalid[:, Li:] = text_mask.to(torch.bool)
    for b in range(batch):
        offs = offsets_per_sample[b] if b < len(offsets_per_sample) else None
        if offs is None:
            continue
        tm = text_mask[b] if text_mask is not None else None
        row_action, head, actions = intra_segment_rows(Li, Lt, offs, windows_tok, tm)
        tv = head[None, :].expand(Li + Lt, Lt).clone()
        sel = row_action >= 0
        if sel.any():
            tv[sel] |= actions[row_action[sel]]
        vis[b, :, Lh + Li:] = tv
        none = row_action == -2
        vis[b, none] = False
        qvalid[b] = ~none
    return vis, qvalid


def intra_segment_attention(img_q, img_k, img_v, txt_q, txt_k, txt_v, hist_k, hist_v, offsets_per_sample,
                            windows_tok, *, history_mask=None, text_mask=None, group_tokens=0,
                            softmax_scale=None, return_magnitude=False):
    """Cached attention with intra-segment action masks, fp32 [B, Li, H, D] / [B, Lt, H, D].
    Rows without ranges (image rows outside every window, text rows past the last action,
    padded text rows) are zero, as in ``_intra_seg_cache_forward`` (nomas_cpt.py:236, :325-331)."""
    B, Li, H, D = img_q.shape
    Lt = txt_q.shape[1]
    Lh = hist_k.shape[1]
    if hist_k.shape[0] != B:
        hist_k = hist_k.expand(B, -1, -1, -1)
        hist_v = hist_v.expand(B, -1, -1, -1)
    k = torch.cat([hist_k.float(), img_k.float(), txt_k.float()], dim=1)
    v = torch.cat([hist_v.float(), img_v.float(), txt_v.float()], dim=1)
    q = torch.cat([img_q.float(), txt_q.float()], dim=1)
    vis, qvalid = intra_segment_visibility(Lh, Li, Lt, offsets_per_sample, windows_tok, history_mask=history_mask,
                                           text_mask=text_mask, group_tokens=group_tokens, batch=B)
    return _masked_attention(q, k, v, vis, qvalid, Li, softmax_scale, False, return_magnitude)
