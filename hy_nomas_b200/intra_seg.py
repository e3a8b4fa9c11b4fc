"""Intra-segment action masks of the cached path, composed from the library's kernels.

Reference: ``_build_intra_seg_cache_ranges`` and ``_intra_seg_cache_forward``
(hymm/models/dit/nomas_cpt.py:107-332), dispatched at :691-770 when ``cache_txt`` is set and a
per-action payload is given; the reactor's staging path passes the same payload to its
kernel (reactor/hy_nomas_cache.py:300-326).

Per sample, with text offsets ``[o_0, ..., o_A]`` counted over its valid text tokens:

* C = the visible history, the current image keys (block-causal when ``group_tokens`` is
  set) and the head text [o_0 tokens): every query with ranges sees C;
* image rows of a window whose action is a, and the text rows of action a
  ([o_a, o_{a+1}) in valid-token order), also see action a's text keys;
* image rows outside every window, valid text rows at or past o_A and padded text rows are
  zero.

A sample whose offsets are None keeps full attention over its visible tokens.  Overlapping
windows are refused: the reference's flex backend refuses overlapping rectangles
(attention/range_attention.py:97-100) and its magi kernel would count such keys twice.

No kernel of its own; each step is a library call that the other paths use:

1. ``hyb_cached_attention`` with the head text as the text mask: image rows see C, head
   text rows are final, the LSE of every row is kept.
2. Text rows against C: ``hyb_attn_fwd`` over the keys that step 1 staged in its
   workspace, the text queries staged head-major, into an fp32 accumulator.
3. Per action: the rows that see it (its windows' image rows and all text rows, the text
   rows of other actions given LSE -inf) against the action's text keys alone, then
   ``hyb_lse_merge`` with the rows' results over C, and the rows written back.

Over a plain call this adds one pass of the text rows over the staged keys and one key tile
per action.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import torch

from . import _lib

_D = 128


@dataclass
class IntraPlan:
    """Host-side geometry of one sample's intra-segment mask."""

    offsets: list
    windows: list                      # (start, end, action or -1): clamped, nonempty, sorted
    uncovered: list                    # image row ranges outside every window (zero rows)
    action_rows: list = field(default_factory=list)   # per action: its windows' row ranges
    live_actions: list = field(default_factory=list)  # actions whose text slice is nonempty


def plan_intra_segment(img_len: int, offsets, windows, tokens_per_frame: int) -> IntraPlan:
    """Windows in latent frames -> token row ranges (nomas_cpt.py:737-748: frame index times
    ``tokens_per_frame``, or 1 without it), clamped to the image rows as ``_emit`` clamps them
    (:170-175).  Raises ValueError for negative or decreasing offsets and overlapping windows."""
    offs = [int(o) for o in offsets]
    if not offs:
        raise ValueError("intra-segment text offsets must hold at least the head end")
    if any(o < 0 for o in offs) or any(b < a for a, b in zip(offs, offs[1:])):
        raise ValueError("intra-segment text offsets must be nonnegative and nondecreasing")
    tpf = int(tokens_per_frame) if tokens_per_frame and int(tokens_per_frame) > 0 else 1
    A = len(offs) - 1
    wins = []
    for w in windows:
        ws = max(0, min(int(w[0]) * tpf, img_len))
        we = max(0, min(int(w[1]) * tpf, img_len))
        a = int(w[2])
        if we > ws:
            wins.append((ws, we, a if 0 <= a < A else -1))
    wins.sort()
    for (_, e0, _), (s1, _, _) in zip(wins, wins[1:]):
        if s1 < e0:
            raise ValueError("intra-segment video windows overlap")
    uncovered, pos = [], 0
    for ws, we, _ in wins:
        if ws > pos:
            uncovered.append((pos, ws))
        pos = we
    if pos < img_len:
        uncovered.append((pos, img_len))
    action_rows = [[(ws, we) for ws, we, a in wins if a == k] for k in range(A)]
    live = [k for k in range(A) if offs[k] < offs[k + 1]]
    return IntraPlan(offs, wins, uncovered, action_rows, live)


def text_row_masks(text_mask_row, txt_len: int, offsets, device):
    """Head-text and per-action masks over the text rows, computed on the device without a
    host sync: a valid token's compact index is its rank among the valid tokens, and
    clamping the offsets to the valid count (nomas_cpt.py:301-309) changes no comparison
    with a rank that is below that count."""
    tm = (torch.ones(txt_len, dtype=torch.bool, device=device) if text_mask_row is None
          else text_mask_row.reshape(txt_len).to(device=device, dtype=torch.bool))
    rank = torch.cumsum(tm.to(torch.int32), 0) - 1
    head = tm & (rank < offsets[0])
    actions = [tm & (rank >= offsets[a]) & (rank < offsets[a + 1]) for a in range(len(offsets) - 1)]
    return head, actions


def pack_key_bits(mask: torch.Tensor, kwords: int) -> torch.Tensor:
    """bool [L] -> the attention kernel's key bitmap, int32 [kwords] (key j is bit j % 32 of
    word j // 32)."""
    L = mask.numel()
    bits = torch.zeros(kwords * 32, dtype=torch.int64, device=mask.device)
    bits[:L] = mask.reshape(L).to(torch.int64)
    w = (bits.view(kwords, 32) << torch.arange(32, dtype=torch.int64, device=mask.device)).sum(1)
    return torch.where(w >= 2 ** 31, w - 2 ** 32, w).to(torch.int32)


def _sample_cache(kv_cache: dict, b: int) -> dict:
    d = dict(kv_cache)
    for name in ("k", "v", "k_scale", "v_scale"):
        t = d.get(name)
        if torch.is_tensor(t):
            d[name] = t[b:b + 1]
    return d


def _accumulate(lib, stream, status, H, q_head_major, Lq, k, v, Lk, kbits, kwords, scale, splits_hint, v_f16=0):
    """One accumulator-mode launch: rows [Lq] of ``q_head_major`` against keys [Lk] (every
    key visible where its bit is set) -> fp32 rows [Lq, H, 128] and natural-log LSE [H, Lq].
    ``v_f16``: the staged values are fp16 (the cached attention's workspace) rather than bf16."""
    dev = q_head_major.device
    acc = torch.empty((Lq, H, _D), dtype=torch.float32, device=dev)
    acc_lse = torch.empty((H, Lq), dtype=torch.float32, device=dev)
    never_written = torch.empty((1, Lq, H, _D), dtype=torch.bfloat16, device=dev)   # mode 0 writes no bf16
    a = _lib.AttnArgs()
    a.abi_version = _lib.HYB_ABI_VERSION
    a.B, a.H, a.D, a.Lq, a.Lk = 1, H, _D, Lq, Lk
    a.hist_len, a.img_len, a.img_k_len, a.group_tokens = 0, Lq, Lk, 0
    a.softmax_scale = scale
    a.q, a.k, a.v = q_head_major.data_ptr(), k, v
    a.kbits, a.kwords = kbits, kwords
    a.qbits, a.qwords = None, 0
    a.out_img = never_written.data_ptr()
    a.oi_sb, a.oi_st, a.oi_sh = never_written.stride()[:3]
    a.oi_seg, a.oi_sseg = Lq, 0
    a.lse = None
    a.dev_status = status.data_ptr()
    a.kv_splits = max(1, int(splits_hint))
    a.v_f16 = int(v_f16)
    if a.kv_splits > 1:
        part_o = torch.empty((a.kv_splits * H * Lq * _D,), dtype=torch.float32, device=dev)
        part_lse = torch.empty((a.kv_splits * H * Lq,), dtype=torch.float32, device=dev)
        a.part_o, a.part_lse = part_o.data_ptr(), part_lse.data_ptr()
    a.acc_o, a.acc_lse, a.acc_mode = acc.data_ptr(), acc_lse.data_ptr(), 0
    _lib.check(lib.hyb_attn_fwd(ctypes.byref(a), stream), "intra-segment attention")
    return acc, acc_lse


def _stage(lib, stream, t: torch.Tensor, t2: torch.Tensor | None = None):
    """bf16 [1, L, H, 128] (and a second of the same shape) -> head-major [H, L, 128]."""
    L, H = t.shape[1], t.shape[2]
    dst = torch.empty((H, max(L, 1), _D), dtype=torch.bfloat16, device=t.device)
    dst2 = torch.empty_like(dst) if t2 is not None else None
    v1 = _lib.bf16_view(t)
    v2 = _lib.bf16_view(t2) if t2 is not None else None
    _lib.check(lib.hyb_stage_head_major(1, L, H, _D, ctypes.byref(v1), ctypes.byref(v2) if v2 is not None else None,
                                        dst.data_ptr(), dst2.data_ptr() if dst2 is not None else None, stream),
               "intra-segment staging")
    return dst, dst2


def intra_segment_attention(img_q, img_k, img_v, txt_q, txt_k, txt_v, kv_cache, cache_valid_len, *,
                            offsets_per_sample, windows, tokens_per_frame, history_mask=None, text_mask=None,
                            hist_rows=None, group_tokens=0, out_img, out_txt):
    """One rank's cached attention with intra-segment action masks (after any Ulysses
    exchange).  Inputs bf16 [B, L, H, 128]; ``out_img`` / ``out_txt`` bf16 [B, L, H, 128]
    (any strides, unit stride on the last dimension) receive the result."""
    from .attention import Workspace, cached_attention_local, workspace_layout

    lib = _lib.load()
    B, Li, H, _ = img_q.shape
    Lt = txt_q.shape[1]
    dev = img_q.device
    stream = _lib.stream_ptr(dev)
    status = _lib.device_status(dev)
    for b in range(B):
        sl = slice(b, b + 1)
        kv_b = _sample_cache(kv_cache, b) if kv_cache is not None and kv_cache["k"].shape[0] == B else kv_cache
        if kv_b is not None and "staged" in kv_b:   # the text-row passes below reuse the staging workspace
            kv_b = {name: t for name, t in kv_b.items() if name != "staged"}
        hm_b = history_mask[sl] if history_mask is not None and history_mask.shape[0] == B else history_mask
        tm_b = text_mask[sl] if text_mask is not None else None
        oi_b, ot_b = out_img[sl], out_txt[sl]
        cur = (img_q[sl], img_k[sl], img_v[sl], txt_q[sl], txt_k[sl], txt_v[sl])
        offs = offsets_per_sample[b] if b < len(offsets_per_sample) else None
        if offs is None:
            cached_attention_local(*cur, kv_b, cache_valid_len, history_mask=hm_b, text_mask=tm_b,
                                   attend_txt=True, group_tokens=group_tokens, out_img=oi_b, out_txt=ot_b,
                                   hist_rows=hist_rows)
            continue
        plan = plan_intra_segment(Li, offs, windows, tokens_per_frame)
        head, actions = text_row_masks(tm_b, Lt, plan.offsets, dev)
        lse = torch.empty((1, H, Li + Lt), dtype=torch.float32, device=dev)
        ws = Workspace()
        cached_attention_local(*cur, kv_b, cache_valid_len, history_mask=hm_b, text_mask=head[None],
                               attend_txt=True, group_tokens=group_tokens, out_img=oi_b, out_txt=ot_b, lse=lse,
                               hist_rows=hist_rows, workspace=ws)
        for a0, a1 in plan.uncovered:
            oi_b[:, a0:a1].zero_()
        live = plan.live_actions if Lt > 0 else []
        if not live:
            continue
        at = ws.attn_args
        with torch.cuda.device(dev):
            # text rows against C, over the keys the call above staged
            qt, _ = _stage(lib, stream, cur[3])
            lay = workspace_layout(1, H, at.Lk - Lt, 0, Lt, True)
            acc_t, lse_t = _accumulate(lib, stream, status, H, qt, Lt, at.k, at.v, at.Lk, at.kbits, at.kwords,
                                       at.softmax_scale, lay.kv_splits, v_f16=at.v_f16)
            kt, vt = _stage(lib, stream, cur[4], cur[5])
            kwords_t = ((Lt + 127) // 128) * 4
            for a in live:
                rows = plan.action_rows[a]
                n_img = sum(e - s for s, e in rows)
                n = n_img + Lt
                qa = torch.cat([cur[0][:, s:e] for s, e in rows] + [cur[3]], dim=1)
                qa_h, _ = _stage(lib, stream, qa)
                bits = pack_key_bits(actions[a], kwords_t)
                acc_a, lse_a = _accumulate(lib, stream, status, H, qa_h, n, kt.data_ptr(), vt.data_ptr(), Lt,
                                           bits.data_ptr(), kwords_t, at.softmax_scale, 1)
                lse_a[:, n_img:].masked_fill_(~actions[a][None, :], float("-inf"))
                base_o = torch.cat([oi_b[0, s:e].float() for s, e in rows] + [acc_t], dim=0).contiguous()
                base_lse = torch.cat([lse[0, :, s:e] for s, e in rows] + [lse_t], dim=1).contiguous()
                _lib.check(lib.hyb_lse_merge(n, H, _D, acc_a.data_ptr(), lse_a.data_ptr(), base_o.data_ptr(), 1,
                                             base_lse.data_ptr(), stream), "intra-segment merge")
                off = 0
                for s, e in rows:
                    oi_b[0, s:e].copy_(acc_a[off:off + e - s])
                    off += e - s
                ot_b[0].copy_(torch.where(actions[a][:, None, None], acc_a[n_img:].to(torch.bfloat16), ot_b[0]))
    return out_img, out_txt
