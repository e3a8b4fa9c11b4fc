"""Bounded segment-AR history (the sliding-window cache) of the cached path.

Reference: hymm/models/dit/modules/swa_cache.py (``append_dense_record`` :23-35,
``eviction_cut`` :46-61, ``trim_records`` :64-93, ``commit_window`` :96-138), called after
the attention by ``causal_attention_with_cache_mp`` when ``update_cache`` is set and the
cache dict carries ``swa_capacity`` (nomas_cpt.py:593-597, :845-852).  The pipeline enables
it with ``inference.sliding_window`` (hymm/pipeline/causal_ar.py:1637-1657, :1930-1932).

The cache keeps the reference's positional layout (rows [0, swa_valid_len) are the history in
time order, its mask beside it) because the pipeline reads that layout, ``swa_valid_len`` and
``swa_evicted`` between calls (causal_ar.py:2731-2770).  A commit, after the attention has
read the old history:

1. records the chunk: start, image tokens, end, first frame index, and its frame geometry
   (height 1, width ``tokens_per_frame``);
2. cut = the smallest prefix that brings history + chunk within ``swa_capacity`` and ends on
   a frame boundary, or at a record's end when no frame of that record would be left
   (text is never kept without its video);
3. moves history rows [cut, valid) to the front (through a temporary, as the rows overlap);
4. writes the chunk from its first kept token at row valid - cut: quantise-on-write for
   INT8 / E4M3 caches (the library's append kernel), a copy for a bf16 cache;
5. updates the mask, the records, ``swa_valid_len`` and ``swa_evicted``.

The records are the reference's format (a dataclass with the same fields), so either side
can read what the other wrote.  The frame ring of ``window.py`` (sink frames plus a window,
no row moves) is the other history bound this build offers; this module is the drop-in for
callers that use the reference's dict protocol.
"""
from __future__ import annotations

from dataclasses import dataclass, replace

import torch

from . import kv_cache as _kvc

ARCHIVED_SAMPLINGS = ("uniform", "recent_mix_uniform", "temporal_context")


@dataclass
class DenseVideo:
    """One committed chunk: rows [start, end) hold ``image_tokens`` video tokens then text;
    its first frame is ``time_start``; a frame is ``height * width`` tokens."""

    start: int
    image_tokens: int
    end: int
    time_start: int
    height: int
    width: int


def _frame_tokens(record) -> int:
    if record.height <= 0 or record.width <= 0:
        raise ValueError("SWA video frame height and width must be positive")
    ft = record.height * record.width
    if record.image_tokens <= 0 or record.image_tokens % ft:
        raise ValueError("SWA video records must contain a positive whole number of frames")
    return ft


def check_dense_record(cache: dict, valid_len: int, image_tokens: int, tokens_per_frame: int) -> None:
    """The checks of ``append_dense_record``, made before any device work."""
    if tokens_per_frame <= 0 or image_tokens % tokens_per_frame:
        raise ValueError("Dense SWA requires complete video frames and tokens_per_frame > 0")
    if sum(r.end - r.start for r in cache.get("swa_video", [])) != valid_len:
        raise ValueError("Dense SWA metadata does not cover the existing KV cache")


def append_dense_record(cache: dict, valid_len: int, image_tokens: int, text_tokens: int,
                        tokens_per_frame: int) -> None:
    check_dense_record(cache, valid_len, image_tokens, tokens_per_frame)
    records = cache.setdefault("swa_video", [])
    first = cache.get("swa_next_frame", 0)
    records.append(DenseVideo(valid_len, image_tokens, valid_len + image_tokens + text_tokens, first, 1,
                              tokens_per_frame))
    cache["swa_next_frame"] = first + image_tokens // tokens_per_frame


def eviction_cut(records, total: int, capacity: int) -> int:
    """Rows to drop from the front so that ``total`` rows fit ``capacity``: whole frames of
    the first record that reaches past the excess, or all of it when none of its frames
    would stay."""
    excess = total - capacity
    if excess <= 0:
        return 0
    for r in records:
        if r.end < excess:
            continue
        ft = _frame_tokens(r)
        frames = max(0, -((r.start - excess) // ft))     # ceil((excess - start) / ft)
        cut = r.start + frames * ft
        return r.end if cut >= r.start + r.image_tokens else cut
    raise ValueError("SWA frame records do not cover the cache")


def trim_records(records, cut: int):
    """Records after dropping rows [0, cut): shifted, the partly cut one shortened by its
    removed frames."""
    kept = []
    for r in records:
        if r.end <= cut:
            continue
        removed = max(0, cut - r.start)
        ft = _frame_tokens(r)
        if removed % ft or removed >= r.image_tokens:
            raise ValueError("SWA eviction must retain complete video frames")
        if getattr(r, "prototypes", None) is not None:
            raise NotImplementedError("sparse-routing SWA records are not supported by the b200 path")
        kept.append(replace(r, start=max(0, r.start - cut), end=r.end - cut, image_tokens=r.image_tokens - removed,
                            time_start=r.time_start + removed // ft))
    return kept


def _tail(segments, skip: int):
    """The segments [s_0 | s_1] without their first ``skip`` rows."""
    out = []
    for s in segments:
        n = s.shape[1]
        if skip >= n:
            skip -= n
            continue
        out.append(s[:, skip:])
        skip = 0
    return out


def commit_window(cache: dict, mask: torch.Tensor, seg_k, seg_v, cur_mask: torch.Tensor, valid_len: int, *,
                  assume_finite: bool = False) -> None:
    """Commit the chunk ``[seg_0 | seg_1]`` (bf16 [B, L, H, D] each; image then text) with its
    validity ``cur_mask`` bool [B, sum L] after the attention; see the module docstring."""
    capacity = int(cache["swa_capacity"])
    n = sum(s.shape[1] for s in seg_k)
    total = valid_len + n
    key = "swa_video" if "swa_video" in cache else "sparse_video"
    records = cache[key]
    cut = eviction_cut(records, total, capacity)
    hist_start = min(cut, valid_len)
    kept_hist = valid_len - hist_start
    cur_start = max(0, cut - valid_len)
    fmt = _kvc.cache_format(cache)
    compressed = fmt in ("int8", _kvc.FP8_FORMAT)
    names = ("k", "v", "k_scale", "v_scale") if compressed else ("k", "v")
    if kept_hist and hist_start:
        for name in names:
            cache[name][:, :kept_hist].copy_(cache[name][:, hist_start:valid_len].clone())
        mask[:, :kept_hist].copy_(mask[:, hist_start:valid_len].clone())
    new_len = total - cut
    if cur_start < n:
        ks, vs = _tail(seg_k, cur_start), _tail(seg_v, cur_start)
        if compressed:
            _kvc.quantize_kv_segments_into(cache, ks, vs, kept_hist, assume_finite=assume_finite)
        else:
            row = kept_hist
            for tk, tv in zip(ks, vs):
                cache["k"][:, row:row + tk.shape[1]].copy_(tk)
                cache["v"][:, row:row + tv.shape[1]].copy_(tv)
                row += tk.shape[1]
    mask[:, kept_hist:new_len].copy_(cur_mask[:, cur_start:])
    mask[:, new_len:] = False
    mask._action_tail_ranges = []
    cache[key] = trim_records(records, cut)
    cache["swa_valid_len"] = new_len
    cache["swa_evicted"] = cut
    if fmt == "int8" and cur_start < n:
        stats = cache.setdefault("kv_codec_stats", {})
        stats["encode_calls"] = stats.get("encode_calls", 0) + 1
