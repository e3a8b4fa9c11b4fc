"""Drop-in ``causal_attention_with_cache_mp`` on the sm_100a library.

Same signature, argument meaning, mutation contract and exceptions as the reference
(``hymm/models/dit/nomas_cpt.py:335-884``), including the reactor's older positional
order (``reactor/hy_nomas_cache.py:192-209``, which lacks ``sp_metadata`` and
``attention_metadata``).  One call on one rank:

1. SP in (Ulysses): packed Q|K|V all-to-all seq->head, text heads sliced
   (nomas_cpt.py:410-429).
2. Cache write when ``update_cache``: quantise-on-write (INT8 / E4M3) or bf16 copy at
   token offset ``cache_valid_len``; ``cache_mask`` updated in place (:592-606).
3. Attention over [visible history | current image | current text] (:608-685) by
   ``hyb_cached_attention``: history decoded from its codes inside the staging pass,
   masked keys excluded, masked text queries produce zero rows (flash3 semantics,
   :786-829).  ``chunk_causal_frames`` (keyword-only extension) restricts image queries
   to image keys of the same or earlier G-frame blocks, the chunk-causal ranges of
   ``attention/magi_attn.py:290-309``; 0 keeps the reference's bidirectional chunk.
4. SP out: O head->seq all-to-all, text all-gather over heads (:864-872); cast to the
   input dtypes and reshape to [B, L, H*D] (:874-884).

Intra-segment action masks (``intra_seg_txt_offsets`` / ``intra_seg_vid_windows`` with
``cache_txt``, :691-770) run in ``intra_seg.py`` on the same kernels; a cache dict with
``swa_capacity`` is committed after the attention by ``swa.py`` (bounded history, :593-597,
:845-852).  Modes the reference routes elsewhere and this build does not implement raise:
``qvg`` storage, ``sparse_context`` and the archived history samplings of the SWA cache.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional

import torch

from . import _lib
from . import kv_cache as kvc
from . import parallel_states as _ps
from . import swa as _swa

_BACKENDS = ("magi", "flex", "b200")

# Parallel-state provider: (get_sequence_parallel_state, nccl_info).  install.install()
# points this at the reference's hymm.distributed.parallel_states.
_STATE = {"get_state": _ps.get_sequence_parallel_state, "info": _ps.nccl_info}

stats = {"calls": 0, "writes": 0}


def set_parallel_state_provider(get_state, info) -> None:
    _STATE["get_state"] = get_state
    _STATE["info"] = info


def _assume_finite() -> bool:
    return os.environ.get("HYB_ASSUME_FINITE_KV", "0") == "1"


def _kernel_layout(x: torch.Tensor) -> torch.Tensor:
    """The kernels read [B, L, H, D] rows with a unit stride on head_dim, 16-byte aligned.
    The reference accepts any layout, so a tensor in another one is copied once into that form
    (the DiT's projections already have it, and pass through untouched)."""
    st = x.stride()
    if st[-1] == 1 and x.data_ptr() % 16 == 0 and all(s % 8 == 0 for s in st[:-1]):
        return x
    return x.clone(memory_format=torch.contiguous_format)


def _new_out(B, L, H, D, device):
    return torch.empty((B, L, H, D), dtype=torch.bfloat16, device=device)


def workspace_layout(B, H, Lh, Li, Lt, attend_txt, D=128) -> "_lib.WorkspaceLayout":
    """Byte offsets of the staging workspace on the current device (from the library)."""
    lay = _lib.WorkspaceLayout()
    _lib.check(_lib.load().hyb_cached_attention_workspace_layout(B, H, D, Lh, Li, Lt, int(bool(attend_txt)), lay),
               "workspace layout")
    return lay


class Workspace:
    """Reusable staging buffer.  After a call, ``attn_args`` re-launches the attention
    kernel alone on the staged tensors (``hyb_attn_fwd``), e.g. to time it."""

    def __init__(self):
        self.buf = None
        self.attn_args = None
        self.keep = ()

    def get(self, nbytes, device):
        if self.buf is None or self.buf.numel() < nbytes or self.buf.device != device:
            self.buf = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=device)
        return self.buf


def cached_attention_local(
    img_q, img_k, img_v, txt_q, txt_k, txt_v, kv_cache, cache_valid_len, *,
    history_mask=None, text_mask=None, attend_txt=True, group_tokens=0,
    softmax_scale=None, out_img=None, out_img_strides=None, out_txt=None, lse=None,
    hist_rows=None, workspace=None, q_pos0=0, k_pos0=0, img_kv_fmt=None, scatter=None,
):
    """Single-rank attention of the current chunk over [history | image | text].

    Inputs are bf16 [B, L, H, D] (any strides with unit stride on D).  History is
    ``kv_cache`` rows [0, cache_valid_len) in its storage format; ``history_mask`` is
    bool [B or 1, >= cache_valid_len], indexed by cache row.  ``hist_rows`` (int32
    [cache_valid_len] on the device) maps composed history position -> cache row (a
    sink + sliding-window ring); None means rows [0, cache_valid_len).  Returns ``(out_img, out_txt)`` bf16
    [B, L, H, D]; ``out_img`` may be supplied pre-allocated with custom element
    strides ``(sb, st, sh)`` or ``(sb, st, sh, seg, sseg)`` where image row t lands at
    ``(t // seg) * sseg + (t % seg) * st`` (e.g. the Ulysses O send buffer).
    ``q_pos0`` / ``k_pos0`` shift the block-causal rule to global positions (ring steps);
    with ``img_kv_fmt`` (HYB_FMT_E4M3 / HYB_FMT_INT8) ``img_k`` / ``img_v`` are
    ``(codes, scale)`` pairs of a quantised block.

    The image keys may be fewer than the image queries (``img_k`` [B, Lik, H, D]) only together
    with ``scatter`` (an ``_lib.PartScatter``): a rank of a KV-stationary schedule attends every
    query of the chunk to the keys it holds, and the partial rows go to their owner ranks'
    buffers (no outputs here; returns ``(None, None)``).

    A cache that keeps its rows decoded (``kv_cache["staged"]``, see
    ``kv_cache.attach_decoded_mirror`` and ``window.SinkWindowKVCache(decoded=True)``) is read
    from its mirror: rows [0, cache_valid_len) in the mirror's order (``hist_rows`` is then not
    used), and this call's own keys are staged into the mirror rows after them.
    """
    lib = _lib.load()
    B, Li, H, D = img_q.shape
    Lt = txt_q.shape[1]
    Lik = (img_k[0] if img_kv_fmt is not None else img_k).shape[1]
    if Lik != Li and scatter is None:
        raise ValueError(f"image keys ({Lik}) and queries ({Li}) differ without a partial scatter")
    dev = img_q.device
    if kv_cache is None:   # no history: a zero-length bf16 placeholder
        kv_cache = {"k": img_q[:, :0], "v": img_q[:, :0]}
    fmt_name = kvc.cache_format(kv_cache)
    if fmt_name == "none":
        hk, hv = kv_cache["k"], kv_cache["v"]
        if hk.dtype != torch.bfloat16:
            raise RuntimeError(f"b200 cached attention requires a bf16 or quantised cache, got {hk.dtype}")
        hist_k, hist_v = _lib.bf16_view(hk), _lib.bf16_view(hv)
    elif fmt_name in ("int8", kvc.FP8_FORMAT):
        code = _lib.HYB_FMT_INT8 if fmt_name == "int8" else _lib.HYB_FMT_E4M3
        hist_k = _lib.coded_view(kv_cache["k"], kv_cache["k_scale"], code)
        hist_v = _lib.coded_view(kv_cache["v"], kv_cache["v_scale"], code)
    else:
        raise ValueError(f"b200 cached attention does not support {fmt_name!r} storage")
    cache_batch = kv_cache["k"].shape[0]
    _lib.require_same_device(dev, "cached attention tensors", img_k, img_v, txt_q, txt_k, txt_v, kv_cache["k"],
                             kv_cache["v"], history_mask, text_mask, hist_rows, out_img, out_txt, lse,
                             *(kv_cache[n] for n in ("k_scale", "v_scale") if torch.is_tensor(kv_cache.get(n))))
    if scatter is None and out_img is None:
        out_img = _new_out(B, Li, H, D, dev)
    if scatter is None and out_txt is None:
        out_txt = _new_out(B, Lt, H, D, dev)
    oi = tuple(out_img_strides) if out_img_strides is not None else \
        (tuple(out_img.stride()[:3]) if out_img is not None else (0, 0, 0))
    if len(oi) == 3:
        oi = oi + (0, 0)
    # a cache that keeps its history decoded (window.SinkWindowKVCache(decoded=True)): rows
    # [0, cache_valid_len) of its head-major buffers, in slot order; this call stages its own
    # keys after them
    staged = kv_cache.get("staged")
    if staged is not None:
        sk, sv, pitch = staged
        if tuple(sk.shape) != (B, H, pitch, D) or tuple(sv.shape) != (B, H, pitch, D) or sk.dtype != torch.bfloat16 \
                or sv.dtype != torch.float16 or not (sk.is_contiguous() and sv.is_contiguous()):
            raise ValueError(f"a decoded history mirror must be contiguous bf16 K / fp16 V [{B}, {H}, pitch, {D}] "
                             "(one batch row per query batch row)")
        _lib.require_same_device(dev, "decoded history mirror", sk, sv)
        if cache_valid_len + Lik + (Lt if attend_txt else 0) > pitch:
            raise ValueError(f"the decoded history mirror has {pitch} rows; this call needs "
                             f"{cache_valid_len + Lik + (Lt if attend_txt else 0)}")
    ws_bytes = lib.hyb_cached_attention_workspace_bytes_ex(B, H, D, cache_valid_len, Li, Lt, int(attend_txt),
                                                           int(staged is not None))
    if ws_bytes < 0:
        raise RuntimeError("hyb200: unsupported sizes for cached attention (head_dim must be 128)")
    ws_obj = workspace if isinstance(workspace, Workspace) else None
    workspace = ws_obj.get(int(ws_bytes), dev) if ws_obj is not None else \
        torch.empty(max(int(ws_bytes), 256), dtype=torch.uint8, device=dev)
    # The kernels read the masks through raw pointers for every row of this call's geometry, so
    # their shapes are checked here (the reference fails on the same inputs in torch's shape
    # checks); a one-row history mask over a batched cache is broadcast, as SDPA broadcasts it.
    if history_mask is not None:
        history_mask = history_mask.to(torch.bool)
        need = kv_cache["k"].shape[1] if hist_rows is not None else cache_valid_len
        if history_mask.ndim != 2 or history_mask.shape[0] not in (1, cache_batch) or history_mask.shape[1] < need:
            raise ValueError(f"history mask must be bool [1 or {cache_batch}, >= {need}], "
                             f"got {tuple(history_mask.shape)}")
        if history_mask.stride(-1) != 1:
            history_mask = history_mask.contiguous()
        if history_mask.shape[0] != cache_batch:
            history_mask = history_mask.expand(cache_batch, -1)
    if text_mask is not None:
        if Lt > 0 and tuple(text_mask.shape) != (B, Lt):
            raise ValueError(f"text mask must be bool [{B}, {Lt}], got {tuple(text_mask.shape)}")
        text_mask = text_mask.to(torch.bool).contiguous()
    empty = _lib.Tensor4()
    args = _lib.CachedAttnArgs()
    args.abi_version = _lib.HYB_ABI_VERSION
    args.B, args.H, args.D = B, H, D
    args.cache_batch = cache_batch
    args.valid_len = cache_valid_len
    args.img_len, args.txt_len = Li, Lt
    args.attend_txt = int(bool(attend_txt))
    args.group_tokens = int(group_tokens)
    args.softmax_scale = float(softmax_scale) if softmax_scale else 0.0
    args.hist_k, args.hist_v = hist_k, hist_v
    args.q_pos0, args.k_pos0 = int(q_pos0), int(k_pos0)
    args.img_q = _lib.bf16_view(img_q) if Li else empty
    if img_kv_fmt is None:
        args.img_k = _lib.bf16_view(img_k) if Lik else empty
        args.img_v = _lib.bf16_view(img_v) if Lik else empty
    else:
        # quantised current keys/values: (codes, scale) pairs in the given format
        args.img_k = _lib.coded_view(img_k[0], img_k[1], img_kv_fmt) if Lik else empty
        args.img_v = _lib.coded_view(img_v[0], img_v[1], img_kv_fmt) if Lik else empty
    args.img_k_len = Lik if Lik != Li else 0
    args.scatter = ctypes.cast(ctypes.pointer(scatter), ctypes.c_void_p) if scatter is not None else None
    args.txt_q = _lib.bf16_view(txt_q) if Lt else empty
    args.txt_k = _lib.bf16_view(txt_k) if Lt else empty
    args.txt_v = _lib.bf16_view(txt_v) if Lt else empty
    if hist_rows is not None:
        if hist_rows.dtype != torch.int32 or hist_rows.numel() < cache_valid_len or not hist_rows.is_contiguous():
            raise ValueError("hist_rows must be a contiguous int32 tensor with cache_valid_len entries")
    args.hist_rows = _lib.ptr(hist_rows)
    args.cache_mask = _lib.ptr(history_mask)
    args.cache_mask_sb = history_mask.stride(0) if history_mask is not None else 0
    args.text_mask = _lib.ptr(text_mask)
    args.text_mask_sb = text_mask.stride(0) if text_mask is not None else 0
    args.out_img = _lib.ptr(out_img)
    args.oi_sb, args.oi_st, args.oi_sh, args.oi_seg, args.oi_sseg = oi
    args.out_txt = _lib.ptr(out_txt)
    args.ot_sb, args.ot_st, args.ot_sh = out_txt.stride()[:3] if out_txt is not None else (0, 0, 0)
    args.lse = _lib.ptr(lse)
    args.workspace = workspace.data_ptr()
    args.workspace_bytes = workspace.numel()
    args.dev_status = _lib.device_status(dev).data_ptr()
    if staged is not None:
        args.staged_k, args.staged_v, args.staged_pitch = staged[0].data_ptr(), staged[1].data_ptr(), int(staged[2])
    with torch.cuda.device(dev):
        _lib.check(lib.hyb_cached_attention(args, _lib.stream_ptr(dev)), "cached attention")
    if ws_obj is not None and staged is not None:
        ws_obj.attn_args = None   # the kernel-only relaunch covers the staging-workspace layout only
    if ws_obj is not None and scatter is None and staged is None:
        with torch.cuda.device(dev):
            lay = workspace_layout(B, H, cache_valid_len, Li, Lt, attend_txt, D)
        base = workspace.data_ptr()
        at = _lib.AttnArgs()
        at.abi_version = _lib.HYB_ABI_VERSION
        at.B, at.H, at.D, at.Lq, at.Lk = B, H, D, lay.Lq, lay.Lk
        at.hist_len, at.img_len, at.group_tokens = cache_valid_len, Li, int(group_tokens)
        at.softmax_scale = args.softmax_scale
        at.q_pos0, at.k_pos0 = args.q_pos0, args.k_pos0
        at.q, at.k, at.v = base + lay.q, base + lay.k, base + lay.v
        at.kbits, at.kwords = base + lay.kbits, lay.kwords
        at.qbits, at.qwords = base + lay.qbits, lay.qwords
        at.kv_splits = lay.kv_splits
        at.v_f16 = 1   # the staged V is fp16 (P.V in fp16)
        at.part_o, at.part_lse = base + lay.part_o, base + lay.part_lse
        at.out_img = args.out_img
        at.oi_sb, at.oi_st, at.oi_sh = oi[0], oi[1], oi[2]
        at.oi_seg, at.oi_sseg = (oi[3], oi[4]) if oi[3] > 0 else (max(Li, 1), 0)
        at.out_txt = args.out_txt
        at.ot_sb, at.ot_st, at.ot_sh = args.ot_sb, args.ot_st, args.ot_sh
        at.lse = args.lse
        at.dev_status = args.dev_status
        ws_obj.attn_args = at
        ws_obj.keep = (out_img, out_txt, lse)
    return out_img, out_txt


def causal_attention_with_cache_mp(
    q,
    k,
    v,
    kv_cache,
    cache_valid_len: int = 0,
    attn_mode: Optional[str] = None,
    text_mask: Optional[torch.Tensor] = None,
    update_cache: bool = False,
    cache_txt: bool = True,
    cache_mask: Optional[torch.Tensor] = None,
    intra_seg_txt_offsets=None,
    intra_seg_vid_windows=None,
    tokens_per_frame: int = 0,
    seg_ar_attention_backend: str = "magi",
    sparse_context=None,
    sp_metadata=None,
    attention_metadata=None,
    *,
    chunk_causal_frames: int = 0,
):
    """Multi-prompt causal attention with KV cache on B200 (see module docstring)."""
    if seg_ar_attention_backend not in _BACKENDS:
        raise ValueError("Invalid seg_ar_attention_backend")
    # "flash3" and "torch" are the reference's cached-path modes (nomas_cpt.py:771-838); both run
    # with flash3's semantics here (padded text queries give zero rows, the cache mask always
    # applies), and None selects them too.
    if attn_mode not in (None, "flash3", "torch"):
        raise ValueError(f"Unsupported attn_mode for KV cache: {attn_mode}")
    if seg_ar_attention_backend == "flex" and torch.is_grad_enabled():
        raise RuntimeError("Flex cached attention requires no-grad inference")
    if sparse_context is not None:
        raise NotImplementedError("b200 cached attention: sparse_context routing is not implemented")
    intra = bool(cache_txt and intra_seg_vid_windows is not None and len(intra_seg_vid_windows) > 0
                 and intra_seg_txt_offsets is not None and any(o is not None for o in intra_seg_txt_offsets))
    if intra and attn_mode != "flash3":
        raise RuntimeError(
            "intra_segment_action_mask cache payload requires attn_mode='flash3', "
            f"got {attn_mode!r}")
    swa_commit = bool(update_cache and "swa_capacity" in kv_cache)
    if swa_commit and kv_cache.get("swa_sampling", "recent") in _swa.ARCHIVED_SAMPLINGS:
        raise NotImplementedError("b200 cached attention: archived SWA history sampling is not implemented")

    get_state, info = _STATE["get_state"], _STATE["info"]
    is_sp = bool(get_state())
    sp_group = info.sp_group

    img_q, txt_q = q
    img_k, txt_k = k
    img_v, txt_v = v
    img_q, txt_q, img_k, txt_k, img_v, txt_v = (
        _kernel_layout(x) for x in (img_q, txt_q, img_k, txt_k, img_v, txt_v))
    img_output_dtype = img_q.dtype
    txt_output_dtype = txt_q.dtype

    storage_format = kvc.cache_format(kv_cache)
    if storage_format == "qvg":
        raise ValueError("QVG requires single-slot dense Flex segment attention (not built for b200)")
    compressed = storage_format in ("int8", kvc.FP8_FORMAT)
    cache_shape, cache_device, cache_dtype = kvc.cache_geometry(kv_cache)
    if kv_cache["k"].dtype != kv_cache["v"].dtype:
        raise RuntimeError("KV cache K/V dtype mismatch")
    if kv_cache["k"].device != kv_cache["v"].device:
        raise RuntimeError("KV cache K/V device mismatch")
    if (compressed or "swa_capacity" in kv_cache) and torch.is_grad_enabled():
        raise ValueError("Compressed KV/SWA requires no-grad inference")
    if img_q.device != cache_device or txt_q.device != cache_device:
        raise RuntimeError(
            "Current Q and KV cache must be on the same device: "
            f"img_q={img_q.device}, txt_q={txt_q.device}, cache={cache_device}")
    _lib.require_device(img_q)
    _lib.require_same_device(cache_device, "Current Q/K/V, masks and KV cache", img_k, img_v, txt_k, txt_v,
                             text_mask, cache_mask, kv_cache.get("history_rows"),
                             *(kv_cache[n] for n in ("k_scale", "v_scale") if torch.is_tensor(kv_cache.get(n))))

    from . import communications as comm

    o_send = None
    exchange = None
    if is_sp:
        if sp_metadata is None:
            sp_metadata = comm.prepare_sp_communication(img_q.shape[1], img_q.shape[2], img_q.device, sp_group)
        if (comm.peer_exchange_enabled(sp_metadata.sequence_lengths, img_q.shape[2])
                and img_q.dtype == torch.bfloat16 and img_k.dtype == torch.bfloat16 and img_v.dtype == torch.bfloat16):
            exchange = comm.peer_exchange(sp_group, img_q.shape[0], img_q.shape[1], img_q.shape[2], txt_q.shape[1],
                                          img_q.device)
            img_q, img_k, img_v = exchange.push_qkv(img_q, img_k, img_v)
        else:
            img_q, img_k, img_v = comm.all_to_all_qkv(
                img_q, img_k, img_v, group=sp_group, sequence_lengths=sp_metadata.sequence_lengths)
        if txt_q.shape[2] != img_q.shape[2]:
            shard = img_q.shape[2]
            start_h = info.rank_within_spgroup * shard
            txt_q = txt_q[:, :, start_h:start_h + shard, :]
            txt_k = txt_k[:, :, start_h:start_h + shard, :]
            txt_v = txt_v[:, :, start_h:start_h + shard, :]

    # Kernel dtype is bf16 for every storage format (cache dtype for a bf16 cache).
    img_q, txt_q, img_k, txt_k, img_v, txt_v = (
        x if x.dtype == torch.bfloat16 else x.to(torch.bfloat16)
        for x in (img_q, txt_q, img_k, txt_k, img_v, txt_v))
    if not compressed and cache_dtype != torch.bfloat16:
        raise RuntimeError(f"b200 cached attention requires a bf16 cache, got {cache_dtype}")

    B = img_q.shape[0]
    img_len = img_k.shape[1]
    txt_len = txt_k.shape[1]
    H, D = img_q.shape[2], img_q.shape[3]
    # No text mask means every text token is valid: the kernels read a NULL mask that way, so
    # no all-true mask is built per call.
    cur_txt_mask = text_mask.bool() if text_mask is not None else None

    history_batch = kv_cache["k"].shape[0]
    if history_batch != B:
        if update_cache:
            raise ValueError(
                "KV-cache batch mismatch during update: "
                f"current={B}, cache={history_batch}. "
                "Read-only history broadcasting is supported, cache writes are not.")
        if history_batch != 1:
            raise ValueError(
                "KV-cache batch mismatch: "
                f"current={B}, cache={history_batch}; only a single canonical "
                "history slot can be broadcast.")
    if cache_valid_len < 0 or cache_valid_len > cache_shape[1]:
        raise ValueError("Invalid KV valid length")

    if swa_commit:
        if not cache_txt or cache_mask is None:
            raise ValueError("SWA requires a masked segment-AR cache write")
        _swa.check_dense_record(kv_cache, cache_valid_len, img_len, tokens_per_frame)

    # ---- cache write (validated before either payload is touched)
    # A window ring cache is written after the attention has staged its history (the slot a new
    # frame takes may hold the oldest frame this call still attends).
    window = kv_cache.get("window")
    if update_cache and "history_rows" in kv_cache and window is None:
        raise NotImplementedError("a ring cache without its SinkWindowKVCache cannot be written")
    if update_cache and window is not None and cache_txt and txt_k.shape[1] > 0:
        raise NotImplementedError("window caches hold whole image frames; pass cache_txt=False")
    if swa_commit and kv_cache.get("staged") is not None:
        raise NotImplementedError("a decoded mirror is not kept for bounded (SWA) histories: their commit "
                                  "moves history rows")
    mirror_rows = 0   # rows written before the attention, decoded into the cache's mirror after it
    if update_cache and window is None and not swa_commit:
        seg_k = [img_k, txt_k] if cache_txt else [img_k]
        seg_v = [img_v, txt_v] if cache_txt else [img_v]
        write_tokens = sum(t.shape[1] for t in seg_k)
        new_end = cache_valid_len + write_tokens
        if new_end > cache_shape[1]:
            raise ValueError("KV pair shape, capacity, dtype, or device mismatch")
        if compressed:
            # with a decoded mirror the attention stages this call's keys into the mirror rows
            # this write covers, so their decode runs after the attention
            mirror_rows = write_tokens if kv_cache.get("staged") is not None else 0
            kvc.quantize_kv_segments_into(kv_cache, [t.detach() for t in seg_k], [t.detach() for t in seg_v],
                                          cache_valid_len, assume_finite=_assume_finite(), decode=mirror_rows == 0)
        else:
            off = cache_valid_len
            for tk, tv in zip(seg_k, seg_v):
                kv_cache["k"][:, off:off + tk.shape[1]] = tk.detach()
                kv_cache["v"][:, off:off + tv.shape[1]] = tv.detach()
                off += tk.shape[1]
        if cache_mask is not None:
            if cache_txt and cur_txt_mask is not None:
                cache_mask[:, cache_valid_len:cache_valid_len + img_len] = True
                cache_mask[:, cache_valid_len + img_len:new_end] = cur_txt_mask
            else:
                cache_mask[:, cache_valid_len:new_end] = True
        stats["writes"] += 1

    # A sink + sliding-window ring cache (window.SinkWindowKVCache.view) carries the row map of
    # its history; its cache_mask, if given, is indexed by cache row.
    hist_rows = kv_cache.get("history_rows")
    if hist_rows is not None:
        if hist_rows.numel() != cache_valid_len:
            raise ValueError("cache_valid_len must equal the window cache's history length")
        # A window's own maps index its slots by construction; a map supplied without its window
        # is checked once (one host sync), since the staging kernel reads the rows it names.
        if window is None and hist_rows.numel() and (int(hist_rows.min()) < 0 or int(hist_rows.max()) >= cache_shape[1]):
            raise ValueError("history_rows must name rows of the cache")
        history_mask = cache_mask if (cache_mask is not None and cache_valid_len > 0) else None
    else:
        history_mask = cache_mask[:, :cache_valid_len] if (cache_mask is not None and cache_valid_len > 0) else None
    attend_txt = bool(cache_txt or update_cache)
    group_tokens = int(chunk_causal_frames) * int(tokens_per_frame) if chunk_causal_frames else 0

    out_img_strides = None
    if is_sp:
        o_send, out_img_strides = comm.o_send_buffer(
            B, sp_metadata.sequence_lengths, H, D, img_q.device)
    if intra:
        from .intra_seg import intra_segment_attention
        plain = o_send if (o_send is not None and out_img_strides is None) else _new_out(B, img_len, H, D, img_q.device)
        out_txt = _new_out(B, txt_len, H, D, img_q.device)
        intra_segment_attention(
            img_q, img_k, img_v, txt_q, txt_k, txt_v, kv_cache, cache_valid_len,
            offsets_per_sample=intra_seg_txt_offsets, windows=intra_seg_vid_windows,
            tokens_per_frame=tokens_per_frame, history_mask=history_mask, text_mask=cur_txt_mask,
            hist_rows=hist_rows, group_tokens=group_tokens, out_img=plain, out_txt=out_txt)
        if o_send is not None and out_img_strides is not None:
            comm.fill_o_send(o_send, plain)
        out_img = o_send if o_send is not None else plain
    else:
        out_img, out_txt = cached_attention_local(
            img_q, img_k, img_v, txt_q, txt_k, txt_v, kv_cache, cache_valid_len,
            history_mask=history_mask, text_mask=cur_txt_mask, attend_txt=attend_txt,
            group_tokens=group_tokens, out_img=o_send, out_img_strides=out_img_strides, hist_rows=hist_rows)
    stats["calls"] += 1
    if mirror_rows:
        kvc.refresh_decoded(kv_cache, cache_valid_len, mirror_rows)
    if swa_commit:
        # the bounded history is committed after the attention has read the old rows
        write_mask = torch.ones(B, img_len + txt_len, dtype=torch.bool, device=img_q.device)
        if cur_txt_mask is not None:
            write_mask[:, img_len:] = cur_txt_mask
        _swa.append_dense_record(kv_cache, cache_valid_len, img_len, txt_len, tokens_per_frame)
        _swa.commit_window(kv_cache, cache_mask, [img_k.detach(), txt_k.detach()], [img_v.detach(), txt_v.detach()],
                           write_mask, cache_valid_len, assume_finite=_assume_finite())
        stats["writes"] += 1
    if update_cache and window is not None:
        window.append(img_k.detach(), img_v.detach(), assume_finite=_assume_finite())
        stats["writes"] += 1

    if is_sp and exchange is not None:
        img_attn, txt_attn = exchange.push_o(o_send, out_txt)
    elif is_sp:
        img_attn = comm.all_to_all_o(o_send, group=sp_group, batch=B,
                                     sequence_lengths=sp_metadata.sequence_lengths, heads_local=H, dim=D)
        txt_attn = comm.all_gather(out_txt, dim=2, group=sp_group, sizes=sp_metadata.head_sizes)
    else:
        img_attn, txt_attn = out_img, out_txt

    if img_attn.dtype != img_output_dtype:
        img_attn = img_attn.to(dtype=img_output_dtype)
    if txt_attn.dtype != txt_output_dtype:
        txt_attn = txt_attn.to(dtype=txt_output_dtype)
    img_attn = img_attn.reshape(img_attn.size(0), img_attn.size(1), img_attn.size(2) * img_attn.size(3))
    txt_attn = txt_attn.reshape(txt_attn.size(0), txt_attn.size(1), txt_attn.size(2) * txt_attn.size(3))
    return img_attn, txt_attn
