"""Install the B200 cached attention into a running Hy-Nomas process.

Same pattern as the reactor's ``CacheStaging`` installer (reactor/hy_nomas_cache.py:76-100)
and the backend's patch points (reactor/hy_nomas_backend.py:53-56, :149-156): the module
attribute ``hymm.models.dit.nomas_cpt.causal_attention_with_cache_mp`` is replaced, so every
``MMDoubleStreamBlock.forward_with_cache`` (nomas_cpt.py:1398-1416) and the TP block
(modules/tensor_parallel.py:180) call the B200 path.  The replacement reads the reference's
own sequence-parallel state (``hymm.distributed.parallel_states``) and keeps the native
function for the modes this build does not implement (QVG storage, sparse routing, the
archived history samplings of the SWA cache, non-bf16 caches).  Intra-segment action masks
and the bounded ("recent") SWA history run on the B200 path.
"""
from __future__ import annotations

import functools

import torch

from . import attention as _att
from . import kv_cache as _kvc
from . import swa as _swa

_INSTALLED = {}


def _eligible(kv_cache, update_cache, sparse_context):
    fmt = _kvc.cache_format(kv_cache)
    if fmt not in ("none", "int8", _kvc.FP8_FORMAT):
        return False
    if fmt == "none" and kv_cache["k"].dtype != torch.bfloat16:
        return False
    if sparse_context is not None:
        return False
    if ("swa_capacity" in kv_cache and update_cache
            and kv_cache.get("swa_sampling", "recent") in _swa.ARCHIVED_SAMPLINGS):
        return False
    if not kv_cache["k"].is_cuda:
        return False
    return True


def install(native_module=None):
    """Patch ``native_module.causal_attention_with_cache_mp`` (default: the reference's
    ``hymm.models.dit.nomas_cpt``).  Returns the original function."""
    if native_module is None:
        import importlib
        native_module = importlib.import_module("hymm.models.dit.nomas_cpt")
    key = id(native_module)
    if key in _INSTALLED:
        return _INSTALLED[key][1]
    original = native_module.causal_attention_with_cache_mp
    _att.set_parallel_state_provider(native_module.get_sequence_parallel_state, native_module.nccl_info)

    @functools.wraps(original)
    def patched(q, k, v, kv_cache, cache_valid_len=0, attn_mode=None, text_mask=None,
                update_cache=False, cache_txt=True, cache_mask=None, intra_seg_txt_offsets=None,
                intra_seg_vid_windows=None, tokens_per_frame=0, seg_ar_attention_backend="magi",
                sparse_context=None, sp_metadata=None, attention_metadata=None, **extra):
        if not _eligible(kv_cache, update_cache, sparse_context) or attn_mode == "torch":
            if extra.get("chunk_causal_frames"):
                raise NotImplementedError(
                    "chunk_causal_frames (frame-level block-causal chunks) runs on the b200 path only; "
                    "this call would fall back to the reference, which has no such mask")
            patched.stats["fallbacks"] += 1
            # The reactor's CacheStaging (reactor/hy_nomas_cache.py:192-209), which may sit behind
            # this patch, takes the older signature without the last two arguments.
            newer = {}
            if sp_metadata is not None:
                newer["sp_metadata"] = sp_metadata
            if attention_metadata is not None:
                newer["attention_metadata"] = attention_metadata
            return original(q, k, v, kv_cache, cache_valid_len, attn_mode, text_mask, update_cache,
                            cache_txt, cache_mask, intra_seg_txt_offsets, intra_seg_vid_windows,
                            tokens_per_frame, seg_ar_attention_backend, sparse_context, **newer)
        patched.stats["calls"] += 1
        return _att.causal_attention_with_cache_mp(
            q, k, v, kv_cache, cache_valid_len, attn_mode, text_mask, update_cache, cache_txt,
            cache_mask, intra_seg_txt_offsets, intra_seg_vid_windows, tokens_per_frame,
            "b200" if seg_ar_attention_backend not in ("magi", "flex", "b200") else seg_ar_attention_backend,
            sparse_context, sp_metadata, attention_metadata, **extra)

    patched.stats = {"calls": 0, "fallbacks": 0}
    patched.original = original
    native_module.causal_attention_with_cache_mp = patched
    _INSTALLED[key] = (native_module, original)
    return original


def uninstall(native_module=None):
    if native_module is None:
        import importlib
        native_module = importlib.import_module("hymm.models.dit.nomas_cpt")
    entry = _INSTALLED.pop(id(native_module), None)
    if entry is not None:
        native_module.causal_attention_with_cache_mp = entry[1]
