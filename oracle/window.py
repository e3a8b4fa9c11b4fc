"""Sink + sliding-window history selection restated — test infrastructure only.

``slide(cache_rows, frames, sink, keep, T)`` restates the memmove of
``SelfForcingTrainingPipeline._slide_kv_cache``
(hymm/models/self_forcing/causal_training_pipeline.py:203-236): keep the first
``sink`` frames, move the last ``keep`` frames right after them, zero the rest.
``visible_frames`` gives the frame order the attention sees after that eviction.
"""
from __future__ import annotations

import torch


def slide(k: torch.Tensor, frames: int, sink: int, keep: int, T: int):
    """Apply the reference eviction to a [B, cap, H, D] cache; returns (k_after, new_count)."""
    k = k.clone()
    sink_tokens, keep_tokens, valid = sink * T, keep * T, frames * T
    src_start = valid - keep_tokens
    if src_start <= sink_tokens:
        return k, frames
    k[:, sink_tokens:sink_tokens + keep_tokens] = k[:, src_start:valid].clone()
    k[:, sink_tokens + keep_tokens:valid] = 0
    return k, sink + keep


def visible_frames(frames: int, sink: int, keep: int):
    """Temporal frame indices attended after eviction: sink frames, then the last ``keep``."""
    if frames - keep <= sink:
        return list(range(frames))
    return list(range(sink)) + list(range(frames - keep, frames))
