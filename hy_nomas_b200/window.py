"""Sink + sliding-window KV history for long rollouts, stored as a frame ring.

The reference keeps the first ``sink_frames`` frames and the last ``cache_keep_frames``
frames by copying the kept frames over the evicted ones after every block
(``SelfForcingTrainingPipeline._slide_kv_cache`` / ``_gradual_evict_cache``,
hymm/models/self_forcing/causal_training_pipeline.py:178-236: a ``.clone()`` memmove of
the whole window per layer, then zero fill), and the bounded segment cache does the same
for its budget (``commit_window``, hymm/models/dit/modules/swa_cache.py:91-138).

Here nothing moves.  The cache holds ``sink + keep`` frame slots: sink frames in slots
[0, sink), window frames in slots sink + (f - sink) % keep, so appending frame f overwrites
the slot of the frame that leaves the window (quantise-on-write straight into that slot,
one kernel per append).  The attention reads the history in temporal order through a
row map (``history_rows``: composed history position -> cache row) that the staging
kernel follows; the maps of every ring rotation are built once, on the device.
The visible frames after each append are the reference's: sink frames, then the last
``keep`` frames (oracle/window.py restates the reference slide for the tests).

With ``decoded=True`` (quantised storage) each appended frame is also decoded once into a
head-major mirror of the slots (bf16 K, fp16 V: the values the attention's staging pass would
produce from the codes), and the attention reads the history from the mirror in slot order
instead of decoding the whole window on every call (the reference decodes the whole cache per
call, nomas_cpt.py:529-531; a 1-frame rollout step then re-decodes 33 unchanged frames).  The
slot order is not the temporal order, which the attention does not need: it is a sum over the
set of visible keys.  Memory: the mirror holds 4 bytes per cached value next to the cache's
~2 (e4m3 K and V + scales), plus a tail of ``tail_rows`` rows where each call stages its own
keys.
"""
from __future__ import annotations

import torch

from . import kv_cache as _kvc


class SinkWindowKVCache:
    """History of one attention layer (one rank's heads): ``sink_frames`` first frames plus a
    sliding window of the last ``keep_frames`` frames, ``tokens_per_frame`` tokens each."""

    def __init__(self, batch: int, heads: int, tokens_per_frame: int, sink_frames: int, keep_frames: int, *,
                 head_dim: int = 128, storage_format: str = "fp8_e4m3", device=None, decoded: bool = False,
                 tail_rows: int | None = None):
        if tokens_per_frame <= 0 or sink_frames < 0 or keep_frames <= 0:
            raise ValueError("window cache needs tokens_per_frame > 0, sink_frames >= 0, keep_frames > 0")
        self.B, self.H, self.D = batch, heads, head_dim
        self.T, self.sink, self.keep = tokens_per_frame, sink_frames, keep_frames
        self.slots = sink_frames + keep_frames
        self.device = torch.device(device) if device is not None else torch.device("cuda")
        cap = self.slots * tokens_per_frame
        if storage_format == "fp8_e4m3":
            self.cache = _kvc.make_fp8_kv_block(batch, cap, heads, head_dim, device=self.device)
        elif storage_format == "int8":
            self.cache = _kvc.make_int8_kv_block(batch, cap, heads, head_dim, device=self.device)
        elif storage_format == "bf16":
            self.cache = {"k": torch.zeros(batch, cap, heads, head_dim, dtype=torch.bfloat16, device=self.device),
                          "v": torch.zeros(batch, cap, heads, head_dim, dtype=torch.bfloat16, device=self.device)}
        else:
            raise ValueError(f"unknown storage format {storage_format!r}")
        self.storage_format = storage_format
        self.frames = 0            # frames appended so far (temporal count)
        self.mirror = None
        if decoded:
            if storage_format == "bf16":
                raise ValueError("decoded=True mirrors a quantised cache (fp8_e4m3 or int8)")
            tail = tokens_per_frame + 256 if tail_rows is None else int(tail_rows)
            self.pitch = cap + tail  # rows per (batch, head): the slots, then the call's own keys
            self.mirror = (torch.empty(batch, heads, self.pitch, head_dim, dtype=torch.bfloat16, device=self.device),
                           torch.empty(batch, heads, self.pitch, head_dim, dtype=torch.float16, device=self.device))
        # Row maps, built on the device without a host sync: before the window wraps, frame f
        # sits in slot f (a prefix of the identity); once it wraps, rotation r = (frames - sink)
        # % keep puts the oldest visible window frame in slot sink + r.
        T = tokens_per_frame
        self._identity = torch.arange(cap, dtype=torch.int32, device=self.device)
        base = torch.arange(T, dtype=torch.int32, device=self.device)
        j = torch.arange(keep_frames, dtype=torch.int32, device=self.device)
        self._ring = []
        for r in range(keep_frames):
            slots = (j + r) % keep_frames + sink_frames
            win_rows = (slots[:, None] * T + base[None, :]).reshape(-1)
            self._ring.append(torch.cat([self._identity[:sink_frames * T], win_rows]).contiguous())

    # ------------------------------------------------------------------ geometry
    def slot_of(self, frame: int) -> int:
        if frame < self.sink:
            return frame
        return self.sink + (frame - self.sink) % self.keep

    def history_frames(self):
        """Temporal indices of the frames the next attention sees, in order."""
        if self.frames <= self.slots:
            return list(range(self.frames))
        return list(range(self.sink)) + list(range(self.frames - self.keep, self.frames))

    @property
    def valid_len(self) -> int:
        return min(self.frames, self.slots) * self.T

    def history_rows(self) -> torch.Tensor:
        """int32 [valid_len] on the device: cache row of composed history position t."""
        if self.frames <= self.slots:
            return self._identity[:self.frames * self.T]
        return self._ring[(self.frames - self.sink) % self.keep]

    def view(self) -> dict:
        """The ``kv_cache`` argument of ``causal_attention_with_cache_mp`` for the next call
        (with ``cache_valid_len=self.valid_len``).  With ``update_cache=True`` (and
        ``cache_txt=False``) the call appends the chunk's image frames after its attention."""
        d = dict(self.cache)
        d["history_rows"] = self.history_rows()
        d["window"] = self          # update_cache=True appends the chunk's frames here
        if self.mirror is not None:
            d["staged"] = (self.mirror[0], self.mirror[1], self.pitch)   # history rows in slot order
        return d

    # ------------------------------------------------------------------ writes
    def append(self, k: torch.Tensor, v: torch.Tensor, *, assume_finite: bool = False) -> None:
        """Quantise-on-write of whole frames k/v [B, n*T, H, D] into their ring slots; the frames
        that leave the window are overwritten in place."""
        if k.shape != v.shape or k.ndim != 4 or k.shape[0] != self.B or k.shape[2] != self.H or k.shape[3] != self.D:
            raise ValueError("window append: k/v must be [B, n*T, H, D] of the cache's geometry")
        L = k.shape[1]
        if L % self.T:
            raise ValueError("window append: whole frames only (length a multiple of tokens_per_frame)")
        for i in range(L // self.T):
            slot = self.slot_of(self.frames)
            ks = k[:, i * self.T:(i + 1) * self.T]
            vs = v[:, i * self.T:(i + 1) * self.T]
            if self.storage_format == "bf16":
                self.cache["k"][:, slot * self.T:(slot + 1) * self.T] = ks
                self.cache["v"][:, slot * self.T:(slot + 1) * self.T] = vs
            else:
                _kvc.quantize_kv_pair_into(self.cache, ks, vs, slot * self.T, assume_finite=assume_finite)
                if self.mirror is not None:
                    self._decode_slot(slot)
            self.frames += 1

    def _decode_slot(self, slot: int) -> None:
        """Decode the codes of one slot into its rows of the mirror."""
        from . import _lib
        lib = _lib.load()
        code = _lib.HYB_FMT_INT8 if self.storage_format == "int8" else _lib.HYB_FMT_E4M3
        rows = slice(slot * self.T, (slot + 1) * self.T)
        src_k = _lib.coded_view(self.cache["k"][:, rows], self.cache["k_scale"][:, rows], code)
        src_v = _lib.coded_view(self.cache["v"][:, rows], self.cache["v_scale"][:, rows], code)
        with torch.cuda.device(self.device):
            _lib.check(lib.hyb_decode_rows(self.B, self.T, self.H, self.D, src_k, src_v, self.mirror[0].data_ptr(),
                                           self.mirror[1].data_ptr(), self.pitch, slot * self.T,
                                           _lib.stream_ptr(self.device)), "window decode")
