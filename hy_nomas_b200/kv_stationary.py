"""KV-stationary sequence parallelism for decode-size chunks over a sequence-sharded cache.

The reference's long rollout attends one latent frame (about 1.5k queries) to a sink +
sliding-window history of tens of thousands of keys.  Its sequence-parallel ring
(``DynamicRingAttention.forward``, hymm/models/dit/modules/attention/dynamic_ring_attention.py:
115-286) passes every rank's K/V block around the ring: P - 1 hops of the whole window per step.
Here the K/V stays where it was written.  Rank r holds its own sequence slice of every frame (a
``SinkWindowKVCache`` with tokens_per_frame / P tokens per frame, appended from the rank's own
shard of each new frame, so the cache write needs no exchange), and what moves is small:

  1. Q all-gather: every rank pushes its Q slice into every rank's full-Q buffer (one push
     kernel over peer memory ending in a device barrier; two buffers used alternately, as the
     Ulysses exchange does).
  2. Local attention of every query of the frame to the keys this rank holds (its history
     slices through the window's row map, its slice of the current frame, the text keys on rank
     0 only).  The attention epilogue writes each row's fp32 partial (O / l) and LSE straight
     into the buffers of the rank that owns the row (``hyb_part_scatter``: the kernel's stores
     go to peer memory; a text row goes to every rank).
  3. A device barrier; each owner merges the P x slices partials of its rows by log-sum-exp
     (``hyb_merge_partials``, the merge of dynamic_ring_attention.py:86-105).

Per rank and step at P = 8 on BASELINE config 5 (1,560 queries, 24 heads, 53,040 visible keys):
8.4 MB of Q in and 16.8 MB of fp32 partials out, against 7 x 25 MB of e4m3 K/V for the ring.
Heads need not divide by P (the Ulysses constraint, hymm/distributed/communications.py:41-42).
"""
from __future__ import annotations

import ctypes
import math

import torch
import torch.distributed as dist

from . import _lib
from .attention import Workspace, _assume_finite, cached_attention_local

_D = 128


def choose_slices(B: int, H: int, Lq: int, Lk: int, sms: int, fixed_tiles: float = 2.0) -> int:
    """Key slices per query pair for a partial-scatter launch (every pair gets the same count, so
    each owner merges a fixed number of partials): the count minimising the simulated makespan
    ceil(CTAs / sms) x (key tiles per slice + a fixed ~2 tiles per CTA), at least 4 tiles a slice."""
    pairs = B * H * ((Lq + 255) // 256)
    tiles = max(1, (Lk + 127) // 128)
    best, best_t = 1, math.inf
    for s in range(1, 17):
        if s > 1 and tiles / s < 4:
            break
        t = math.ceil(pairs * s / sms) * (math.ceil(tiles / s) + fixed_tiles)
        if t < best_t * 0.99:
            best, best_t = s, t
    return best


def _fp32_from(ptr: int, numel: int, device) -> torch.Tensor:
    from .communications import _DeviceArray
    return torch.as_tensor(_DeviceArray(ptr, (numel,), "<f4"), device=device)


class _Owners:
    """Partial buffers of every owner rank as seen from here, and the scatter descriptor."""

    def __init__(self, o_ptrs, lse_ptrs, ranks: int, rows: int, rank: int, slices: int, device):
        self.o_tab = torch.tensor(o_ptrs, dtype=torch.int64, device=device)
        self.lse_tab = torch.tensor(lse_ptrs, dtype=torch.int64, device=device)
        self.count = ranks * slices
        self.scatter = _lib.PartScatter(self.o_tab.data_ptr(), self.lse_tab.data_ptr(), ranks, rows, rank * slices,
                                        self.count, slices, 0)


def _merge(count, B, H, Ls, Lt, part_o, part_lse, out_img, out_txt, text_mask, device):
    lib = _lib.load()
    tm = text_mask.to(torch.bool).contiguous() if text_mask is not None else None
    with torch.cuda.device(device):
        _lib.check(lib.hyb_merge_partials(count, B, H, _D, Ls, Lt, part_o, part_lse,
                                          out_img.data_ptr(), *out_img.stride()[:3],
                                          _lib.ptr(out_txt) if Lt else None,
                                          *(out_txt.stride()[:3] if Lt else (0, 0, 0)),
                                          _lib.ptr(tm), tm.stride(0) if tm is not None else 0, None,
                                          _lib.stream_ptr(device)), "merge partials")


class KVStationaryAttention:
    """One geometry of the schedule on one rank of ``group`` (created collectively; buffers are
    reused across calls).  ``B`` must be 1 (the Q slice is pushed as one contiguous block);
    ``Ls`` tokens of each frame per rank, ``Lt`` text tokens (replicated on every rank), ``H``
    heads, history of at most ``hist_max`` tokens per rank."""

    def __init__(self, group, B: int, Ls: int, H: int, Lt: int, hist_max: int, device, *, sms: int | None = None):
        if B != 1:
            raise ValueError("KV-stationary attention pushes the Q slice as one block: batch 1 only")
        from .communications import PeerBuffers
        self.P = P = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.B, self.Ls, self.H, self.Lt = B, Ls, H, Lt
        self.device = dev = torch.device(device)
        self.lib = _lib.load()
        if sms is None:
            sms = torch.cuda.get_device_properties(dev).multi_processor_count
        self.slices = choose_slices(B, H, P * Ls + Lt, hist_max + Ls + Lt, sms)
        R = Ls + Lt
        count = P * self.slices
        q_bytes = B * P * Ls * H * _D * 2
        self.po_numel = count * B * H * R * _D
        self.pl_numel = count * B * H * R
        self.buf = PeerBuffers(group, [q_bytes, q_bytes, self.po_numel * 4, self.pl_numel * 4], dev,
                               geometry=(B, Ls, H, Lt, self.slices))
        from .communications import _bf16_tensor
        self.full_q = [_bf16_tensor(self.buf.local[i], (B, P * Ls, H, _D), dev) for i in (0, 1)]
        self._q_tab = [self.buf.table(i, offset=self.rank * Ls * H * _D * 2) for i in (0, 1)]
        self.owners = _Owners(self.buf.ptrs[2], self.buf.ptrs[3], P, Ls, self.rank, self.slices, dev)
        self.ws = Workspace()
        self.calls = 0

    def __call__(self, q, k, v, txt_q, txt_k, txt_v, window, *, text_mask=None, attend_txt=True,
                 update_cache=True, out_img=None, out_txt=None):
        """q, k, v: this rank's slice of the current frame, bf16 [1, Ls, H, 128]; txt_*: the text
        tokens [1, Lt, H, 128] (the same on every rank); ``window``: this rank's
        ``SinkWindowKVCache`` (tokens_per_frame = Ls).  Returns this rank's image rows
        [1, Ls, H, 128] and the text rows [1, Lt, H, 128]; with ``update_cache`` the rank's
        slice of the frame is appended to its window after the attention."""
        B, Ls, H, Lt, P, dev = self.B, self.Ls, self.H, self.Lt, self.P, self.device
        if q.shape != (B, Ls, H, _D) or k.shape != q.shape or v.shape != q.shape:
            raise ValueError(f"KV-stationary shard must be [{B}, {Ls}, {H}, {_D}]")
        if txt_q.shape != (B, Lt, H, _D):
            raise ValueError(f"text tokens must be [{B}, {Lt}, {H}, {_D}]")
        if window.T != Ls or window.H != H:
            raise ValueError("the window cache must hold this rank's slice (tokens_per_frame = Ls) of every head")
        _lib.require_same_device(dev, "KV-stationary tensors", q, k, v, txt_q, txt_k, txt_v, text_mask)
        cur = self.calls % 2
        self.calls += 1
        qc = q.contiguous()
        out_img = out_img if out_img is not None else torch.empty((B, Ls, H, _D), dtype=torch.bfloat16, device=dev)
        out_txt = out_txt if out_txt is not None else torch.empty((B, Lt, H, _D), dtype=torch.bfloat16, device=dev)
        with torch.cuda.device(dev):
            stream = _lib.stream_ptr(dev)
            _lib.check(self.lib.hyb_peer_push_bytes(P, self.rank, qc.data_ptr(), qc.numel() * 2, self._q_tab[cur],
                                                    ctypes.byref(self.buf.sync), stream), "KV-stationary Q push")
            cache = window.view()
            cached_attention_local(self.full_q[cur], k, v, txt_q, txt_k, txt_v, cache, window.valid_len,
                                   text_mask=text_mask, attend_txt=bool(attend_txt) and self.rank == 0,
                                   hist_rows=cache["history_rows"], workspace=self.ws, scatter=self.owners.scatter)
            _lib.check(self.lib.hyb_peer_barrier(P, self.rank, ctypes.byref(self.buf.sync), stream),
                       "KV-stationary partial barrier")
        _merge(self.owners.count, B, H, Ls, Lt, self.buf.local[2], self.buf.local[3], out_img, out_txt, text_mask, dev)
        if update_cache:
            # the drop-in's rule: without HYB_ASSUME_FINITE_KV=1 the reference's finite check
            # runs first (a host synchronisation)
            window.append(k, v, assume_finite=_assume_finite())
        return out_img, out_txt

    def close(self) -> None:
        self.buf.close()


def kv_stationary_emulated(q, k, v, txt_q, txt_k, txt_v, windows, *, text_mask=None, attend_txt=True,
                           update_cache=True, slices: int | None = None):
    """All ranks of the schedule in one process on one GPU (tests): ``windows[r]`` is rank r's
    sequence-sharded window cache; q/k/v the whole frame [B, T, H, 128] with rank r's slice
    rows [r T / P, (r + 1) T / P).  Every rank's attention scatters into owner buffers in
    local memory, then every owner merges.  Returns the image rows [B, T, H, 128] and the text
    rows [B, Lt, H, 128] (as merged by owner 0)."""
    P = len(windows)
    B, T, H, _ = q.shape
    Lt = txt_q.shape[1]
    if T % P:
        raise ValueError("the frame's tokens must split evenly over the ranks")
    Ls = T // P
    dev = q.device
    R = Ls + Lt
    hist_max = max(w.slots * w.T for w in windows)
    if slices is None:
        slices = choose_slices(B, H, T + Lt, hist_max + Ls + Lt, torch.cuda.get_device_properties(dev).multi_processor_count)
    count = P * slices
    part_o = [torch.empty(count * B * H * R * _D, dtype=torch.float32, device=dev) for _ in range(P)]
    part_lse = [torch.empty(count * B * H * R, dtype=torch.float32, device=dev) for _ in range(P)]
    owners = [_Owners([t.data_ptr() for t in part_o], [t.data_ptr() for t in part_lse], P, Ls, r, slices, dev)
              for r in range(P)]
    qf = q.contiguous()
    for r in range(P):
        sl = slice(r * Ls, (r + 1) * Ls)
        cache = windows[r].view()
        cached_attention_local(qf, k[:, sl], v[:, sl], txt_q, txt_k, txt_v, cache, windows[r].valid_len,
                               text_mask=text_mask, attend_txt=bool(attend_txt) and r == 0,
                               hist_rows=cache["history_rows"], scatter=owners[r].scatter)
    out_img = torch.empty((B, T, H, _D), dtype=torch.bfloat16, device=dev)
    out_txt = torch.empty((B, Lt, H, _D), dtype=torch.bfloat16, device=dev)
    for r in reversed(range(P)):   # owner 0 last: its text rows are the ones returned
        _merge(count, B, H, Ls, Lt, part_o[r].data_ptr(), part_lse[r].data_ptr(), out_img[:, r * Ls:(r + 1) * Ls],
               out_txt, text_mask, dev)
    if update_cache:
        for r in range(P):
            windows[r].append(k[:, r * Ls:(r + 1) * Ls], v[:, r * Ls:(r + 1) * Ls])
    torch.cuda.synchronize(dev)    # the owner tables and partial buffers are freed on return
    return out_img, out_txt
