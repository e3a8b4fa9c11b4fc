"""Ulysses sequence-parallel exchange for the cached attention (B200 / NCCL).

Mirrors ``hymm/distributed/communications.py`` (``prepare_sp_communication`` :24-43,
``all_to_all_4D`` :260-267 / ``_all_to_all_4D`` :66-200, ``all_to_all_qkv`` :270-280,
``all_gather`` :410-421) with the same names, layouts and errors.  The difference is
the data movement around the collectives: the reference builds each send buffer with
cat + reshape + transpose + contiguous and unpacks with more copies; here one pack
kernel writes the send buffer directly from the (strided) inputs, the Q/K/V receive
buffer is consumed in place through strided views, and the cached attention writes
its image output straight into the O send buffer (``o_send_buffer``), so the head->
sequence direction costs one all_to_all_single plus one unpack kernel.

The exchange itself is ``torch.distributed.all_to_all_single`` (NCCL over NVLink on
B200).  ``exchange`` is the bare collective step; the pack / unpack kernels are CUDA
only, and the CPU process-group tests drive ``exchange`` with host-built buffers.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Tuple

import torch
import torch.distributed as dist

from . import _lib


@dataclass(frozen=True)
class SPCommunicationMetadata:
    """Per-rank sizes of one sequence-parallel model forward: ``sequence_lengths[r]`` image tokens
    held by rank r before the sequence->head exchange, ``head_sizes[r]`` heads held after it.
    The type and its two field names are what the reference's block passes as ``sp_metadata``
    and reads back (hymm/distributed/communications.py:16-21)."""

    sequence_lengths: Tuple[int, ...]
    head_sizes: Tuple[int, ...]


def prepare_sp_communication(local_sequence_length, heads, device, group):
    """Gather every rank's (tokens, heads) once per forward so the per-layer exchanges need no
    size collectives (the reference's helper of the same name, communications.py:24-43).  The
    table crosses to the host once; heads must agree across ranks and divide by the group size,
    otherwise ValueError with the reference's messages."""
    ranks = dist.get_world_size(group)
    mine = torch.tensor([local_sequence_length, heads], dtype=torch.int64, device=device).unsqueeze(0)
    table = mine
    if ranks > 1:
        table = mine.new_empty((ranks, 2))
        dist.all_gather_into_tensor(table, mine, group=group)
    per_rank = [tuple(pair) for pair in table.cpu().tolist()]
    tokens = tuple(t for t, _ in per_rank)
    if min(tokens) < 0:
        raise ValueError("SP sequence lengths must be nonnegative")
    if {h for _, h in per_rank} != {heads} or heads <= 0 or heads % ranks != 0:
        raise ValueError("SP ranks require identical head counts divisible by SP size")
    return SPCommunicationMetadata(tokens, (heads // ranks,) * ranks)


def _validate_sizes(sizes, world_size):
    """Per-rank sizes as a tuple of nonnegative Python ints, one per rank, else ValueError with the
    reference's message."""
    out = tuple(sizes)
    well_formed = len(out) == world_size and all(type(n) is int and n >= 0 for n in out)
    if not well_formed:
        raise ValueError("Expected one nonnegative Python integer size per process-group rank")
    return out


def exchange(send: torch.Tensor, group) -> torch.Tensor:
    """The collective step: equal-split all_to_all_single along dim 0 (P blocks)."""
    world = dist.get_world_size(group)
    if send.shape[0] != world:
        raise ValueError("send buffer's leading dimension must equal the SP world size")
    if world == 1:
        return send
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    return recv


def _legacy_lengths(length, world_size):
    chunk = (length + world_size - 1) // world_size
    return tuple(min(chunk, max(0, length - rank * chunk)) for rank in range(world_size))


def all_to_all_qkv(q, k, v, group, sequence_lengths=None):
    """Sequence-sharded [B, Ls, H, D] Q/K/V -> head-sharded [B, L, H/P, D], one collective.

    Returns strided views into the receive buffer when every rank holds the same number
    of tokens (the common case), compact tensors otherwise."""
    if any(t.shape != q.shape or t.dtype != q.dtype or t.device != q.device for t in (k, v)):
        raise ValueError("Fused QKV all-to-all requires identical shapes, dtypes and devices")
    if q.ndim != 4 or q.shape[0] == 0:
        raise ValueError("Fused QKV all-to-all requires nonempty-batch [B,S,H,D] tensors")
    return _seq_to_heads((q, k, v), group, sequence_lengths)


def _seq_to_heads(tensors, group, sequence_lengths):
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    x0 = tensors[0]
    B, Ls, H, D = x0.shape
    if sequence_lengths is None:
        sizes = torch.empty(world, dtype=torch.int64, device=x0.device)
        dist.all_gather_into_tensor(sizes, torch.tensor([Ls], dtype=torch.int64, device=x0.device), group=group)
        sequence_lengths = tuple(sizes.tolist())
    sequence_lengths = _validate_sizes(sequence_lengths, world)
    if Ls != sequence_lengths[rank]:
        raise ValueError("Local sequence length does not match SP metadata")
    if H % world:
        raise ValueError(f"Invalid Head size: {H}, which should be divisible by spsize {world}")
    Hp = H // world
    Ls_max = max(sequence_lengths)
    total = sum(sequence_lengths)
    n = len(tensors)
    if total == 0:
        return tuple(x0.new_empty((B, 0, Hp, D)) for _ in tensors)
    tensors = tuple(t if t.dtype == torch.bfloat16 else t.to(torch.bfloat16) for t in tensors)
    send = torch.empty((world, Ls_max, n * B, Hp, D), dtype=torch.bfloat16, device=x0.device)
    lib = _lib.load()
    views = [_lib.bf16_view(t) for t in tensors]
    with torch.cuda.device(x0.device):
        _lib.check(lib.hyb_ulysses_pack_qkv(
            world, B, Ls, Ls_max, H, D, views[0],
            views[1] if n == 3 else None, views[2] if n == 3 else None,
            send.data_ptr(), _lib.stream_ptr(x0.device)), "ulysses pack")
    recv = exchange(send, group)                      # [P(src), Ls_max, nB, Hp, D]
    if any(length != Ls_max for length in sequence_lengths):
        recv = torch.cat([recv[src, :length] for src, length in enumerate(sequence_lengths)], dim=0)
    else:
        recv = recv.reshape(world * Ls_max, n * B, Hp, D)
    full = recv.permute(1, 0, 2, 3)                   # [nB, L, Hp, D] strided view
    out = tuple(full[i * B:(i + 1) * B] for i in range(n))
    return tuple(t if t.dtype == x.dtype else t.to(x.dtype) for t, x in zip(out, tensors))


def o_send_buffer(B, sequence_lengths, Hp, D, device):
    """Allocate the head->sequence send buffer [P, Hp, Ls_max, B, D] and the element strides
    (sb, st, sh, seg, sseg) with which the attention epilogue writes image row t of head h
    straight into it.  Needs equal per-rank lengths (else returns a plain [B, L, Hp, D]
    buffer that ``all_to_all_o`` packs with a kernel)."""
    P = len(sequence_lengths)
    Ls_max = max(sequence_lengths) if sequence_lengths else 0
    if all(length == Ls_max for length in sequence_lengths) and Ls_max > 0:
        buf = torch.empty((P, Hp, Ls_max, B, D), dtype=torch.bfloat16, device=device)
        # offset(b, t, h) = ((t // Ls) * Hp + h) * Ls * B * D + (t % Ls) * B * D + b * D
        strides = (D, B * D, Ls_max * B * D, Ls_max, Hp * Ls_max * B * D)
        return buf, strides
    total = sum(sequence_lengths)
    buf = torch.empty((B, total, Hp, D), dtype=torch.bfloat16, device=device)
    return buf, None



def fill_o_send(send, plain):
    """Copy a head-sharded output held plainly, [B, L, Hp, D], into the packed send buffer
    [P, Hp, Ls, B, D] of ``o_send_buffer`` (equal per-rank lengths, L = P * Ls)."""
    P, Hp, Ls, B, D = send.shape
    send.copy_(plain.view(B, P, Ls, Hp, D).permute(1, 3, 2, 0, 4))


def all_to_all_o(send, group, batch, sequence_lengths, heads_local, dim):
    """Head-sharded attention output -> sequence-sharded [B, Ls, H, D]."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    sequence_lengths = _validate_sizes(sequence_lengths, world)
    Ls_max = max(sequence_lengths)
    lib = _lib.load()
    dev = send.device
    if send.ndim == 4:  # [B, L, Hp, D]: pack into the send layout first
        packed = torch.empty((world, heads_local, Ls_max, batch, dim), dtype=torch.bfloat16, device=dev)
        lens = (ctypes.c_int32 * world)(*sequence_lengths)
        with torch.cuda.device(dev):
            _lib.check(lib.hyb_ulysses_pack_o(world, batch, lens, Ls_max, heads_local, dim,
                                              _lib.bf16_view(send), packed.data_ptr(),
                                              _lib.stream_ptr(dev)), "ulysses pack o")
        send = packed
    recv = exchange(send, group)                      # [P(src), Hp, Ls_max, B, D]
    Ls = sequence_lengths[rank]
    H = heads_local * world
    out = torch.empty((batch, Ls, H, dim), dtype=torch.bfloat16, device=dev)
    with torch.cuda.device(dev):
        _lib.check(lib.hyb_ulysses_unpack_o(world, batch, Ls, Ls_max, H, dim, recv.data_ptr(), out.data_ptr(),
                                            *out.stride()[:3], _lib.stream_ptr(dev)), "ulysses unpack")
    return out


def all_to_all_4D(input_: torch.Tensor, group, scatter_dim: int = 2, gather_dim: int = 1,
                  sequence_lengths=None):
    """Generic 4-D all-to-all (forward only), same layouts as the reference."""
    if input_.dim() != 4:
        raise ValueError(f"input must be 4D tensor, got {input_.dim()} and shape {input_.shape}")
    world = dist.get_world_size(group)
    if scatter_dim == 2 and gather_dim == 1:
        return _seq_to_heads((input_,), group, sequence_lengths)[0]
    if scatter_dim == 1 and gather_dim == 2:
        B, L, Hp, D = input_.shape
        if sequence_lengths is None:
            sequence_lengths = _legacy_lengths(L, world)
        sequence_lengths = _validate_sizes(sequence_lengths, world)
        if L != sum(sequence_lengths):
            raise ValueError("Full sequence length does not match SP metadata")
        x = input_ if input_.dtype == torch.bfloat16 else input_.to(torch.bfloat16)
        out = all_to_all_o(x, group, B, sequence_lengths, Hp, D)
        return out if out.dtype == input_.dtype else out.to(input_.dtype)
    raise RuntimeError("scatter_idx must be 1 or 2 and gather_idx must be 1 or 2")


def all_gather(input_: torch.Tensor, dim: int = 1, group=None, sizes=None):
    """Concatenate every rank's tensor along ``dim`` (uneven sizes padded, as the reference)."""
    dim = dim % input_.dim()
    world = dist.get_world_size(group)
    if sizes is None:
        local = torch.tensor([input_.shape[dim]], dtype=torch.int64, device=input_.device)
        all_sizes = torch.empty(world, dtype=torch.int64, device=input_.device)
        dist.all_gather_into_tensor(all_sizes, local, group=group)
        sizes = all_sizes.tolist()
    sizes = _validate_sizes(sizes, world)
    if input_.shape[dim] != sizes[dist.get_rank(group)]:
        raise ValueError("Local gather size does not match supplied metadata")
    if world == 1:
        return input_.contiguous()
    max_size = max(sizes)
    x = input_.movedim(dim, 0)
    if x.shape[0] < max_size:
        pad = torch.zeros((max_size - x.shape[0], *x.shape[1:]), dtype=x.dtype, device=x.device)
        x = torch.cat([x, pad], dim=0)
    x = x.contiguous()
    gathered = torch.empty((world * x.shape[0], *x.shape[1:]), dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(gathered, x, group=group)
    gathered = gathered.view(world, *x.shape)
    parts = [gathered[r, :sizes[r]] for r in range(world)]
    return torch.cat(parts, dim=0).movedim(0, dim).contiguous()


# ------------------------------------------------------------------------------------------
# Exchange over peer memory (CUDA IPC): replaces the three collectives of one Ulysses call.
# ------------------------------------------------------------------------------------------
class _DeviceArray:
    """__cuda_array_interface__ view of a raw device allocation (for torch.as_tensor)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


def _bf16_tensor(ptr: int, shape, device) -> torch.Tensor:
    return torch.as_tensor(_DeviceArray(ptr, shape, "<i2"), device=device).view(torch.bfloat16)


def require_same_on_every_rank(group, values, what: str, device=None) -> None:
    """Raise ValueError on every rank of ``group`` unless all ranks passed the same integers.

    The push kernels write into the other ranks' buffers with this rank's sizes, so ranks that
    disagree on a buffer size or a geometry would write past a peer's allocation (a device fault,
    where the reference's collectives fail with an error); this collective check runs before
    any buffer is allocated or written."""
    vals = [int(v) for v in values]
    n = len(vals)
    dev = torch.device(device) if device is not None else torch.device("cpu")
    mine = torch.tensor([n] + vals, dtype=torch.int64, device=dev)
    world = dist.get_world_size(group)
    counts = [torch.zeros(1, dtype=torch.int64, device=dev) for _ in range(world)]
    dist.all_gather(counts, mine[:1], group=group)
    if len({int(c.item()) for c in counts}) != 1:
        raise ValueError(f"{what}: ranks disagree on the number of sizes ({[int(c.item()) for c in counts]})")
    rows = [torch.zeros_like(mine) for _ in range(world)]
    dist.all_gather(rows, mine, group=group)
    table = [tuple(int(x) for x in r.tolist()[1:]) for r in rows]
    if len(set(table)) != 1:
        raise ValueError(f"{what}: ranks disagree on sizes / geometry: {table}")


class PeerBuffers:
    """Device buffers every rank of ``group`` maps with CUDA IPC, plus the flag arrays of the
    device barrier that ends each push kernel.  ``ptrs[i][r]`` is buffer i of rank r as mapped
    in this process; ``local[i]`` is this rank's own.  Every rank must request the same sizes
    (and pass the same ``geometry``): checked collectively first, ValueError on every rank."""

    def __init__(self, group, sizes, device, geometry=()):
        self.group = group
        self.P = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = torch.device(device)
        self.lib = lib = _lib.load()
        sizes = [max(int(n), 256) for n in sizes] + [256]   # last: the barrier flags int32[<= 64]
        require_same_on_every_rank(group, list(sizes) + [int(g) for g in geometry], "peer buffers", self.device)
        self.sizes = sizes
        self.local = []
        self._opened = []
        handles = bytearray()
        with torch.cuda.device(self.device):
            for nbytes in sizes:
                ptr = ctypes.c_void_p()
                h = (ctypes.c_uint8 * 64)()
                _lib.check(lib.hyb_peer_alloc(nbytes, ctypes.byref(ptr), h), "peer alloc")
                self.local.append(ptr.value)
                handles += bytes(h)
            mine = torch.tensor(list(handles), dtype=torch.uint8, device=self.device)
            every = torch.empty((self.P, mine.numel()), dtype=torch.uint8, device=self.device)
            dist.all_gather_into_tensor(every, mine, group=group)
            every = every.cpu().numpy()
            self.ptrs = [[0] * self.P for _ in sizes]
            for rr in range(self.P):
                for i in range(len(sizes)):
                    if rr == self.rank:
                        self.ptrs[i][rr] = self.local[i]
                        continue
                    peer = ctypes.c_void_p()
                    _lib.check(lib.hyb_peer_open(bytes(every[rr, 64 * i:64 * (i + 1)]), ctypes.byref(peer)),
                               "peer open")
                    self.ptrs[i][rr] = peer.value
                    self._opened.append(peer.value)
        self.state = torch.zeros(2, dtype=torch.int32, device=self.device)
        self.sync = _lib.PeerSync()
        for rr in range(self.P):
            self.sync.flags[rr] = self.ptrs[-1][rr]
        self.sync.state = self.state.data_ptr()
        self.sync.dev_status = _lib.device_status(self.device).data_ptr()
        # every rank has mapped every buffer before anyone writes into them
        torch.cuda.synchronize(self.device)
        dist.barrier(group=group)

    def table(self, i, offset: int = 0):
        """ctypes array of buffer i of every rank (+ a byte offset)."""
        return (ctypes.c_void_p * self.P)(*[p + offset for p in self.ptrs[i]])

    def close(self) -> None:
        torch.cuda.synchronize(self.device)
        for p in self._opened:
            self.lib.hyb_peer_close(p)
        for p in self.local:
            self.lib.hyb_peer_free(p)
        self._opened, self.local = [], []


class PeerExchange:
    """Ulysses exchange of one geometry (group, batch B, per-rank length Ls, heads H, text
    length Lt) over buffers that every rank maps with CUDA IPC.  ``push_qkv`` writes this rank's
    Q|K|V heads straight into every rank's receive buffer (the receive layout of
    ``all_to_all_qkv``; two buffers used alternately, so a rank that runs ahead never
    overwrites one a slower rank still reads) and ``push_o`` writes this rank's output heads
    and text rows straight into every rank's output buffers; each is one kernel ending in a
    device-side barrier.  Equal sequence lengths on every rank."""

    def __init__(self, group, B: int, Ls: int, H: int, Lt: int, device):
        P = dist.get_world_size(group)
        self.P, self.rank = P, dist.get_rank(group)
        self.B, self.Ls, self.H, self.Lt = B, Ls, H, Lt
        self.Hp = H // P
        self.device = torch.device(device)
        self.lib = _lib.load()
        Hp, D = self.Hp, 128
        recv_bytes = P * Ls * 3 * B * Hp * D * 2
        self.buf = PeerBuffers(group, [recv_bytes, recv_bytes, B * Ls * H * D * 2, B * Lt * H * D * 2], device,
                               geometry=(B, Ls, H, Lt))
        recv_shape = (P, Ls, 3 * B, Hp, D)
        self.recv = [_bf16_tensor(self.buf.local[0], recv_shape, self.device),
                     _bf16_tensor(self.buf.local[1], recv_shape, self.device)]
        self.out = _bf16_tensor(self.buf.local[2], (B, Ls, H, D), self.device)
        self.txt_out = _bf16_tensor(self.buf.local[3], (B, Lt, H, D), self.device) if Lt else None
        self.sync = self.buf.sync
        self._recv_tab = [self.buf.table(0), self.buf.table(1)]
        self._out_tab = self.buf.table(2)
        self._txt_tab = self.buf.table(3)
        self.calls = 0

    def push_qkv(self, q, k, v):
        """Sequence-sharded q, k, v [B, Ls, H, D] -> head-sharded [B, P*Ls, H/P, D] views."""
        cur = self.calls % 2
        self.calls += 1
        views = [_lib.bf16_view(t) for t in (q, k, v)]
        with torch.cuda.device(self.device):
            _lib.check(self.lib.hyb_ulysses_push_qkv(self.P, self.rank, self.B, self.Ls, self.H, 128,
                                                     *(ctypes.byref(x) for x in views), self._recv_tab[cur],
                                                     ctypes.byref(self.sync), _lib.stream_ptr(self.device)),
                       "ulysses push qkv")
        full = self.recv[cur].reshape(self.P * self.Ls, 3 * self.B, self.Hp, 128).permute(1, 0, 2, 3)
        return tuple(full[i * self.B:(i + 1) * self.B] for i in range(3))

    def push_o(self, o_send, out_txt):
        """This rank's heads (o_send [P, H/P, Ls, B, D], out_txt [B, Lt, H/P, D]) -> fresh
        [B, Ls, H, D] image and [B, Lt, H, D] text outputs of this rank."""
        txt_view = _lib.bf16_view(out_txt) if self.Lt else None
        with torch.cuda.device(self.device):
            _lib.check(self.lib.hyb_ulysses_push_o(self.P, self.rank, self.B, self.Ls, self.Lt, self.H, 128,
                                                   o_send.data_ptr(),
                                                   ctypes.byref(txt_view) if txt_view is not None else None,
                                                   self._out_tab, self._txt_tab, ctypes.byref(self.sync),
                                                   _lib.stream_ptr(self.device)), "ulysses push o")
        img = self.out.clone()
        txt = self.txt_out.clone() if self.Lt else out_txt.new_empty((self.B, 0, self.H, 128))
        return img, txt

    def close(self) -> None:
        self.buf.close()


_EXCHANGES: dict = {}


def peer_exchange(group, B, Ls, H, Lt, device):
    """The cached PeerExchange of this geometry (created collectively on first use)."""
    key = (id(group), dist.get_world_size(group), B, Ls, H, Lt, str(device))
    ex = _EXCHANGES.get(key)
    if ex is None:
        ex = PeerExchange(group, B, Ls, H, Lt, device)
        _EXCHANGES[key] = ex
    return ex


def release_peer_exchanges() -> None:
    """Unmap and free every exchange's buffers (before destroying the process group)."""
    for ex in _EXCHANGES.values():
        ex.close()
    _EXCHANGES.clear()


def peer_exchange_enabled(sequence_lengths, heads) -> bool:
    """Peer-memory exchange for equal per-rank lengths unless HYB_PEER_EXCHANGE=0."""
    import os
    if os.environ.get("HYB_PEER_EXCHANGE", "1") == "0":
        return False
    P = len(sequence_lengths)
    return 1 < P <= 64 and len(set(sequence_lengths)) == 1 and heads % P == 0
