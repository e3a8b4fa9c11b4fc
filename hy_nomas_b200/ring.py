"""Ring (KV-passing) sequence parallelism with frame-level causal masking.

The sequence of ``seq_len`` tokens is sharded over the P ranks of a group.  The default
layout is zig-zag: the sequence is cut into 2P near-equal chunks and rank r holds chunks r
and 2P-1-r (concatenated in that order), so that under the causal mask every rank does the
same work.  ``layout="contiguous"`` gives rank r the r-th of P chunks.

Each rank quantises its own K/V once into an e4m3 (or int8) block: codes and per-(token,
head) scales in one byte buffer, the message of one ring hop.  At step s rank r attends its
queries to the block of rank (r - s) mod P while NCCL moves the next block from rank r - 1
into the other half of a double buffer.  The transfer and the decode of the received block
into head-major bf16 tiles run on a side stream, overlapped with the current step's
attention on the caller's stream; the two streams are joined by events, with no host sync.
Every step is one attention launch whose epilogue merges its rows into a running fp32
output by log-sum-exp (the last step writes the bf16 output), so no separate merge pass
runs between steps.

Transport and merge follow the reference's ring (``DynamicRingAttention.forward``,
hymm/models/dit/modules/attention/dynamic_ring_attention.py:115-286: isend/irecv to
``(idx + 1) % P`` / from ``(idx - 1) % P``, double-buffered; ``flash_attn_fwd_out_correction``
/ ``_softmax_lse_correction`` merges :86-105).  The reference ring is non-causal and carries
bf16 K/V; the frame-level causal mask is the chunk-causal rule of
``create_magi_mp_causal_ranges`` (attention/magi_attn.py:290-309): query frame f sees key
frames <= f.  Blocks entirely in a query shard's future are not computed.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from . import kv_cache as _kvc

_FMT = {"fp8_e4m3": (_lib.HYB_FMT_E4M3, torch.float8_e4m3fn), "int8": (_lib.HYB_FMT_INT8, torch.int8)}
_D = 128


class RingPlan:
    """Token ownership of a ring over ``world`` ranks: per rank one or two contiguous segments
    of the global sequence, in increasing position order."""

    def __init__(self, seq_len: int, world: int, layout: str = "zigzag"):
        if seq_len < 0 or world <= 0:
            raise ValueError("ring plan needs seq_len >= 0 and world >= 1")
        if layout not in ("zigzag", "contiguous"):
            raise ValueError(f"unknown ring layout {layout!r}")
        self.seq_len, self.world, self.layout = seq_len, world, layout
        n = 2 * world if layout == "zigzag" else world
        # Chunks of at least 4 query pairs start on a 256-token boundary (one query pair of the
        # attention kernel), so that no pair holds rows of both of a rank's chunks: such a pair
        # would load the key range of its later rows for all of its rows.
        align = 256 if seq_len >= n * 1024 else 1
        bounds = [min(seq_len, ((i * seq_len) // n + align // 2) // align * align) for i in range(n)] + [seq_len]
        chunk = [(bounds[i], bounds[i + 1] - bounds[i]) for i in range(n)]
        if layout == "zigzag":
            self.segments = [(chunk[r], chunk[n - 1 - r]) for r in range(world)]
        else:
            self.segments = [(chunk[r], (bounds[r + 1], 0)) for r in range(world)]

    def length(self, rank: int) -> int:
        return sum(n for _, n in self.segments[rank])

    def max_length(self) -> int:
        return max(self.length(r) for r in range(self.world))

    def positions(self, rank: int):
        """(seg0_len, pos0, pos1) of the rank's tokens: token i is at pos0 + i for i < seg0_len,
        else at pos1 + (i - seg0_len)."""
        (p0, n0), (p1, _) = self.segments[rank]
        return n0, p0, p1

    def shard(self, x: torch.Tensor, rank: int, dim: int = 1) -> torch.Tensor:
        parts = [x.narrow(dim, p, n) for p, n in self.segments[rank] if n > 0]
        if not parts:
            return x.narrow(dim, 0, 0)
        return torch.cat(parts, dim) if len(parts) > 1 else parts[0]

    def unshard(self, shards, dim: int = 1) -> torch.Tensor:
        pieces = []
        for r, s in enumerate(shards):
            off = 0
            for p, n in self.segments[r]:
                if n > 0:
                    pieces.append((p, s.narrow(dim, off, n)))
                off += n
        pieces.sort(key=lambda t: t[0])
        return torch.cat([t for _, t in pieces], dim)

    def gather_chunks(self):
        """(position, length, owner rank, row in the owner's block) of every chunk, in position
        order: the table that lays the ranks' blocks out as the whole sequence."""
        chunks = []
        for r in range(self.world):
            off = 0
            for pos, n in self.segments[r]:
                if n > 0:
                    chunks.append((pos, n, r, off))
                off += n
        return sorted(chunks)

    def visible(self, q_rank: int, k_rank: int, group_tokens: int) -> bool:
        """False when every key of k_rank's shard is in a later causal group than every query of
        q_rank's shard (the step is skipped)."""
        if group_tokens <= 0:
            return True
        q_last = max(p + n - 1 for p, n in self.segments[q_rank] if n > 0) if self.length(q_rank) else -1
        k_first = min(p for p, n in self.segments[k_rank] if n > 0) if self.length(k_rank) else None
        if q_last < 0 or k_first is None:
            return False
        return k_first // group_tokens <= q_last // group_tokens


class KVBlock:
    """Quantised K/V of one shard in a single contiguous byte buffer (one P2P message), sized
    for ``L`` tokens; a shard of fewer tokens uses the leading rows."""

    def __init__(self, L: int, H: int, device, fmt: str = "fp8_e4m3", buf: torch.Tensor | None = None):
        self.L, self.H, self.fmt = L, H, fmt
        self.code_fmt, dtype = _FMT[fmt]
        n_codes = L * H * _D
        n_scale = L * H * 4
        if buf is not None and buf.numel() < 2 * (n_codes + n_scale):
            raise ValueError("KV block buffer too small")
        self.buf = buf if buf is not None else torch.empty(2 * (n_codes + n_scale), dtype=torch.uint8, device=device)
        b = self.buf
        self.k = b[:n_codes].view(dtype).view(1, L, H, _D)
        self.v = b[n_codes:2 * n_codes].view(dtype).view(1, L, H, _D)
        self.k_scale = b[2 * n_codes:2 * n_codes + n_scale].view(torch.float32).view(1, L, H, 1)
        self.v_scale = b[2 * n_codes + n_scale:].view(torch.float32).view(1, L, H, 1)

    def cache(self) -> dict:
        d = {"k": self.k, "v": self.v, "k_scale": self.k_scale, "v_scale": self.v_scale}
        if self.fmt == "fp8_e4m3":
            d["storage_format"] = "fp8_e4m3"
        return d

    def fill(self, k: torch.Tensor, v: torch.Tensor) -> None:
        """Quantise-on-write of this shard's bf16 K/V into rows [0, len) (assumed finite)."""
        _kvc.quantize_kv_pair_into(self.cache(), k, v, 0, assume_finite=True)


class RingAttention:
    """Buffers and launch state of one ring geometry (plan, heads, device, KV format).
    ``__call__`` runs one ring pass; ``steps`` lists the ring steps this rank computes."""

    def __init__(self, plan: RingPlan, rank: int, heads: int, device, *, tokens_per_frame: int,
                 causal_frames: int = 1, kv_format: str = "fp8_e4m3", softmax_scale: float | None = None):
        self.plan, self.rank, self.H, self.device = plan, rank, heads, torch.device(device)
        self.G = int(causal_frames) * int(tokens_per_frame)
        self.scale = float(softmax_scale) if softmax_scale else 0.0
        self.kv_format = kv_format
        self.lib = _lib.load()
        P, H, dev = plan.world, heads, self.device
        Lmax = plan.max_length()
        self.Lmax = Lmax
        self.blocks = [KVBlock(Lmax, H, dev, kv_format), KVBlock(Lmax, H, dev, kv_format)]
        # head-major bf16 operands: K at [0], V at [1], each [H, L_src, 128] in its region
        self.kvh = [torch.empty((2, H * Lmax * _D), dtype=torch.bfloat16, device=dev) for _ in range(2)]
        Ls = plan.length(rank)
        self.Ls = Ls
        self.qh = torch.empty((H * max(Ls, 1) * _D,), dtype=torch.bfloat16, device=dev)
        self.acc = torch.empty((max(Ls, 1), H, _D), dtype=torch.float32, device=dev)
        self.acc_lse = torch.empty((H, max(Ls, 1)), dtype=torch.float32, device=dev)
        self.kwords = ((Lmax + 127) // 128) * 4
        self.bits = {}
        with torch.cuda.device(dev):
            stream = _lib.stream_ptr(dev)
            for r in range(P):
                Lk = plan.length(r)
                if Lk not in self.bits:
                    t = torch.empty(max(self.kwords, 4), dtype=torch.int32, device=dev)
                    _lib.check(self.lib.hyb_fill_key_bits(1, Lk, self.kwords, t.data_ptr(), stream), "key bits")
                    self.bits[Lk] = t
            lay = _lib.WorkspaceLayout()
            _lib.check(self.lib.hyb_cached_attention_workspace_layout(1, H, _D, 0, max(Ls, 1), 0, 0,
                                                                      ctypes.byref(lay)), "ring layout")
        self.kv_splits = max(1, lay.kv_splits)
        if self.kv_splits > 1:
            self.part_o = torch.empty((self.kv_splits * H * Ls * _D,), dtype=torch.float32, device=dev)
            self.part_lse = torch.empty((self.kv_splits * H * Ls,), dtype=torch.float32, device=dev)
        else:
            self.part_o = self.part_lse = None
        self.comm_stream = torch.cuda.Stream(device=dev)
        self.status = _lib.device_status(dev)
        self.steps = [s for s in range(P) if plan.visible(rank, (rank - s) % P, self.G)]
        self.launches = 0
        # Optional instrumentation: when a list, each attention launch appends its (start, end)
        # CUDA events recorded on the caller's stream after the step's input is ready.
        self.event_log = None

    # ---------------------------------------------------------------- pieces of one step
    def _stage_block(self, block: KVBlock, Lk: int, kvh: torch.Tensor, stream: int) -> None:
        kv = _lib.coded_view(block.k, block.k_scale, block.code_fmt)
        vv = _lib.coded_view(block.v, block.v_scale, block.code_fmt)
        _lib.check(self.lib.hyb_stage_head_major(1, Lk, self.H, _D, ctypes.byref(kv), ctypes.byref(vv),
                                                 kvh[0].data_ptr(), kvh[1].data_ptr(), stream), "ring stage kv")
        self.launches += 1

    def _attend(self, src: int, kvh: torch.Tensor, out: torch.Tensor, lse, mode: int, stream: int) -> None:
        plan, H, Ls = self.plan, self.H, self.Ls
        Lk = plan.length(src)
        a = _lib.AttnArgs()
        a.abi_version = _lib.HYB_ABI_VERSION
        a.B, a.H, a.D, a.Lq, a.Lk = 1, H, _D, Ls, Lk
        a.hist_len, a.img_len, a.img_k_len = 0, Ls, Lk
        a.group_tokens = self.G
        a.softmax_scale = self.scale
        a.q_seg, a.q_pos0, a.q_pos1 = plan.positions(self.rank)
        a.k_seg, a.k_pos0, a.k_pos1 = plan.positions(src)
        a.q, a.k, a.v = self.qh.data_ptr(), kvh[0].data_ptr(), kvh[1].data_ptr()
        a.kbits, a.kwords = self.bits[Lk].data_ptr(), self.kwords
        a.qbits, a.qwords = None, 0
        a.out_img = out.data_ptr()
        a.oi_sb, a.oi_st, a.oi_sh = out.stride(0), out.stride(1), out.stride(2)
        a.oi_seg, a.oi_sseg = Ls, 0
        a.lse = lse.data_ptr() if lse is not None else None
        a.dev_status = self.status.data_ptr()
        a.kv_splits = self.kv_splits
        if self.kv_splits > 1:
            a.part_o, a.part_lse = self.part_o.data_ptr(), self.part_lse.data_ptr()
        a.acc_o, a.acc_lse, a.acc_mode = self.acc.data_ptr(), self.acc_lse.data_ptr(), mode
        _lib.check(self.lib.hyb_attn_fwd(ctypes.byref(a), stream), "ring attention step")
        self.launches += 2 if self.kv_splits > 1 else 1

    def _modes(self):
        """acc_mode per computed step: bit 0 merge with the accumulator, bit 1 final."""
        modes = {}
        for i, s in enumerate(self.steps):
            modes[s] = (1 if i > 0 else 0) | (2 if i == len(self.steps) - 1 else 0)
        return modes

    # ---------------------------------------------------------------- one ring pass
    def __call__(self, q, k, v, group=None, *, out=None, lse=None):
        """This rank's shard q/k/v bf16 [1, Ls, H, 128] -> out bf16 [1, Ls, H, 128] (and the
        natural-log LSE [1, H, Ls] into ``lse`` when given)."""
        P, r, H, Ls, dev = self.plan.world, self.rank, self.H, self.Ls, self.device
        if q.shape != (1, Ls, H, _D) or k.shape != q.shape or v.shape != q.shape:
            raise ValueError(f"ring shard must be [1, {Ls}, {H}, {_D}] on rank {r}")
        if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16 or v.dtype != torch.bfloat16:
            raise ValueError("ring attention takes bf16 q/k/v")
        _lib.require_same_device(dev, "ring q/k/v and outputs", q, k, v, out, lse)
        out = out if out is not None else torch.empty_like(q)
        ranks = dist.get_process_group_ranks(group) if (P > 1 and group is not None) else list(range(P))
        nxt, prv = ranks[(r + 1) % P], ranks[(r - 1) % P]
        compute = torch.cuda.current_stream(dev)
        comm = self.comm_stream
        cs, ms = compute.cuda_stream, comm.cuda_stream
        modes = self._modes()
        self.launches = 0
        if Ls == 0:
            return out
        with torch.cuda.device(dev):
            # own block: quantise-on-write, then decode it and stage Q (caller's stream)
            self.blocks[0].fill(k, v)
            self.launches += 1
            qv = _lib.bf16_view(q)
            _lib.check(self.lib.hyb_stage_head_major(1, Ls, H, _D, ctypes.byref(qv), None, self.qh.data_ptr(),
                                                     None, cs), "ring stage q")
            self.launches += 1
            self._stage_block(self.blocks[0], Ls, self.kvh[0], cs)
            ready = [torch.cuda.Event() for _ in range(P)]
            done = [torch.cuda.Event() for _ in range(P)]
            comm.wait_stream(compute)
            for s in range(P):
                src = (r - s) % P
                if s + 1 < P:
                    nsrc = (r - s - 1) % P
                    with torch.cuda.stream(comm):
                        ops = [dist.P2POp(dist.isend, self.blocks[s % 2].buf, nxt, group),
                               dist.P2POp(dist.irecv, self.blocks[(s + 1) % 2].buf, prv, group)]
                        for req in dist.batch_isend_irecv(ops):
                            req.wait()
                        if s >= 1:
                            comm.wait_event(done[s - 1])   # kvh[(s+1)%2] was read by step s-1
                        self._stage_block(self.blocks[(s + 1) % 2], self.plan.length(nsrc), self.kvh[(s + 1) % 2], ms)
                        ready[s + 1].record(comm)
                if s >= 1:
                    compute.wait_event(ready[s])
                if s in modes:
                    if self.event_log is not None:
                        ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                        ev[0].record(compute)
                    self._attend(src, self.kvh[s % 2], out, lse, modes[s], cs)
                    if self.event_log is not None:
                        ev[1].record(compute)
                        self.event_log.append(ev)
                done[s].record(compute)
            compute.wait_stream(comm)
        return out


def _u8_tensor(ptr: int, nbytes: int, device) -> torch.Tensor:
    from .communications import _DeviceArray
    return torch.as_tensor(_DeviceArray(ptr, (nbytes,), "|u1"), device=device)


def position_segments(chunks):
    """Maximal runs of consecutive positions of (position, length, owner, row) chunks given in
    position order: the key position segments of one launch."""
    segs = []
    for pos, n, _, _ in chunks:
        if segs and segs[-1][0] + segs[-1][1] == pos:
            segs[-1] = (segs[-1][0], segs[-1][1] + n)
        else:
            segs.append((pos, n))
    return segs


def overlap_groups(plan: RingPlan, rank: int):
    """Chunks of the overlapped all-gather schedule for ``rank``: its own chunks, and the other
    ranks' non-empty chunk groups, one launch each: those before the end of the rank's last
    chunk (at most two position segments under either layout: the ranges before and between
    the rank's chunks), then those after it (one segment)."""
    chunks = plan.gather_chunks()
    mine = [c for c in chunks if c[2] == rank]
    others = [c for c in chunks if c[2] != rank]
    own_end = max(c[0] + c[1] for c in mine) if mine else 0
    groups = [g for g in ([c for c in others if c[0] < own_end], [c for c in others if c[0] >= own_end]) if g]
    for g in groups:
        if len(position_segments(g)) > 2:
            raise RuntimeError("overlapped ring schedule: more than two key segments in one launch")
    return mine, groups


class GatherAttention:
    """The all-gather schedule of ring attention for a switched fabric.  Every rank quantises
    its K/V into its slot of a block buffer that every rank maps (CUDA IPC), pushes the block
    to every other rank in one kernel (each rank starting from a different peer, so the
    NVSwitch ports carry P - 1 streams at once) and meets them at a device barrier; one
    kernel then decodes all P blocks into a head-major bf16 K/V of the whole sequence in
    position order, and one attention launch covers this rank's query chunks against it.
    Moves the same bytes per rank as the neighbour ring (P - 1 blocks in, P - 1 out) without
    P attention launches and partial merges.  A device barrier before each push keeps a call's
    writes behind every peer's decode of the previous call's blocks (one block buffer per rank,
    safe under CUDA-graph replay because the barrier's epochs live in device memory).  ``emulate=True`` runs every rank in one process
    over a shared local buffer (tests on one GPU)."""

    def __init__(self, plan: RingPlan, rank: int, heads: int, device, *, tokens_per_frame: int,
                 causal_frames: int = 1, kv_format: str = "fp8_e4m3", softmax_scale: float | None = None,
                 group=None, shared=None, overlap: bool = False, push_blocks: int = 24):
        self.plan, self.rank, self.H, self.device = plan, rank, heads, torch.device(device)
        self.G = int(causal_frames) * int(tokens_per_frame)
        self.scale = float(softmax_scale) if softmax_scale else 0.0
        self.lib = lib = _lib.load()
        P, H, dev, L = plan.world, heads, self.device, plan.seq_len
        Lmax = plan.max_length()
        self.Lmax = Lmax
        self.code_fmt = _FMT[kv_format][0]
        self.block_bytes = ((2 * (Lmax * H * _D + Lmax * H * 4)) + 15) // 16 * 16
        self.peers = None
        if shared is not None:                   # emulation: one buffer holds every rank's block
            base = shared.data_ptr()
            self._keep = shared
        elif P > 1:
            from .communications import PeerBuffers
            self.peers = PeerBuffers(group, [P * self.block_bytes], dev, geometry=(L, H, Lmax, self.code_fmt))
            base = self.peers.local[0]
            self._push_dst = self.peers.table(0, offset=rank * self.block_bytes)
        else:
            self._keep = torch.empty(self.block_bytes, dtype=torch.uint8, device=dev)
            base = self._keep.data_ptr()
        self.base = base
        self.slots = [KVBlock(Lmax, H, dev, kv_format, buf=_u8_tensor(base + r * self.block_bytes, self.block_bytes, dev))
                      for r in range(P)]
        chunks = plan.gather_chunks()
        self.nchunks = len(chunks)
        self.bounds = (ctypes.c_int32 * (self.nchunks + 1))(*([c[0] for c in chunks] + [L]))
        self.owner = (ctypes.c_int32 * self.nchunks)(*[c[2] for c in chunks])
        self.row0 = (ctypes.c_int32 * self.nchunks)(*[c[3] for c in chunks])
        self.block_tab = (ctypes.c_void_p * P)(*[base + r * self.block_bytes for r in range(P)])
        self.overlap = bool(overlap) and P > 1
        # the single-launch schedule's head-major K/V of the whole sequence (the overlapped one
        # decodes into per-launch buffers instead)
        self.kv = None if self.overlap else torch.empty((2, H * max(L, 1) * _D), dtype=torch.bfloat16, device=dev)
        Ls = plan.length(rank)
        self.Ls = Ls
        self.qh = torch.empty((H * max(Ls, 1) * _D,), dtype=torch.bfloat16, device=dev)
        self.kwords = ((L + 127) // 128) * 4
        self.bits = torch.empty(max(self.kwords, 4), dtype=torch.int32, device=dev)
        with torch.cuda.device(dev):
            _lib.check(lib.hyb_fill_key_bits(1, L, self.kwords, self.bits.data_ptr(), _lib.stream_ptr(dev)), "key bits")
            lay = _lib.WorkspaceLayout()
            _lib.check(lib.hyb_cached_attention_workspace_layout(1, H, _D, L - Ls, max(Ls, 1), 0, 0, ctypes.byref(lay)),
                       "gather layout")
        self.kv_splits = max(1, lay.kv_splits)
        single = self.kv_splits > 1 and not self.overlap
        self.part_o = torch.empty((self.kv_splits * H * max(Ls, 1) * _D,), dtype=torch.float32, device=dev) \
            if single else None
        self.part_lse = torch.empty((self.kv_splits * H * max(Ls, 1),), dtype=torch.float32, device=dev) \
            if single else None
        self.status = _lib.device_status(dev)
        self.launches = 0
        self.event_log = None
        self.push_blocks = int(push_blocks)
        if self.overlap:
            self._setup_overlap()

    # ------------------------------------------------------------ overlapped schedule
    # The rank attends its own keys while its block crosses NVLink: the push runs on a side
    # stream on `push_blocks` blocks, the own-block launch on the other SMs; the other ranks'
    # keys, decoded once the push barrier has passed, follow in at most two launches (the
    # chunks before the rank's last chunk, two position segments under zig-zag sharding, then
    # those after it, whose keys only the rows of the same frame group see).  The launches
    # merge through the fp32 accumulator (acc_mode); only the last writes the bf16 output.
    def _chunk_table(self, chunks):
        n = len(chunks)
        starts, off = [], 0
        for c in chunks:
            starts.append(off)
            off += c[1]
        bounds = (ctypes.c_int32 * (n + 1))(*(starts + [off]))
        owner = (ctypes.c_int32 * max(n, 1))(*[c[2] for c in chunks])
        row0 = (ctypes.c_int32 * max(n, 1))(*[c[3] for c in chunks])
        return n, off, bounds, owner, row0

    def _setup_overlap(self) -> None:
        H, dev = self.H, self.device
        mine, groups = overlap_groups(self.plan, self.rank)
        self.own_tab = self._chunk_table(mine)
        self.own_segs = position_segments(mine)
        Ls = self.Ls
        self.kv_own = torch.empty((2, H * max(Ls, 1) * _D), dtype=torch.bfloat16, device=dev)
        self.parts = []   # (gather table, head-major K/V buffer, keys, position segments)
        for g in groups:
            n = sum(c[1] for c in g)
            buf = torch.empty((2, H * n * _D), dtype=torch.bfloat16, device=dev)
            self.parts.append((self._chunk_table(g), buf, n, position_segments(g)))
        self.acc = torch.empty((max(Ls, 1), H, _D), dtype=torch.float32, device=dev)
        self.acc_lse = torch.empty((H, max(Ls, 1)), dtype=torch.float32, device=dev)
        self.ov_bits, splits = {}, 1
        with torch.cuda.device(dev):
            stream = _lib.stream_ptr(dev)
            for Lk in [Ls] + [n for _, _, n, _ in self.parts]:
                kw = ((Lk + 127) // 128) * 4
                if Lk not in self.ov_bits:
                    t = torch.empty(max(kw, 4), dtype=torch.int32, device=dev)
                    _lib.check(self.lib.hyb_fill_key_bits(1, Lk, kw, t.data_ptr(), stream), "key bits")
                    self.ov_bits[Lk] = (t, kw)
                lay = _lib.WorkspaceLayout()
                _lib.check(self.lib.hyb_cached_attention_workspace_layout(1, H, _D, Lk - min(Lk, Ls), max(Ls, 1), 0,
                                                                          0, ctypes.byref(lay)), "ring layout")
                splits = max(splits, lay.kv_splits)
        self.ov_splits = splits
        self.ov_part_o = torch.empty((splits * H * max(Ls, 1) * _D,), dtype=torch.float32, device=dev) \
            if splits > 1 else None
        self.ov_part_lse = torch.empty((splits * H * max(Ls, 1),), dtype=torch.float32, device=dev) \
            if splits > 1 else None
        self.side = torch.cuda.Stream(device=dev)

    def _gather(self, tab, dst, stream: int) -> None:
        n, L, bounds, owner, row0 = tab
        if L == 0:
            return
        _lib.check(self.lib.hyb_ring_gather_stage(self.plan.world, self.code_fmt, L, self.H, _D, self.Lmax,
                                                  self.block_tab, n, bounds, owner, row0, dst[0].data_ptr(),
                                                  dst[1].data_ptr(), 1, stream), "ring gather stage")
        self.launches += 1

    def _launch(self, k_ptr, v_ptr, Lk, segs, mode, out, lse, stream: int) -> None:
        plan, H, Ls = self.plan, self.H, self.Ls
        a = _lib.AttnArgs()
        a.abi_version = _lib.HYB_ABI_VERSION
        a.B, a.H, a.D, a.Lq, a.Lk = 1, H, _D, Ls, Lk
        a.hist_len, a.img_len, a.img_k_len = 0, Ls, Lk
        a.group_tokens = self.G
        a.softmax_scale = self.scale
        a.q_seg, a.q_pos0, a.q_pos1 = plan.positions(self.rank)
        if len(segs) == 1:
            a.k_seg, a.k_pos0, a.k_pos1 = 0, segs[0][0], 0
        else:
            a.k_seg, a.k_pos0, a.k_pos1 = segs[0][1], segs[0][0], segs[1][0]
        a.q, a.k, a.v = self.qh.data_ptr(), k_ptr, v_ptr
        bits, kw = self.ov_bits[Lk]
        a.kbits, a.kwords = bits.data_ptr(), kw
        a.qbits, a.qwords = None, 0
        a.out_img = out.data_ptr()
        a.oi_sb, a.oi_st, a.oi_sh = out.stride(0), out.stride(1), out.stride(2)
        a.oi_seg, a.oi_sseg = Ls, 0
        a.lse = lse.data_ptr() if lse is not None else None
        a.dev_status = self.status.data_ptr()
        a.kv_splits = self.ov_splits
        a.v_f16 = 1
        if self.ov_splits > 1:
            a.part_o, a.part_lse = self.ov_part_o.data_ptr(), self.ov_part_lse.data_ptr()
        a.acc_o, a.acc_lse, a.acc_mode = self.acc.data_ptr(), self.acc_lse.data_ptr(), mode
        if self.event_log is not None:
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ev[0].record(torch.cuda.current_stream(self.device))
        _lib.check(self.lib.hyb_attn_fwd(ctypes.byref(a), stream), "ring attention (overlapped)")
        if self.event_log is not None:
            ev[1].record(torch.cuda.current_stream(self.device))
            self.event_log.append(ev)   # the launches of one call add up to its attention time
        self.launches += 2 if self.ov_splits > 1 else 1

    def attend_own(self, q, out, lse, stream: int) -> None:
        """Q staged head-major, the own block decoded, and its launch (first of the merge)."""
        H, Ls = self.H, self.Ls
        qv = _lib.bf16_view(q)
        _lib.check(self.lib.hyb_stage_head_major(1, Ls, H, _D, ctypes.byref(qv), None, self.qh.data_ptr(), None,
                                                 stream), "ring stage q")
        self.launches += 1
        self._gather(self.own_tab, self.kv_own, stream)
        last = not self.parts
        self._launch(self.kv_own[0].data_ptr(), self.kv_own[1].data_ptr(), Ls, self.own_segs, 2 if last else 0,
                     out, lse, stream)

    def attend_others(self, out, lse, stream: int) -> None:
        """The other ranks' keys (after the push barrier): per part a decode and a launch."""
        for i, (tab, buf, n, segs) in enumerate(self.parts):
            self._gather(tab, buf, stream)
            mode = 1 | (2 if i == len(self.parts) - 1 else 0)
            self._launch(buf[0].data_ptr(), buf[1].data_ptr(), n, segs, mode, out, lse, stream)

    def fill_own(self, k, v) -> None:
        self.slots[self.rank].fill(k, v)

    def exchange(self, stream: int) -> None:
        if self.peers is not None:
            # Every peer decodes the blocks of the previous call after that call's push barrier
            # (hyb_ring_gather_stage on its stream), so this call's push may overwrite them only
            # once every rank has passed the entry barrier, i.e. finished that decode.
            _lib.check(self.lib.hyb_peer_barrier(self.plan.world, self.rank, ctypes.byref(self.peers.sync), stream),
                       "ring block barrier")
            self.launches += 1
            _lib.check(self.lib.hyb_peer_push_bytes(self.plan.world, self.rank, self.slots[self.rank].buf.data_ptr(),
                                                    self.block_bytes, self._push_dst, ctypes.byref(self.peers.sync),
                                                    stream), "ring block push")
            self.launches += 1

    def attend(self, q, out, lse, stream: int) -> None:
        plan, H, Ls, L = self.plan, self.H, self.Ls, self.plan.seq_len
        qv = _lib.bf16_view(q)
        _lib.check(self.lib.hyb_stage_head_major(1, Ls, H, _D, ctypes.byref(qv), None, self.qh.data_ptr(), None,
                                                 stream), "ring stage q")
        kv_k, kv_v = self.kv[0].data_ptr(), self.kv[1].data_ptr()
        # V (and so P.V's softmax weights) in fp16: the bf16 decode converted exactly
        _lib.check(self.lib.hyb_ring_gather_stage(plan.world, self.code_fmt, L, H, _D, self.Lmax, self.block_tab,
                                                  self.nchunks, self.bounds, self.owner, self.row0, kv_k, kv_v,
                                                  1, stream), "ring gather stage")
        a = _lib.AttnArgs()
        a.abi_version = _lib.HYB_ABI_VERSION
        a.B, a.H, a.D, a.Lq, a.Lk = 1, H, _D, Ls, L
        a.hist_len, a.img_len, a.img_k_len = 0, Ls, L
        a.group_tokens = self.G
        a.softmax_scale = self.scale
        a.q_seg, a.q_pos0, a.q_pos1 = plan.positions(self.rank)
        a.k_seg, a.k_pos0, a.k_pos1 = 0, 0, 0
        a.q, a.k, a.v = self.qh.data_ptr(), kv_k, kv_v
        a.kbits, a.kwords = self.bits.data_ptr(), self.kwords
        a.qbits, a.qwords = None, 0
        a.out_img = out.data_ptr()
        a.oi_sb, a.oi_st, a.oi_sh = out.stride(0), out.stride(1), out.stride(2)
        a.oi_seg, a.oi_sseg = Ls, 0
        a.lse = lse.data_ptr() if lse is not None else None
        a.dev_status = self.status.data_ptr()
        a.kv_splits = self.kv_splits
        a.v_f16 = 1
        if self.kv_splits > 1:
            a.part_o, a.part_lse = self.part_o.data_ptr(), self.part_lse.data_ptr()
        if self.event_log is not None:
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ev[0].record(torch.cuda.current_stream(self.device))
        _lib.check(self.lib.hyb_attn_fwd(ctypes.byref(a), stream), "ring attention")
        if self.event_log is not None:
            ev[1].record(torch.cuda.current_stream(self.device))
            self.event_log.append(ev)
        self.launches += 3

    def __call__(self, q, k, v, group=None, *, out=None, lse=None):
        H, Ls, dev = self.H, self.Ls, self.device
        if q.shape != (1, Ls, H, _D) or k.shape != q.shape or v.shape != q.shape:
            raise ValueError(f"ring shard must be [1, {Ls}, {H}, {_D}] on rank {self.rank}")
        if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16 or v.dtype != torch.bfloat16:
            raise ValueError("ring attention takes bf16 q/k/v")
        _lib.require_same_device(dev, "ring q/k/v and outputs", q, k, v, out, lse)
        out = out if out is not None else torch.empty_like(q)
        self.launches = 0
        if Ls == 0:
            return out
        with torch.cuda.device(dev):
            cs = _lib.stream_ptr(dev)
            self.fill_own(k, v)
            self.launches += 1
            if not self.overlap:
                self.exchange(cs)
                self.attend(q, out, lse, cs)
                return out
            # Side stream: the entry barrier and the push, after everything this stream did
            # before (the previous call's decodes of the peers' blocks included).
            compute = torch.cuda.current_stream(dev)
            filled = torch.cuda.Event()
            filled.record(compute)
            pushed = torch.cuda.Event()
            with torch.cuda.stream(self.side):
                self.side.wait_event(filled)
                ss = self.side.cuda_stream
                _lib.check(self.lib.hyb_peer_barrier(self.plan.world, self.rank, ctypes.byref(self.peers.sync), ss),
                           "ring block barrier")
                _lib.check(self.lib.hyb_peer_push_bytes_n(self.plan.world, self.rank,
                                                          self.slots[self.rank].buf.data_ptr(), self.block_bytes,
                                                          self._push_dst, ctypes.byref(self.peers.sync),
                                                          self.push_blocks, ss), "ring block push")
                pushed.record(self.side)
            self.launches += 2
            self.attend_own(q, out, lse, cs)
            compute.wait_event(pushed)
            self.attend_others(out, lse, cs)
        return out

    def close(self) -> None:
        if self.peers is not None:
            self.peers.close()
            self.peers = None


_PLANS: dict = {}


SCHEDULES = ("allgather", "allgather_overlap", "ring")


def ring_attention(q, k, v, group=None, *, seq_len: int, tokens_per_frame: int, causal_frames: int = 1,
                   kv_format: str = "fp8_e4m3", layout: str = "zigzag", softmax_scale: float | None = None,
                   schedule: str = "allgather", out=None, lse=None):
    """Frame-causal self-attention of a sequence of ``seq_len`` tokens sharded over the ranks
    of ``group`` by ``RingPlan(seq_len, P, layout)``.  q/k/v: this rank's shard bf16
    [1, Ls, H, 128].  Returns this rank's output [1, Ls, H, 128] bf16.  ``schedule``:
    "allgather" (every block to every rank over peer memory, one attention launch) or "ring"
    (neighbour passing with NCCL send/recv, one launch per step)."""
    P = dist.get_world_size(group) if dist.is_initialized() else 1
    r = dist.get_rank(group) if dist.is_initialized() else 0
    ra = ring_plan_state(q, seq_len=seq_len, world=P, rank=r, tokens_per_frame=tokens_per_frame,
                         causal_frames=causal_frames, kv_format=kv_format, layout=layout,
                         softmax_scale=softmax_scale, schedule=schedule, group=group)
    return ra(q, k, v, group, out=out, lse=lse)


def ring_plan_state(q, *, seq_len, world, rank, tokens_per_frame, causal_frames=1, kv_format="fp8_e4m3",
                    layout="zigzag", softmax_scale=None, schedule="allgather", group=None):
    """The cached ``GatherAttention`` / ``RingAttention`` of this geometry (buffers are reused
    across calls; creating a gather schedule is collective over ``group``)."""
    if schedule not in SCHEDULES:
        raise ValueError(f"unknown ring schedule {schedule!r}")
    P, r = world, rank
    key = (seq_len, P, layout, r, q.shape[2], q.device, tokens_per_frame, causal_frames, kv_format, softmax_scale,
           schedule)
    ra = _PLANS.get(key)
    if ra is None:
        release_ring_states()
        plan = RingPlan(seq_len, P, layout)
        kw = dict(tokens_per_frame=tokens_per_frame, causal_frames=causal_frames, kv_format=kv_format,
                  softmax_scale=softmax_scale)
        if schedule in ("allgather", "allgather_overlap"):
            ra = GatherAttention(plan, r, q.shape[2], q.device, group=group, overlap=schedule == "allgather_overlap",
                                 **kw)
        else:
            ra = RingAttention(plan, r, q.shape[2], q.device, **kw)
        _PLANS[key] = ra
    return ra


def release_ring_states() -> None:
    """Free the cached ring states (peer buffers are unmapped: call before destroying the group)."""
    for ra in _PLANS.values():
        if hasattr(ra, "close"):
            ra.close()
    _PLANS.clear()


def ring_attention_emulated(q, k, v, world: int, *, tokens_per_frame: int, causal_frames: int = 1,
                            kv_format: str = "fp8_e4m3", layout: str = "zigzag", softmax_scale=None,
                            schedule: str = "ring"):
    """``world`` emulated ranks in one process on one GPU: q/k/v are the full sequence
    [1, L, H, 128]; the same kernels, in the same order, as ``ring_attention`` with the given
    schedule.  Returns the full output."""
    if schedule in ("allgather", "allgather_overlap"):
        return _gather_emulated(q, k, v, world, tokens_per_frame=tokens_per_frame, causal_frames=causal_frames,
                                kv_format=kv_format, layout=layout, softmax_scale=softmax_scale,
                                overlap=schedule == "allgather_overlap")
    plan = RingPlan(q.shape[1], world, layout)
    H, dev = q.shape[2], q.device
    rings = [RingAttention(plan, r, H, dev, tokens_per_frame=tokens_per_frame, causal_frames=causal_frames,
                           kv_format=kv_format, softmax_scale=softmax_scale) for r in range(world)]
    blocks = []
    for r in range(world):
        b = KVBlock(plan.max_length(), H, dev, kv_format)
        if plan.length(r):
            b.fill(plan.shard(k, r), plan.shard(v, r))
        blocks.append(b)
    outs = []
    cs = torch.cuda.current_stream(dev).cuda_stream
    with torch.cuda.device(dev):
        for r, ra in enumerate(rings):
            Ls = plan.length(r)
            out = torch.empty((1, Ls, H, _D), dtype=torch.bfloat16, device=dev)
            if Ls:
                qs = plan.shard(q, r).contiguous()
                qv = _lib.bf16_view(qs)
                _lib.check(ra.lib.hyb_stage_head_major(1, Ls, H, _D, ctypes.byref(qv), None, ra.qh.data_ptr(),
                                                       None, cs), "ring stage q")
                modes = ra._modes()
                for s in range(world):
                    src = (r - s) % world
                    if s in modes:
                        ra._stage_block(blocks[src], plan.length(src), ra.kvh[0], cs)
                        ra._attend(src, ra.kvh[0], out, None, modes[s], cs)
            outs.append(out)
    return plan.unshard(outs)


def _gather_emulated(q, k, v, world, *, tokens_per_frame, causal_frames, kv_format, layout, softmax_scale,
                     overlap=False):
    plan = RingPlan(q.shape[1], world, layout)
    H, dev = q.shape[2], q.device
    kw = dict(tokens_per_frame=tokens_per_frame, causal_frames=causal_frames, kv_format=kv_format,
              softmax_scale=softmax_scale)
    block_bytes = ((2 * (plan.max_length() * H * _D + plan.max_length() * H * 4)) + 15) // 16 * 16
    shared = torch.empty(world * block_bytes, dtype=torch.uint8, device=dev)
    # with overlap, the overlapped launches over the shared buffer (no push)
    states = [GatherAttention(plan, r, H, dev, shared=shared, overlap=overlap, **kw) for r in range(world)]
    for r, st in enumerate(states):
        if plan.length(r):
            st.fill_own(plan.shard(k, r).contiguous(), plan.shard(v, r).contiguous())
    outs = []
    cs = torch.cuda.current_stream(dev).cuda_stream
    with torch.cuda.device(dev):
        for r, st in enumerate(states):
            o = torch.empty((1, plan.length(r), H, _D), dtype=torch.bfloat16, device=dev)
            if plan.length(r):
                qs = plan.shard(q, r).contiguous()
                if st.overlap:
                    st.attend_own(qs, o, None, cs)
                    st.attend_others(o, None, cs)
                else:
                    st.attend(qs, o, None, cs)
            outs.append(o)
    return plan.unshard(outs)
