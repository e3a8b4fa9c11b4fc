"""Ring (KV-passing) sequence parallelism with frame-level causal masking.

Each rank holds a contiguous shard of the sequence (queries, keys and values).  Its keys and
values are quantised once to an e4m3 (or int8) block — codes and per-(token, head) scales in
one byte buffer — and the blocks travel around the ring: at step s a rank attends its queries
to the block of rank (r - s) mod P while NCCL moves the next block from rank r - 1 into the
other half of a double buffer (point-to-point copies over NVLink on a side stream, overlapped
with the attention of the current block).  Partial outputs are merged by log-sum-exp.

Transport and merge follow the reference's ring (``DynamicRingAttention.forward``,
hymm/models/dit/modules/attention/dynamic_ring_attention.py:115-286: isend/irecv to
``(idx + 1) % P`` / from ``(idx - 1) % P``, double-buffered, ``flash_attn_fwd_out_correction``
/ ``_softmax_lse_correction`` merges :86-105).  The reference ring is non-causal and serves
the non-cached path; the frame-level causal mask is the chunk-causal rule of
``create_magi_mp_causal_ranges`` (attention/magi_attn.py:290-309): query frame f sees key
frames <= f.  Blocks entirely in a query shard's future are not computed.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib
from . import attention as _att
from . import kv_cache as _kvc

_FMT = {"fp8_e4m3": (_lib.HYB_FMT_E4M3, torch.float8_e4m3fn), "int8": (_lib.HYB_FMT_INT8, torch.int8)}


class KVBlock:
    """Quantised K/V of one shard in a single contiguous byte buffer (one P2P message)."""

    def __init__(self, L: int, H: int, device, fmt: str = "fp8_e4m3", buf: torch.Tensor | None = None):
        self.L, self.H, self.fmt = L, H, fmt
        self.code_fmt, dtype = _FMT[fmt]
        n_codes = L * H * 128
        n_scale = L * H * 4
        self.nbytes = 2 * (n_codes + n_scale)
        self.buf = buf if buf is not None else torch.empty(self.nbytes, dtype=torch.uint8, device=device)
        b = self.buf
        self.k = b[:n_codes].view(dtype).view(1, L, H, 128)
        self.v = b[n_codes:2 * n_codes].view(dtype).view(1, L, H, 128)
        self.k_scale = b[2 * n_codes:2 * n_codes + n_scale].view(torch.float32).view(1, L, H, 1)
        self.v_scale = b[2 * n_codes + n_scale:].view(torch.float32).view(1, L, H, 1)

    def cache(self) -> dict:
        d = {"k": self.k, "v": self.v, "k_scale": self.k_scale, "v_scale": self.v_scale}
        if self.fmt == "fp8_e4m3":
            d["storage_format"] = "fp8_e4m3"
        return d

    def fill(self, k: torch.Tensor, v: torch.Tensor) -> None:
        """Quantise-on-write of this shard's bf16 K/V (assumed finite)."""
        _kvc.quantize_kv_pair_into(self.cache(), k, v, 0, assume_finite=True)


def frames_visible(q_start: int, q_len: int, k_start: int, group_tokens: int) -> bool:
    """False when every key of the block lies in a later causal group than every query."""
    if group_tokens <= 0 or q_len == 0:
        return True
    return k_start // group_tokens <= (q_start + q_len - 1) // group_tokens


def ring_step(q, block: KVBlock, acc, lse_acc, *, q_start: int, k_start: int, group_tokens: int,
              out=None, lse=None):
    """Attend the shard's queries ``q`` [1, Lq, H, D] to one block and merge the partial result
    into ``acc`` (fp32 [Lq, H, D]) / ``lse_acc`` (fp32 [H, Lq]) in place."""
    Lq, H = q.shape[1], q.shape[2]
    if not frames_visible(q_start, Lq, k_start, group_tokens):
        return
    if block.L != Lq:
        raise ValueError("ring blocks must have the query shard's length")
    empty = q[:, :0]
    out = out if out is not None else torch.empty_like(q)
    lse = lse if lse is not None else torch.empty((1, H, Lq), dtype=torch.float32, device=q.device)
    _att.cached_attention_local(
        q, (block.k, block.k_scale), (block.v, block.v_scale), empty, empty, empty, None, 0,
        attend_txt=False, group_tokens=group_tokens, out_img=out, lse=lse, q_pos0=q_start,
        k_pos0=k_start, img_kv_fmt=block.code_fmt)
    lib = _lib.load()
    with torch.cuda.device(q.device):
        _lib.check(lib.hyb_lse_merge(Lq, H, 128, acc.data_ptr(), lse_acc.data_ptr(), out.data_ptr(), 0,
                                     lse.data_ptr(), _lib.stream_ptr(q.device)), "ring merge")


def ring_attention(q, k, v, group=None, *, tokens_per_frame: int, causal_frames: int = 1,
                   kv_format: str = "fp8_e4m3"):
    """Frame-causal self-attention of a sequence sharded contiguously over the ranks of
    ``group`` (every rank holds the same number of tokens).  Returns this rank's output
    [1, Ls, H, D] bf16."""
    P = dist.get_world_size(group)
    r = dist.get_rank(group)
    ranks = dist.get_process_group_ranks(group) if group is not None else list(range(P))
    _, Ls, H, D = q.shape
    if D != 128:
        raise ValueError("head_dim must be 128")
    G = int(causal_frames) * int(tokens_per_frame)
    dev = q.device
    blocks = [KVBlock(Ls, H, dev, kv_format), KVBlock(Ls, H, dev, kv_format)]
    blocks[0].fill(k, v)
    acc = torch.zeros((Ls, H, D), dtype=torch.float32, device=dev)
    lse_acc = torch.full((H, Ls), float("-inf"), dtype=torch.float32, device=dev)
    out = torch.empty_like(q)
    lse = torch.empty((1, H, Ls), dtype=torch.float32, device=dev)
    nxt, prv = ranks[(r + 1) % P], ranks[(r - 1) % P]
    for s in range(P):
        cur = blocks[s % 2]
        reqs = []
        if s + 1 < P:
            ops = [dist.P2POp(dist.isend, cur.buf, nxt, group), dist.P2POp(dist.irecv, blocks[(s + 1) % 2].buf, prv, group)]
            reqs = dist.batch_isend_irecv(ops)
        src = (r - s) % P
        ring_step(q, cur, acc, lse_acc, q_start=r * Ls, k_start=src * Ls, group_tokens=G, out=out, lse=lse)
        for req in reqs:
            req.wait()
    return acc.view(1, Ls, H, D).to(torch.bfloat16)


def ring_attention_emulated(q_shards, k_shards, v_shards, *, tokens_per_frame: int, causal_frames: int = 1,
                            kv_format: str = "fp8_e4m3"):
    """The same schedule for P emulated ranks in one process (one GPU): every rank's queries
    meet every block in ring order.  Used to test the per-step math without a transport."""
    P = len(q_shards)
    G = int(causal_frames) * int(tokens_per_frame)
    Ls, H = q_shards[0].shape[1], q_shards[0].shape[2]
    dev = q_shards[0].device
    blocks = []
    for kk, vv in zip(k_shards, v_shards):
        b = KVBlock(Ls, H, dev, kv_format)
        b.fill(kk, vv)
        blocks.append(b)
    outs = []
    for r in range(P):
        acc = torch.zeros((Ls, H, 128), dtype=torch.float32, device=dev)
        lse_acc = torch.full((H, Ls), float("-inf"), dtype=torch.float32, device=dev)
        for s in range(P):
            src = (r - s) % P
            ring_step(q_shards[r], blocks[src], acc, lse_acc, q_start=r * Ls, k_start=src * Ls, group_tokens=G)
        outs.append(acc.view(1, Ls, H, 128).to(torch.bfloat16))
    return outs
