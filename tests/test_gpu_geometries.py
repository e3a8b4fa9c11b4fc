"""Parity at the remaining BASELINE geometries, with the north-star gate printed.

* config 3: the ring's frame-causal self-attention of 21 frames x 1,560 tokens, one launch
  (N = 1) and every rank of an 8-rank zig-zag ring emulated on one GPU (each rank's launch is
  4,095 queries in two segments against the 32,760 keys), 2 of the 24 heads;
* config 4: a 4-frame chunk against a 48-frame (74,880-token) E4M3 history, 3 heads (one
  rank's heads at Ulysses SP = 8);
* config 5: one 1,560-token frame against a first-frame sink + 32-frame window (51,480 keys
  read through the window's row map, rotated), 2 heads.
K/V are quantised by the oracle's restatement of the rule (CPU) and decoded as the reference
decodes them; the exact attention is computed in float64 on the GPU, query rows in chunks.
Gate: max-abs <= 2e-2 + the bf16 rounding floor of the exact rows, cosine >= 0.9995."""
import pytest
import torch

from hy_nomas_b200 import _lib
from hy_nomas_b200 import attention as hatt
from hy_nomas_b200 import kv_cache as kvc
from hy_nomas_b200 import ring
from hy_nomas_b200.synthetic import make_generator, seeded_kv
from oracle import quant as oq
from parity import check_bf16

pytestmark = pytest.mark.gpu

T = 1560


def exact(q, k, v, visible, chunk=2048):
    """float64 attention of q [Lq, D] over k/v [Lk, D]; visible(rows) -> bool [len(rows), Lk]."""
    out = torch.empty(q.shape[0], q.shape[1], dtype=torch.float64, device=q.device)
    kd, vd = k.double(), v.double()
    for a in range(0, q.shape[0], chunk):
        rows = torch.arange(a, min(a + chunk, q.shape[0]), device=q.device)
        s = (q[rows].double() @ kd.T) / (q.shape[1] ** 0.5)
        s.masked_fill_(~visible(rows), float("-inf"))
        out[rows] = torch.softmax(s, -1) @ vd
    return out


def decoded(x):
    """The bf16 values of an E4M3 cache / block holding x (quantised on the CPU)."""
    return oq.dequantize(*oq.quantize_e4m3(x.cpu()))


@pytest.mark.parametrize("world,schedule", [(1, "allgather"), (8, "allgather"), (8, "allgather_overlap")])
def test_config3_ring_geometry(cuda_lib, world, schedule):
    dev = torch.device("cuda")
    H, L = 2, 21 * T
    gen = make_generator(3003)
    q, k, v = (seeded_kv((1, L, H, 128), gen).to(dev) for _ in range(3))
    if world == 1:
        out = ring.ring_attention(q, k, v, None, seq_len=L, tokens_per_frame=T)
    else:
        out = ring.ring_attention_emulated(q, k, v, world, tokens_per_frame=T, schedule=schedule)
    torch.cuda.synchronize()
    _lib.check_device_status(dev)
    kd, vd = decoded(k).to(dev), decoded(v).to(dev)
    frame = torch.arange(L, device=dev) // T
    for h in range(H):
        ref = exact(q[0, :, h], kd[0, :, h], vd[0, :, h], lambda r: frame[None, :] <= frame[r][:, None])
        check_bf16(out[0, :, h], ref, f"config 3 ring ({schedule}), {world} rank(s), head {h}")


def test_config4_geometry(cuda_lib):
    dev = torch.device("cuda")
    H, Lh, Li, Lt = 3, 48 * T, 4 * T, 1
    gen = make_generator(4004)
    hk, hv = seeded_kv((1, Lh, H, 128), gen), seeded_kv((1, Lh, H, 128), gen)
    cur = [seeded_kv((1, L, H, 128), gen).to(dev) for L in (Li, Lt) for _ in range(3)]
    cache = kvc.make_fp8_kv_block(1, Lh + Li + Lt, H, 128, device=dev)
    with torch.no_grad():
        kvc.quantize_kv_pair_into(cache, hk.to(dev), hv.to(dev), 0)
    out_img, out_txt = hatt.cached_attention_local(*cur, cache, Lh, group_tokens=T)
    torch.cuda.synchronize()
    _lib.check_device_status(dev)
    k = torch.cat([decoded(hk).to(dev), cur[1], cur[4]], 1)
    v = torch.cat([decoded(hv).to(dev), cur[2], cur[5]], 1)
    q = torch.cat([cur[0], cur[3]], 1)
    kpos = torch.arange(k.shape[1], device=dev)
    kframe = torch.where((kpos >= Lh) & (kpos < Lh + Li), (kpos - Lh) // T, torch.full_like(kpos, -1))
    qframe = torch.where(torch.arange(Li + Lt, device=dev) < Li, torch.arange(Li + Lt, device=dev) // T,
                         torch.full((Li + Lt,), 10 ** 9, device=dev))
    got = torch.cat([out_img, out_txt], 1)
    for h in range(H):
        ref = exact(q[0, :, h], k[0, :, h], v[0, :, h], lambda r: kframe[None, :] <= qframe[r][:, None])
        check_bf16(got[0, :, h], ref, f"config 4 geometry, head {h}")


def test_config5_window_geometry(cuda_lib):
    dev = torch.device("cuda")
    H, sink, keep, rot = 2, 1, 32, 5
    slots = sink + keep
    gen = make_generator(5005)
    hk, hv = seeded_kv((1, slots * T, H, 128), gen), seeded_kv((1, slots * T, H, 128), gen)
    cur = [seeded_kv((1, T, H, 128), gen).to(dev) for _ in range(3)]
    empty = cur[0][:, :0]
    cache = kvc.make_fp8_kv_block(1, slots * T, H, 128, device=dev)
    with torch.no_grad():
        kvc.quantize_kv_pair_into(cache, hk.to(dev), hv.to(dev), 0)
    # composed history: the sink frame, then the window's slots oldest first (ring rotated)
    order = [0] + [sink + (j + rot) % keep for j in range(keep)]
    rows = torch.cat([torch.arange(s * T, (s + 1) * T) for s in order]).to(torch.int32)
    out_img, _ = hatt.cached_attention_local(cur[0], cur[1], cur[2], empty, empty, empty, cache, rows.numel(),
                                             hist_rows=rows.to(dev), group_tokens=T, attend_txt=False)
    torch.cuda.synchronize()
    _lib.check_device_status(dev)
    k = torch.cat([decoded(hk)[:, rows.long()].to(dev), cur[1]], 1)
    v = torch.cat([decoded(hv)[:, rows.long()].to(dev), cur[2]], 1)
    everything = torch.ones(1, k.shape[1], dtype=torch.bool, device=dev)
    for h in range(H):
        ref = exact(cur[0][0, :, h], k[0, :, h], v[0, :, h], lambda r: everything.expand(len(r), -1))
        check_bf16(out_img[0, :, h], ref, f"config 5 window geometry, head {h}")
