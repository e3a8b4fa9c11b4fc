"""Sequence-parallel kernels on one GPU with emulated ranks: the Ulysses pack / unpack kernels
and the attention epilogue that writes straight into the O all-to-all send buffer, against
the oracle layouts (pinned to the reference collectives by test_oracle_golden.py), and the
ring LSE merge against the oracle merge (pinned to dynamic_ring_attention.py)."""
import ctypes

import pytest
import torch

from conftest import load_golden
from hy_nomas_b200 import _lib
from hy_nomas_b200 import attention as hatt
from hy_nomas_b200.synthetic import make_generator, seeded_kv
from oracle import sp as osp

pytestmark = pytest.mark.gpu


def _stream():
    return torch.cuda.current_stream().cuda_stream


@pytest.mark.parametrize("P,lens", [(2, (7, 7)), (4, (5, 3, 5, 0)), (8, (4,) * 8)])
def test_pack_qkv_and_receive_views(cuda_lib, P, lens):
    dev = torch.device("cuda")
    B, H, D = 2, 8, 128
    gen = make_generator(10 + P)
    per_rank = [[seeded_kv((B, lens[r], H, D), gen) for _ in range(3)] for r in range(P)]
    Ls_max = max(lens)
    sends = []
    for r in range(P):
        q, k, v = (t.to(dev) for t in per_rank[r])
        send = torch.empty((P, Ls_max, 3 * B, H // P, D), dtype=torch.bfloat16, device=dev)
        views = [_lib.bf16_view(t) for t in (q, k, v)]
        _lib.check(cuda_lib.hyb_ulysses_pack_qkv(P, B, lens[r], Ls_max, H, D, *views, send.data_ptr(),
                                                 _stream()), "pack")
        ref = osp.pack_seq_to_heads(per_rank[r], P, Ls_max)
        assert torch.equal(send.cpu().view(torch.int16), ref.view(torch.int16))
        sends.append(send.cpu())
    for r, recv in enumerate(osp.simulate_all_to_all(sends)):
        ref = osp.unpack_seq_to_heads(recv, lens, 3)
        # product receive path: strided views into the receive buffer
        full = torch.cat([recv[src, :lens[src]] for src in range(P)], 0).permute(1, 0, 2, 3)
        for i in range(3):
            assert torch.equal(full[i * B:(i + 1) * B].contiguous().view(torch.int16), ref[i].view(torch.int16))


@pytest.mark.parametrize("P,lens", [(2, (6, 6)), (4, (3, 5, 0, 2))])
def test_pack_o_and_unpack_o(cuda_lib, P, lens):
    dev = torch.device("cuda")
    B, Hp, D = 2, 3, 128
    gen = make_generator(50 + P)
    outs = [seeded_kv((B, sum(lens), Hp, D), gen) for _ in range(P)]   # each rank's heads
    Ls_max = max(lens)
    sends = []
    for r in range(P):
        x = outs[r].to(dev)
        send = torch.empty((P, Hp, Ls_max, B, D), dtype=torch.bfloat16, device=dev)
        clens = (ctypes.c_int32 * P)(*lens)
        _lib.check(cuda_lib.hyb_ulysses_pack_o(P, B, clens, Ls_max, Hp, D, _lib.bf16_view(x), send.data_ptr(),
                                               _stream()), "pack o")
        ref = osp.pack_heads_to_seq(outs[r], lens)
        assert torch.equal(send.cpu().view(torch.int16), ref.view(torch.int16))
        sends.append(send.cpu())
    for r, recv in enumerate(osp.simulate_all_to_all(sends)):
        out = torch.empty((B, lens[r], Hp * P, D), dtype=torch.bfloat16, device=dev)
        recv_dev = recv.to(dev)
        _lib.check(cuda_lib.hyb_ulysses_unpack_o(P, B, lens[r], Ls_max, Hp * P, D, recv_dev.data_ptr(),
                                                 out.data_ptr(), *out.stride()[:3], _stream()), "unpack o")
        ref = osp.unpack_heads_to_seq(recv, lens[r])
        assert torch.equal(out.cpu().view(torch.int16), ref.view(torch.int16))


def test_attention_writes_the_o_send_buffer(cuda_lib):
    """Head-sharded attention output written through the send-buffer strides equals the plain
    output packed by the oracle layout."""
    from hy_nomas_b200 import communications as comm
    dev = torch.device("cuda")
    P, B, Hp, Ls = 4, 1, 2, 96
    gen = make_generator(77)
    L = P * Ls
    cur = [seeded_kv((B, n, Hp, 128), gen).to(dev) for n in (L, 1) for _ in range(3)]
    cache = {"k": torch.zeros(B, 1, Hp, 128, dtype=torch.bfloat16, device=dev),
             "v": torch.zeros(B, 1, Hp, 128, dtype=torch.bfloat16, device=dev)}
    plain, _ = hatt.cached_attention_local(*cur, cache, 0, group_tokens=32)
    buf, strides = comm.o_send_buffer(B, (Ls,) * P, Hp, 128, dev)
    hatt.cached_attention_local(*cur, cache, 0, group_tokens=32, out_img=buf, out_img_strides=strides)
    ref = osp.pack_heads_to_seq(plain.cpu(), (Ls,) * P)
    assert torch.equal(buf.cpu().view(torch.int16), ref.view(torch.int16))


def test_lse_merge_kernel_matches_oracle(cuda_lib):
    g = load_golden("ring_merge.npz")
    dev = torch.device("cuda")
    out_a = torch.from_numpy(g["out_a"])[0].float()
    lse_a = torch.from_numpy(g["lse_a"]).float()
    out_b = torch.from_numpy(g["out_b"])[0].float()
    lse_b = torch.from_numpy(g["lse_b"]).float()
    S, H, D = out_a.shape
    acc = out_a.clone().to(dev)
    lacc = lse_a.clone().to(dev)
    out_b_dev, lse_b_dev = out_b.to(dev), lse_b.to(dev)   # keep the device copies alive
    _lib.check(cuda_lib.hyb_lse_merge(S, H, D, acc.data_ptr(), lacc.data_ptr(), out_b_dev.data_ptr(), 1,
                                      lse_b_dev.data_ptr(), _stream()), "lse merge")
    ref_out, ref_lse = osp.lse_merge(out_a.double(), lse_a.double(), out_b.double(), lse_b.double())
    torch.testing.assert_close(lacc.cpu().double(), ref_lse, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(acc.cpu().double(), ref_out, rtol=1e-5, atol=1e-5)
    # and against the reference's own merged output
    torch.testing.assert_close(acc.cpu().double(), torch.from_numpy(g["out"])[0], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("schedule", ["ring", "allgather", "allgather_overlap"])
@pytest.mark.parametrize("P,frames,T,layout", [(1, 5, 64, "zigzag"), (4, 21, 48, "zigzag"),
                                               (3, 7, 100, "zigzag"), (3, 7, 100, "contiguous"),
                                               (8, 21, 39, "zigzag")])
def test_ring_schedule_matches_frame_causal_oracle(cuda_lib, P, frames, T, layout, schedule):
    """The ring's per-step attention launches with the accumulating epilogue, over P emulated
    ranks, equal frame-causal attention over the whole sequence (shards not aligned to frames,
    ragged zig-zag chunks when L is not a multiple of 2P)."""
    from hy_nomas_b200 import ring
    from oracle import attention as oatt
    from oracle import quant as oq
    dev = torch.device("cuda")
    H, L = 2, frames * T - 1
    gen = make_generator(900 + P)
    q, k, v = (seeded_kv((1, L, H, 128), gen) for _ in range(3))
    got = ring.ring_attention_emulated(q.to(dev), k.to(dev), v.to(dev), P, tokens_per_frame=T, layout=layout,
                                       schedule=schedule)
    # keys and values as the blocks carry them: e4m3 per (token, head), decoded
    kd = oq.dequantize(*oq.quantize_e4m3(k))
    vd = oq.dequantize(*oq.quantize_e4m3(v))
    e = q[:, :0]
    ref, _, (mag, _) = oatt.cached_attention(q, kd, vd, e, e, e, kd[:, :0], vd[:, :0], attend_txt=False,
                                             group_tokens=T, return_magnitude=True)
    o, r = got.cpu().float().flatten(), ref.flatten()
    bound = 2e-2 + 2.0 ** -7 * r.abs() + 2.0 ** -8 * mag.flatten()
    assert ((o - r).abs() <= bound).all(), ((o - r).abs() - bound).max()
    assert torch.nn.functional.cosine_similarity(o[None], r[None]).item() >= 0.9995


def test_stage_head_major_matches_dequant(cuda_lib):
    """hyb_stage_head_major decodes e4m3 blocks exactly as the oracle dequantiser, head-major."""
    from oracle import quant as oq
    dev = torch.device("cuda")
    gen = make_generator(5)
    x = seeded_kv((1, 77, 3, 128), gen)
    codes, scale = oq.quantize_e4m3(x)
    c_dev, s_dev = codes.to(dev), scale.to(dev)
    out = torch.empty((3, 77, 128), dtype=torch.bfloat16, device=dev)
    tv = _lib.coded_view(c_dev, s_dev, _lib.HYB_FMT_E4M3)
    _lib.check(cuda_lib.hyb_stage_head_major(1, 77, 3, 128, ctypes.byref(tv), None, out.data_ptr(), None,
                                             _stream()), "stage")
    ref = oq.dequantize(codes, scale)[0].permute(1, 0, 2).contiguous()
    assert torch.equal(out.cpu().view(torch.int16), ref.view(torch.int16))


def test_peer_barrier_times_out_into_the_status_word(cuda_lib):
    """The device barrier that ends every peer push waits for a flag that nothing sets here
    (the second "rank" is a local buffer no one signals from): after its bounded spin it
    records HYB_DEV_TIMEOUT in the status word and returns, and the context stays usable."""
    dev = torch.device("cuda")
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    src = torch.arange(64, dtype=torch.int32, device=dev)
    dst = [torch.zeros(64, dtype=torch.int32, device=dev) for _ in range(2)]
    flags = [torch.zeros(64, dtype=torch.int32, device=dev) for _ in range(2)]
    state = torch.zeros(2, dtype=torch.int32, device=dev)
    sync = _lib.PeerSync()
    sync.flags[0], sync.flags[1] = flags[0].data_ptr(), flags[1].data_ptr()
    sync.state = state.data_ptr()
    sync.dev_status = status.data_ptr()
    table = (ctypes.c_void_p * 2)(dst[0].data_ptr(), dst[1].data_ptr())
    _lib.check(cuda_lib.hyb_peer_push_bytes(2, 0, src.data_ptr(), src.numel() * 4, table, ctypes.byref(sync),
                                            _stream()), "push")
    torch.cuda.synchronize()
    assert status.item() & _lib.HYB_DEV_TIMEOUT
    assert torch.equal(dst[1], src) and torch.equal(dst[0], src)   # both destinations differ from the source
    assert flags[1][0].item() == 1 and flags[0][0].item() == 1 and flags[0][1].item() == 0
    assert int(state[0].item()) == 0 and int(state[1].item()) == 1
    assert torch.equal(src + 1, torch.arange(1, 65, dtype=torch.int32, device=dev))   # context still usable
