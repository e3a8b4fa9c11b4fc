"""Pin the CPU oracle to the reference: every restatement against the fixtures that the
reference's own functions produced (tests/golden/make_golden.py)."""
import numpy as np
import pytest
import torch

from conftest import bf16, e4m3, intra_case, load_golden
from oracle import attention as oatt
from oracle import quant as oq
from oracle import sp as osp
from oracle import window as owin

ATTN_CASES = ["int8_basic", "int8_update", "int8_nocachetxt", "int8_update_nocachetxt",
              "int8_cfg", "int8_empty_history"]

# The reference runs SDPA on bf16 inputs and rounds its output to bf16; the oracle keeps
# fp32.  Their difference is bounded by bf16 output rounding (2^-8 relative) plus the
# reference's internal rounding; the product tolerance (2e-2 abs, cos 0.9995) is looser.
ORACLE_ATOL = 2e-2
ORACLE_RTOL = 1e-2


def test_int8_quantiser_matches_reference_bitwise():
    g = load_golden("quant_int8.npz")
    for key in ("k", "v"):
        codes, scale = oq.quantize_int8(bf16(g[key]))
        assert np.array_equal(codes.numpy(), g[f"{key}_codes"])
        assert np.array_equal(scale.numpy().view(np.int32), g[f"{key}_scale"].view(np.int32))
        deq = oq.dequantize(codes, scale)
        assert torch.equal(deq.view(torch.int16), torch.from_numpy(g[f"{key}_deq"]))


def test_int8_quantiser_edge_rows():
    g = load_golden("quant_int8.npz")
    codes, scale = oq.quantize_int8(bf16(g["k"]))
    assert torch.all(codes[0, 0] == 0) and torch.all(scale[0, 0] == 1.0)      # zero row -> scale 1
    assert codes.abs().max() <= 127


def test_e4m3_quantiser_rule():
    gen = torch.Generator().manual_seed(3)
    from hy_nomas_b200.synthetic import seeded_kv
    x = seeded_kv((2, 33, 3, 128), gen)
    x[0, 0] = 0
    x[1, 2, 1] *= 1e-20
    codes, scale = oq.quantize_e4m3(x)
    assert codes.dtype == torch.float8_e4m3fn
    peak = x.float().abs().amax(-1, keepdim=True)
    expect = torch.where(peak > 0, peak / 448.0, torch.ones_like(peak))
    assert torch.equal(scale, expect)
    assert torch.all(scale[0, 0] == 1.0) and torch.all(codes[0, 0].float() == 0)
    # the row maximum maps to +-448 exactly; decode error is within one e4m3 half-ulp
    c = codes.float()
    assert torch.all(c.abs().amax(-1) <= 448)
    rel = ((c * scale) - x.float()).abs() / torch.clamp(x.float().abs(), min=1e-30)
    big = x.float().abs() > peak * 2 ** -6        # normal e4m3 range
    assert rel[big].max() <= 2 ** -4 + 1e-6


@pytest.mark.parametrize("case", ATTN_CASES)
def test_oracle_attention_matches_reference(case):
    g = load_golden(f"attn_{case}.npz")
    Lh = int(g["Lh"])
    hk = oq.dequantize(torch.from_numpy(g["hist_k"][:, :Lh]), torch.from_numpy(g["hist_k_scale"][:, :Lh]))
    hv = oq.dequantize(torch.from_numpy(g["hist_v"][:, :Lh]), torch.from_numpy(g["hist_v_scale"][:, :Lh]))
    cache_txt, update = bool(g["cache_txt"]), bool(g["update_cache"])
    tmask = torch.from_numpy(g["text_mask"])
    out_img, out_txt = oatt.cached_attention(
        bf16(g["img_q"]), bf16(g["img_k"]), bf16(g["img_v"]),
        bf16(g["txt_q"]), bf16(g["txt_k"]), bf16(g["txt_v"]), hk, hv,
        history_mask=torch.from_numpy(g["cache_mask"]), text_mask=tmask,
        attend_txt=cache_txt or update)
    ref_img = bf16(g["out_img"]).float()
    ref_txt = bf16(g["out_txt"]).float()
    torch.testing.assert_close(out_img, ref_img, atol=ORACLE_ATOL, rtol=ORACLE_RTOL)
    # torch mode computes padded text rows; the flash3 semantics (and the oracle) zero them
    valid = tmask.bool()
    torch.testing.assert_close(out_txt[valid], ref_txt[valid], atol=ORACLE_ATOL, rtol=ORACLE_RTOL)
    assert torch.all(out_txt[~valid] == 0)


@pytest.mark.parametrize("case", ["int8_update", "int8_update_nocachetxt"])
def test_oracle_cache_write_matches_reference(case):
    g = load_golden(f"attn_{case}.npz")
    Lh = int(g["Lh"])
    cache_txt = bool(g["cache_txt"])
    k = bf16(g["img_k"])
    v = bf16(g["img_v"])
    if cache_txt:
        k = torch.cat([k, bf16(g["txt_k"])], dim=1)
        v = torch.cat([v, bf16(g["txt_v"])], dim=1)
    n = k.shape[1]
    for key, x in (("k", k), ("v", v)):
        codes, scale = oq.quantize_int8(x)
        assert np.array_equal(codes.numpy(), g[f"written_{key}"][:, Lh:Lh + n])
        assert np.array_equal(scale.numpy().view(np.int32), g[f"written_{key}_scale"][:, Lh:Lh + n].view(np.int32))
    after = g["cache_mask_after"]
    img = g["img_k"].shape[1]
    assert after[:, Lh:Lh + img].all()
    if cache_txt:
        assert np.array_equal(after[:, Lh + img:Lh + n], g["text_mask"])


def test_oracle_fp8_o2_matches_reference():
    g = load_golden("attn_fp8_o2.npz")
    # pin the restated E4M3 quantiser on the fixture's raw history
    ck, sk = oq.quantize_e4m3(bf16(g["hist_k_raw"]))
    assert np.array_equal(ck.view(torch.uint8).numpy(), g["hist_k"])
    assert np.array_equal(sk.numpy(), g["hist_k_scale"])
    hk = oq.dequantize(e4m3(g["hist_k"]), torch.from_numpy(g["hist_k_scale"]))
    hv = oq.dequantize(e4m3(g["hist_v"]), torch.from_numpy(g["hist_v_scale"]))
    out_img, out_txt = oatt.cached_attention(
        bf16(g["img_q"]), bf16(g["img_k"]), bf16(g["img_v"]),
        bf16(g["txt_q"]), bf16(g["txt_k"]), bf16(g["txt_v"]), hk, hv)
    torch.testing.assert_close(out_img, bf16(g["out_img"]).float(), atol=ORACLE_ATOL, rtol=ORACLE_RTOL)
    torch.testing.assert_close(out_txt, bf16(g["out_txt"]).float(), atol=ORACLE_ATOL, rtol=ORACLE_RTOL)


def test_oracle_frame_causal_matches_per_frame_reference_calls():
    g = load_golden("attn_frame_causal_o3.npz")
    Lh, T = int(g["Lh"]), int(g["tokens_per_frame"])
    hk = oq.dequantize(torch.from_numpy(g["hist_k"][:, :Lh]), torch.from_numpy(g["hist_k_scale"][:, :Lh]))
    hv = oq.dequantize(torch.from_numpy(g["hist_v"][:, :Lh]), torch.from_numpy(g["hist_v_scale"][:, :Lh]))
    out_img, out_txt = oatt.cached_attention(
        bf16(g["img_q"]), bf16(g["img_k"]), bf16(g["img_v"]),
        bf16(g["txt_q"]), bf16(g["txt_k"]), bf16(g["txt_v"]), hk, hv, group_tokens=T)
    torch.testing.assert_close(out_img, bf16(g["out_img"]).float(), atol=ORACLE_ATOL, rtol=ORACLE_RTOL)
    torch.testing.assert_close(out_txt, bf16(g["out_txt"]).float(), atol=ORACLE_ATOL, rtol=ORACLE_RTOL)


def test_oracle_visibility_counts_match_flops():
    from hy_nomas_b200.flops import visible_pairs
    for Lh, Li, Lt, G, att in [(96, 64, 4, 16, True), (0, 50, 2, 16, True), (30, 48, 3, 0, False),
                               (24960 // 64, 6240 // 64, 1, 1560 // 64, True)]:
        vis = oatt.visibility(Lh, Li, Lt, att, G)
        assert int(vis.sum()) == visible_pairs(Lh, Li, Lt, att, G)


def test_oracle_sp_layouts_match_reference_collectives():
    r0, r1 = load_golden("sp_rank0.npz"), load_golden("sp_rank1.npz")
    ranks = [r0, r1]
    for case in ("even", "uneven"):
        lens = [int(x) for x in r0[f"{case}_lens"]]
        Ls_max = max(lens)
        sends = [osp.pack_seq_to_heads([bf16(r[f"{case}_{n}"]) for n in "qkv"], 2, Ls_max) for r in ranks]
        recvs = osp.simulate_all_to_all(sends)
        for r, rec in zip(ranks, recvs):
            q, k, v = osp.unpack_seq_to_heads(rec, lens, 3)
            for name, t in zip(("oq", "ok", "ov"), (q, k, v)):
                assert torch.equal(t.view(torch.int16), torch.from_numpy(r[f"{case}_{name}"]))
        sends = [osp.pack_heads_to_seq(bf16(r[f"{case}_o_in"]), lens) for r in ranks]
        recvs = osp.simulate_all_to_all(sends)
        for rank, (r, rec) in enumerate(zip(ranks, recvs)):
            out = osp.unpack_heads_to_seq(rec, lens[rank])
            assert torch.equal(out.view(torch.int16), torch.from_numpy(r[f"{case}_o_out"]))


def test_oracle_lse_merge_matches_reference():
    g = load_golden("ring_merge.npz")
    out, lse = osp.lse_merge(torch.from_numpy(g["out_a"])[0], torch.from_numpy(g["lse_a"]),
                             torch.from_numpy(g["out_b"])[0], torch.from_numpy(g["lse_b"]))
    torch.testing.assert_close(lse, torch.from_numpy(g["lse"]), rtol=1e-12, atol=1e-12)
    torch.testing.assert_close(out, torch.from_numpy(g["out"])[0], rtol=1e-10, atol=1e-10)


def test_oracle_window_slide_matches_reference():
    g = load_golden("window_slide.npz")
    T, frames, sink, keep = (int(g[k]) for k in ("tokens_per_frame", "frames", "sink", "keep"))
    k = torch.arange(frames * T, dtype=torch.float32).reshape(1, frames * T, 1, 1).repeat(1, 1, 2, 1)
    k_after, count = owin.slide(k, frames, sink, keep, T)
    assert count == int(g["new_count"])
    assert np.array_equal(k_after.numpy(), g["k_after"])
    vis = owin.visible_frames(frames, sink, keep)
    rows = torch.cat([torch.arange(f * T, (f + 1) * T) for f in vis])
    assert torch.equal(k[:, rows], k_after[:, :len(vis) * T])


def test_oracle_config1_matches_reference():
    """BASELINE config 1 (8 heads, a 256-token frame against 4 cached E4M3 frames + 1 text
    token): the regenerated inputs are the fixture's, and the oracle equals the reference."""
    from conftest import config1_inputs
    g = load_golden("attn_config1.npz")
    hk, hv, cur, sums = config1_inputs()
    assert np.array_equal(sums, g["checksums"])
    dk = oq.dequantize(*oq.quantize_e4m3(hk))
    dv = oq.dequantize(*oq.quantize_e4m3(hv))
    out_img, out_txt = oatt.cached_attention(*cur, dk, dv, group_tokens=256)
    torch.testing.assert_close(out_img, bf16(g["out_img"]).float(), atol=ORACLE_ATOL, rtol=ORACLE_RTOL)
    torch.testing.assert_close(out_txt, bf16(g["out_txt"]).float(), atol=ORACLE_ATOL, rtol=ORACLE_RTOL)


INTRA_CASES = ["basic", "batch", "nohist_update"]


@pytest.mark.parametrize("name", INTRA_CASES)
def test_oracle_intra_segment_visibility_is_the_reference_ranges(name):
    """Row by row, the restated mask equals the rectangles the reference's range builder made
    (exact: a single key too many or too few could hide inside the output tolerance)."""
    g, Lh, T, offsets, windows, hk, hv, cur = intra_case(name)
    B, Li = cur[0].shape[:2]
    Lt = cur[3].shape[1]
    vis, qvalid = oatt.intra_segment_visibility(
        Lh, Li, Lt, offsets, windows, history_mask=torch.from_numpy(g["cache_mask"]),
        text_mask=torch.from_numpy(g["text_mask"]), batch=B)
    assert torch.equal(vis & qvalid[:, :, None], torch.from_numpy(g["ref_visibility"]))


@pytest.mark.parametrize("name", INTRA_CASES)
def test_oracle_intra_segment_matches_reference(name):
    g, Lh, T, offsets, windows, hk, hv, cur = intra_case(name)
    out_img, out_txt = oatt.intra_segment_attention(
        *cur, hk, hv, offsets, windows, history_mask=torch.from_numpy(g["cache_mask"]),
        text_mask=torch.from_numpy(g["text_mask"]))
    torch.testing.assert_close(out_img, bf16(g["out_img"]).float(), atol=ORACLE_ATOL, rtol=ORACLE_RTOL)
    torch.testing.assert_close(out_txt, bf16(g["out_txt"]).float(), atol=ORACLE_ATOL, rtol=ORACLE_RTOL)
    # rows without ranges are exactly zero in both
    ref_zero = bf16(g["out_img"]).float().abs().amax(dim=(2, 3)) == 0
    assert torch.equal(out_img.abs().amax(dim=(2, 3)) == 0, ref_zero)


def test_oracle_intra_segment_rejects_overlaps_and_unordered_offsets():
    with pytest.raises(ValueError, match="overlap"):
        oatt.intra_segment_rows(32, 2, [1, 2], [[0, 20, 0], [16, 32, -1]])
    with pytest.raises(ValueError, match="nondecreasing"):
        oatt.intra_segment_rows(32, 4, [3, 1, 4], [[0, 32, 0]])
