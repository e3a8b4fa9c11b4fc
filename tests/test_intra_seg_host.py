"""Host logic of the intra-segment action masks (hy_nomas_b200/intra_seg.py) on the CPU: the
window / offset plan, the device-side text masks, the key bitmap, the send-layout copy, the
reference's argument checks, and the three-step composition (common call, text rows over the
staged keys, per-action LSE merges) restated with the oracle's primitives against the oracle's
direct masked attention."""
import numpy as np
import pytest
import torch

from conftest import intra_case
from hy_nomas_b200 import attention as hatt
from hy_nomas_b200 import communications as comm
from hy_nomas_b200 import intra_seg as iseg
from oracle import attention as oatt
from oracle import sp as osp


def test_plan_turns_frame_windows_into_token_rows():
    plan = iseg.plan_intra_segment(48, [2, 4, 6], [[2, 3, 1], [0, 1, 0], [1, 2, -1]], 16)
    assert plan.windows == [(0, 16, 0), (16, 32, -1), (32, 48, 1)]
    assert plan.uncovered == []
    assert plan.action_rows == [[(0, 16)], [(32, 48)]]
    assert plan.live_actions == [0, 1]
    # clamped to the image rows, an empty window dropped, an out-of-range action is a gap,
    # empty text slices are not live, uncovered rows listed
    plan = iseg.plan_intra_segment(40, [1, 3, 3, 7], [[0, 1, 5], [2, 9, 0], [3, 3, 1]], 16)
    assert plan.windows == [(0, 16, -1), (32, 40, 0)]
    assert plan.uncovered == [(16, 32)]
    assert plan.live_actions == [0, 2]
    # without tokens_per_frame a window is counted in tokens
    assert iseg.plan_intra_segment(10, [0], [[2, 5, -1]], 0).windows == [(2, 5, -1)]


def test_plan_rejects_overlaps_and_bad_offsets():
    with pytest.raises(ValueError, match="overlap"):
        iseg.plan_intra_segment(64, [1, 2], [[0, 2, 0], [1, 3, -1]], 16)
    with pytest.raises(ValueError, match="nondecreasing"):
        iseg.plan_intra_segment(64, [3, 1, 4], [[0, 4, 0]], 16)
    with pytest.raises(ValueError, match="nondecreasing"):
        iseg.plan_intra_segment(64, [-1, 2], [[0, 4, 0]], 16)
    with pytest.raises(ValueError, match="head end"):
        iseg.plan_intra_segment(64, [], [[0, 4, 0]], 16)


@pytest.mark.parametrize("seed", range(6))
def test_text_masks_match_the_oracle_rows(seed):
    gen = torch.Generator().manual_seed(seed)
    Lt = int(torch.randint(1, 40, (1,), generator=gen))
    tm = torch.rand(Lt, generator=gen) < 0.7
    offs = sorted(int(x) for x in torch.randint(0, Lt + 4, (4,), generator=gen))
    head, acts = iseg.text_row_masks(tm, Lt, offs, "cpu")
    _, o_head, o_acts = oatt.intra_segment_rows(0, Lt, offs, [], tm)
    assert torch.equal(head, o_head)
    assert torch.equal(torch.stack(acts), o_acts)


def test_key_bits_pack_bit_j_of_word_j_div_32():
    gen = torch.Generator().manual_seed(1)
    for L in (1, 31, 32, 33, 127, 128, 300):
        mask = torch.rand(L, generator=gen) < 0.5
        kwords = ((L + 127) // 128) * 4
        words = iseg.pack_key_bits(mask, kwords)
        assert words.dtype == torch.int32 and words.numel() == kwords
        ref = np.packbits(np.pad(mask.numpy(), (0, kwords * 32 - L)), bitorder="little").view(np.int32)
        assert np.array_equal(words.numpy(), ref)


def test_fill_o_send_matches_the_epilogue_strides():
    """The plain output copied into the packed send buffer lands where the attention epilogue
    writes image row t of head h (offset (t // Ls) * sseg + (t % Ls) * st + h * sh + b * sb)."""
    B, P, Ls, Hp, D = 2, 3, 5, 2, 128
    send, strides = comm.o_send_buffer(B, [Ls] * P, Hp, D, torch.device("cpu"))
    sb, st, sh, seg, sseg = strides
    plain = torch.randn(B, P * Ls, Hp, D).to(torch.bfloat16)
    comm.fill_o_send(send, plain)
    view = torch.as_strided(send, (B, P, Ls, Hp, D), (sb, sseg, st, sh, 1))
    assert seg == Ls
    assert torch.equal(view.reshape(B, P * Ls, Hp, D), plain)


def test_drop_in_requires_flash3_for_an_intra_payload():
    x = torch.zeros(1, 16, 2, 128, dtype=torch.bfloat16)
    t = torch.zeros(1, 2, 2, 128, dtype=torch.bfloat16)
    cache = {"k": torch.zeros(1, 32, 2, 128, dtype=torch.bfloat16), "v": torch.zeros(1, 32, 2, 128, dtype=torch.bfloat16)}
    with pytest.raises(RuntimeError, match="requires attn_mode='flash3'"):
        hatt.causal_attention_with_cache_mp((x, t), (x, t), (x, t), cache, attn_mode="torch",
                                            intra_seg_txt_offsets=[[1, 2]], intra_seg_vid_windows=[[0, 1, 0]],
                                            tokens_per_frame=16)


def composed(cur, hk, hv, offsets, windows, T, text_mask, history_mask, group_tokens=0):
    """The product's three steps with the oracle standing in for each kernel: the common call
    (text mask = head text) with its LSE, the text rows over the staged keys C, and per live
    action the LSE merge of its rows with the action's text keys.  Intermediate image rows
    pass through bf16 as in the product (they are read back from the bf16 output)."""
    B, Li, H, D = cur[0].shape
    Lt = cur[3].shape[1]
    Lh = hk.shape[1]
    out_img = torch.zeros(B, Li, H, D)
    out_txt = torch.zeros(B, Lt, H, D)
    for b in range(B):
        c = [t[b:b + 1] for t in cur]
        hm = history_mask[b:b + 1] if history_mask.shape[0] == B else history_mask
        tm = text_mask[b:b + 1]
        hkb = hk[b:b + 1] if hk.shape[0] == B else hk
        hvb = hv[b:b + 1] if hv.shape[0] == B else hv
        offs = offsets[b] if b < len(offsets) else None
        if offs is None:
            oi, ot = oatt.cached_attention(*c, hkb, hvb, history_mask=hm, text_mask=tm, group_tokens=group_tokens)
            out_img[b], out_txt[b] = oi[0].bfloat16().float(), ot[0].bfloat16().float()
            continue
        plan = iseg.plan_intra_segment(Li, offs, windows, T)
        head, acts = iseg.text_row_masks(tm[0], Lt, plan.offsets, "cpu")
        oi, ot, lse = oatt.cached_attention(*c, hkb, hvb, history_mask=hm, text_mask=head[None],
                                            group_tokens=group_tokens, return_lse=True)
        oi, ot = oi[0].bfloat16().float(), ot[0].bfloat16().float()
        for a0, a1 in plan.uncovered:
            oi[a0:a1] = 0
        # text rows against C (every image key, visible history, head text; no block-causal rule)
        k_all = torch.cat([hkb.float(), c[1].float(), c[4].float()], dim=1)
        v_all = torch.cat([hvb.float(), c[2].float(), c[5].float()], dim=1)
        kvis = torch.cat([hm[0, :Lh].bool() if Lh else torch.zeros(0, dtype=torch.bool),
                          torch.ones(Li, dtype=torch.bool), head])
        _, acc_t, lse_t = oatt._masked_attention(c[3].float(), k_all, v_all, kvis[None, None].expand(1, Lt, -1),
                                                 torch.ones(1, Lt, dtype=torch.bool), 0, return_lse=True)
        for a in plan.live_actions:
            rows = plan.action_rows[a]
            n_img = sum(e - s for s, e in rows)
            qa = torch.cat([c[0][:, s:e] for s, e in rows] + [c[3]], dim=1).float()
            n = qa.shape[1]
            _, acc_a, lse_a = oatt._masked_attention(qa, c[4].float(), c[5].float(),
                                                     acts[a][None, None].expand(1, n, -1),
                                                     torch.ones(1, n, dtype=torch.bool), 0, return_lse=True)
            lse_a = lse_a[0].clone()
            lse_a[:, n_img:] = lse_a[:, n_img:].masked_fill(~acts[a][None, :], float("-inf"))
            base_o = torch.cat([oi[s:e] for s, e in rows] + [acc_t[0]], dim=0)
            base_lse = torch.cat([lse[0, :, s:e] for s, e in rows] + [lse_t[0]], dim=1)
            merged, _ = osp.lse_merge(acc_a[0], lse_a, base_o, base_lse)
            off = 0
            for s, e in rows:
                oi[s:e] = merged[off:off + e - s].bfloat16().float()
                off += e - s
            ot = torch.where(acts[a][:, None, None], merged[n_img:].bfloat16().float(), ot)
        out_img[b], out_txt[b] = oi, ot
    return out_img, out_txt


@pytest.mark.parametrize("name", ["basic", "batch", "nohist_update"])
def test_composition_equals_the_direct_mask(name):
    g, Lh, T, offsets, windows_tok, hk, hv, cur = intra_case(name)
    tm = torch.from_numpy(g["text_mask"])
    cm = torch.from_numpy(g["cache_mask"])
    ci, ct = composed(cur, hk, hv, offsets, g["windows"].tolist(), T, tm, cm)
    di, dt = oatt.intra_segment_attention(*cur, hk, hv, offsets, windows_tok, history_mask=cm, text_mask=tm)
    # bf16 rounding of the intermediate rows and of the result only
    torch.testing.assert_close(ci, di, atol=2e-2, rtol=2 ** -7)
    torch.testing.assert_close(ct, dt, atol=2e-2, rtol=2 ** -7)
    assert torch.equal(ci.abs().amax(dim=(2, 3)) == 0, di.abs().amax(dim=(2, 3)) == 0)
    assert torch.equal(ct.abs().amax(dim=(2, 3)) == 0, dt.abs().amax(dim=(2, 3)) == 0)


def test_composition_with_block_causal_rows():
    from hy_nomas_b200.synthetic import seeded_kv
    gen = torch.Generator().manual_seed(9)
    T, F, Lt, Lh, H = 16, 4, 9, 40, 2
    Li = T * F
    cur = [seeded_kv((1, L, H, 128), gen) for L in (Li, Lt) for _ in range(3)]
    hk, hv = seeded_kv((1, Lh, H, 128), gen), seeded_kv((1, Lh, H, 128), gen)
    tm = torch.tensor([[1, 1, 0, 1, 1, 1, 1, 1, 0]], dtype=torch.bool)
    cm = torch.ones(1, Lh, dtype=torch.bool)
    cm[:, 3:11] = False
    offsets, windows = [[2, 4, 7]], [[0, 2, 1], [3, 4, 0]]
    ci, ct = composed(cur, hk, hv, offsets, windows, T, tm, cm, group_tokens=2 * T)
    di, dt = oatt.intra_segment_attention(*cur, hk, hv, offsets, [[a * T, b * T, c] for a, b, c in windows],
                                          history_mask=cm, text_mask=tm, group_tokens=2 * T)
    torch.testing.assert_close(ci, di, atol=2e-2, rtol=2 ** -7)
    torch.testing.assert_close(ct, dt, atol=2e-2, rtol=2 ** -7)
