"""The tcgen05 cached-attention kernel against the oracle and the reference's outputs.

Tolerances.  The north star asks for max-abs-err 2e-2 and cosine >= 0.9995.  The cached path
computes with bf16 Q/K, fp16 V and P (P.V in fp16 with fp32 accumulation) and returns bf16
(the reference returns the input dtype).  The bf16 output's own rounding exceeds a flat 2e-2
on the benchmark's x8 outlier channels (outputs reach |o| ~ 20, where half a bf16 ulp is
0.03-0.06); the reference's own outputs carry exactly that error (tests/test_parity_floor.py),
and tests/test_gpu_parity_gate.py shows the kernel's fp32 rows within the flat gate and its
bf16 outputs at the reference's floor.  The elementwise bounds here are wider and also cover
the paths that keep bf16 P (ring, intra-segment): against the fp32 oracle
    |out - ref| <= 2e-2 + 2^-7 * |ref| + 2^-8 * (softmax(S) @ |V|)
(2e-2, plus one output ulp, plus twice a bf16 P's rounding on the element's weighted value
magnitude, computed by the oracle), with cosine >= 0.9995 over all valid rows.  Against the
reference's own bf16 outputs (golden fixtures, which carry their own rounding) the relative
term is 1e-2, and the north-star gate against the exact result is asserted and printed as
well.  Padded text query rows are exactly zero."""
import numpy as np
import pytest
import torch

from conftest import bf16, e4m3, intra_case, load_golden
from hy_nomas_b200 import attention as hatt
from hy_nomas_b200 import kv_cache as kvc
from hy_nomas_b200.synthetic import make_generator, seeded_kv
from oracle import attention as oatt
from oracle import quant as oq
from parity import check_bf16, metrics

pytestmark = pytest.mark.gpu

ATOL = 2e-2
RTOL = 2.0 ** -7       # one bf16 ulp of the reference value
COS = 0.9995


def errs(out: torch.Tensor, ref: torch.Tensor):
    o = out.float().flatten().cpu()
    r = ref.float().flatten().cpu()
    mae = (o - r).abs().max().item() if o.numel() else 0.0
    cos = torch.nn.functional.cosine_similarity(o[None], r[None]).item() if o.numel() else 1.0
    return mae, cos


MAG = 2.0 ** -8        # twice the bf16 rounding of P, on the weighted |V| magnitude


def assert_close(out, ref, what="", mag=None):
    mae, cos = errs(out, ref)
    o = out.float().flatten().cpu()
    r = ref.float().flatten().cpu()
    bound = ATOL + RTOL * r.abs()
    if mag is not None:
        bound = bound + MAG * mag.float().flatten().cpu()
    excess = ((o - r).abs() - bound).max().item() if o.numel() else -1.0
    assert excess <= 0 and cos >= COS, (
        f"{what}: max_abs_err={mae:.3e} excess_over_bound={excess:.3e} cos={cos:.6f}")


def make_case(B, Bc, Lh, Li, Lt, H, fmt, seed, cap_extra=8):
    gen = make_generator(seed)
    hk = seeded_kv((Bc, Lh, H, 128), gen)
    hv = seeded_kv((Bc, Lh, H, 128), gen)
    cur = [seeded_kv((B, L, H, 128), gen) for L in (Li, Lt) for _ in range(3)]
    cap = Lh + Li + Lt + cap_extra
    if fmt == "bf16":
        cache = {"k": torch.zeros(Bc, cap, H, 128, dtype=torch.bfloat16),
                 "v": torch.zeros(Bc, cap, H, 128, dtype=torch.bfloat16)}
        cache["k"][:, :Lh] = hk
        cache["v"][:, :Lh] = hv
        dk, dv = hk, hv
    else:
        ck, sk = oq.quantize(hk, fmt)
        cv, sv = oq.quantize(hv, fmt)
        dt = torch.int8 if fmt == "int8" else torch.float8_e4m3fn
        cache = {"k": torch.zeros(Bc, cap, H, 128, dtype=dt), "v": torch.zeros(Bc, cap, H, 128, dtype=dt),
                 "k_scale": torch.ones(Bc, cap, H, 1), "v_scale": torch.ones(Bc, cap, H, 1)}
        cache["k"][:, :Lh], cache["v"][:, :Lh] = ck, cv
        cache["k_scale"][:, :Lh], cache["v_scale"][:, :Lh] = sk, sv
        if fmt == "fp8_e4m3":
            cache["storage_format"] = "fp8_e4m3"
        dk, dv = oq.dequantize(ck, sk), oq.dequantize(cv, sv)
    return cache, cur, dk, dv


def to_dev(cache, dev):
    return {k: (v.to(dev) if isinstance(v, torch.Tensor) else v) for k, v in cache.items()}


CASES = [
    # B, Bc, Lh,   Li,  Lt, H, fmt,        G,   text_mask,        hist holes
    (1, 1, 256, 128, 1, 2, "fp8_e4m3", 0, None, []),
    (1, 1, 300, 200, 3, 2, "fp8_e4m3", 50, [1, 0, 1], [(5, 9)]),
    (1, 1, 0, 130, 2, 1, "int8", 0, [1, 1], []),
    (1, 1, 1000, 384, 1, 3, "int8", 128, None, [(100, 356)]),
    (2, 1, 513, 257, 4, 2, "fp8_e4m3", 64, [1, 1, 0, 0, 1, 0, 1, 1], [(0, 1)]),
    (2, 2, 129, 64, 1, 2, "bf16", 16, None, []),
    (1, 1, 64, 1, 1, 1, "fp8_e4m3", 0, None, []),
    (1, 1, 4096, 1560, 1, 2, "fp8_e4m3", 390, None, []),
]


@pytest.mark.parametrize("case", CASES, ids=[f"c{i}" for i in range(len(CASES))])
def test_cached_attention_vs_oracle(cuda_lib, case):
    B, Bc, Lh, Li, Lt, H, fmt, G, tmask, holes = case
    dev = torch.device("cuda")
    cache, cur, dk, dv = make_case(B, Bc, Lh, Li, Lt, H, fmt, seed=100 + CASES.index(case))
    hmask = torch.ones(Bc, Lh, dtype=torch.bool)
    for a, b in holes:
        hmask[:, a:b] = False
    text_mask = torch.tensor(tmask, dtype=torch.bool).reshape(B, Lt) if tmask else None
    lse = torch.empty(B, H, Li + Lt, dtype=torch.float32, device=dev)
    out_img, out_txt = hatt.cached_attention_local(
        *(t.to(dev) for t in cur), to_dev(cache, dev), Lh,
        history_mask=hmask.to(dev), text_mask=text_mask.to(dev) if text_mask is not None else None,
        attend_txt=True, group_tokens=G, lse=lse)
    torch.cuda.synchronize()
    from hy_nomas_b200 import _lib
    _lib.check_device_status(dev)
    ref_img, ref_txt, ref_lse, (mag_img, mag_txt) = oatt.cached_attention(
        *cur, dk, dv, history_mask=hmask, text_mask=text_mask, group_tokens=G, return_lse=True,
        return_magnitude=True)
    assert_close(out_img, ref_img, "image rows", mag_img)
    if Lt:
        valid = text_mask if text_mask is not None else torch.ones(B, Lt, dtype=torch.bool)
        assert_close(out_txt.cpu()[valid], ref_txt[valid], "text rows", mag_txt[valid])
        assert torch.all(out_txt.cpu()[~valid] == 0)
    fin = torch.isfinite(ref_lse)
    assert torch.equal(torch.isfinite(lse.cpu()), fin)
    assert (lse.cpu()[fin] - ref_lse[fin]).abs().max() < 1e-3


GOLDEN_CASES = ["int8_basic", "int8_update", "int8_nocachetxt", "int8_update_nocachetxt",
                "int8_cfg", "int8_empty_history"]


@pytest.mark.parametrize("case", GOLDEN_CASES)
def test_drop_in_matches_reference_outputs(cuda_lib, case):
    g = load_golden(f"attn_{case}.npz")
    dev = torch.device("cuda")
    Lh = int(g["Lh"])
    update, cache_txt = bool(g["update_cache"]), bool(g["cache_txt"])
    cache = {"k": torch.from_numpy(g["hist_k"]).to(dev), "v": torch.from_numpy(g["hist_v"]).to(dev),
             "k_scale": torch.from_numpy(g["hist_k_scale"]).to(dev),
             "v_scale": torch.from_numpy(g["hist_v_scale"]).to(dev)}
    cmask = torch.from_numpy(g["cache_mask"]).to(dev)
    tmask = torch.from_numpy(g["text_mask"]).to(dev)
    q = (bf16(g["img_q"]).to(dev), bf16(g["txt_q"]).to(dev))
    k = (bf16(g["img_k"]).to(dev), bf16(g["txt_k"]).to(dev))
    v = (bf16(g["img_v"]).to(dev), bf16(g["txt_v"]).to(dev))
    with torch.no_grad():
        out_img, out_txt = hatt.causal_attention_with_cache_mp(
            q, k, v, cache, cache_valid_len=Lh, attn_mode="flash3", text_mask=tmask,
            update_cache=update, cache_txt=cache_txt, cache_mask=cmask)
    torch.cuda.synchronize()
    B, Li, H, D = g["img_q"].shape
    Lt = g["txt_q"].shape[1]
    ref_img = bf16(g["out_img"]).float()
    ref_txt = bf16(g["out_txt"]).float()
    out_img = out_img.reshape(B, Li, H, D).float().cpu()
    out_txt = out_txt.reshape(B, Lt, H, D).float().cpu()
    assert ((out_img - ref_img).abs() <= ATOL + 1e-2 * ref_img.abs()).all()
    valid = torch.from_numpy(g["text_mask"])
    assert ((out_txt[valid] - ref_txt[valid]).abs() <= ATOL + 1e-2 * ref_txt[valid].abs()).all()
    assert torch.all(out_txt[~valid] == 0)
    # the north-star gate against the exact result of the same inputs (printed)
    import test_parity_floor as floor
    exact, ref_rows = floor._case(case)
    mae_ref, cos_ref = metrics(ref_rows, exact)
    print(f"{case}: reference bf16 vs exact max_abs={mae_ref:.4e} cos={cos_ref:.7f}")
    check_bf16(torch.cat([out_img.flatten(), out_txt[valid].flatten()]), exact, f"{case} drop-in bf16 output")
    if update:
        n = Li + (Lt if cache_txt else 0)
        for key in ("k", "v"):
            assert np.array_equal(cache[key][:, Lh:Lh + n].cpu().numpy(), g[f"written_{key}"][:, Lh:Lh + n])
            assert np.array_equal(cache[f"{key}_scale"][:, Lh:Lh + n].cpu().numpy().view(np.int32),
                                  g[f"written_{key}_scale"][:, Lh:Lh + n].view(np.int32))
        assert np.array_equal(cmask.cpu().numpy(), g["cache_mask_after"])


def test_frame_causal_matches_per_frame_reference_calls(cuda_lib):
    g = load_golden("attn_frame_causal_o3.npz")
    dev = torch.device("cuda")
    Lh, T, F = int(g["Lh"]), int(g["tokens_per_frame"]), int(g["frames"])
    cache = {"k": torch.from_numpy(g["hist_k"]).to(dev), "v": torch.from_numpy(g["hist_v"]).to(dev),
             "k_scale": torch.from_numpy(g["hist_k_scale"]).to(dev),
             "v_scale": torch.from_numpy(g["hist_v_scale"]).to(dev)}
    q = (bf16(g["img_q"]).to(dev), bf16(g["txt_q"]).to(dev))
    k = (bf16(g["img_k"]).to(dev), bf16(g["txt_k"]).to(dev))
    v = (bf16(g["img_v"]).to(dev), bf16(g["txt_v"]).to(dev))
    with torch.no_grad():
        out_img, out_txt = hatt.causal_attention_with_cache_mp(
            q, k, v, cache, cache_valid_len=Lh, attn_mode="flash3", tokens_per_frame=T,
            chunk_causal_frames=1)
    B, Li, H, D = g["img_q"].shape
    ref_img = bf16(g["out_img"]).float()
    got = out_img.reshape(B, Li, H, D).float().cpu()
    assert ((got - ref_img).abs() <= ATOL + 1e-2 * ref_img.abs()).all()
    ref_txt = bf16(g["out_txt"]).float()
    got_t = out_txt.reshape(ref_txt.shape).float().cpu()
    assert ((got_t - ref_txt).abs() <= ATOL + 1e-2 * ref_txt.abs()).all()


def test_fp8_drop_in_matches_o2_reference(cuda_lib):
    g = load_golden("attn_fp8_o2.npz")
    dev = torch.device("cuda")
    Lh = int(g["Lh"])
    cap = Lh + 80
    cache = kvc.make_fp8_kv_block(1, cap, 2, 128, device=dev)
    cache["k"][:, :Lh] = e4m3(g["hist_k"]).to(dev)
    cache["v"][:, :Lh] = e4m3(g["hist_v"]).to(dev)
    cache["k_scale"][:, :Lh] = torch.from_numpy(g["hist_k_scale"]).to(dev)
    cache["v_scale"][:, :Lh] = torch.from_numpy(g["hist_v_scale"]).to(dev)
    q = (bf16(g["img_q"]).to(dev), bf16(g["txt_q"]).to(dev))
    k = (bf16(g["img_k"]).to(dev), bf16(g["txt_k"]).to(dev))
    v = (bf16(g["img_v"]).to(dev), bf16(g["txt_v"]).to(dev))
    with torch.no_grad():
        out_img, out_txt = hatt.causal_attention_with_cache_mp(q, k, v, cache, cache_valid_len=Lh,
                                                               attn_mode="flash3")
    ref = bf16(g["out_img"]).float()
    got = out_img.reshape(ref.shape).float().cpu()
    assert ((got - ref).abs() <= ATOL + 1e-2 * ref.abs()).all()


def test_config2_geometry_vs_torch_fp32(cuda_lib):
    """BASELINE config 2 geometry (history 16 frames x 1560, 4-frame chunk, frame-causal)
    with 2 of the 24 heads, against an fp32 torch computation on the GPU."""
    dev = torch.device("cuda")
    H, T = 2, 1560
    Lh, Li, Lt = 16 * T, 4 * T, 1
    cache, cur, dk, dv = make_case(1, 1, Lh, Li, Lt, H, "fp8_e4m3", seed=1236)
    out_img, out_txt = hatt.cached_attention_local(
        *(t.to(dev) for t in cur), to_dev(cache, dev), Lh, group_tokens=T)
    torch.cuda.synchronize()
    q = torch.cat([cur[0], cur[3]], 1).to(dev).float()
    k = torch.cat([dk, cur[1], cur[4]], 1).to(dev).float()
    v = torch.cat([dv, cur[2], cur[5]], 1).to(dev).float()
    Lq, Lk = q.shape[1], k.shape[1]
    kpos = torch.arange(Lk, device=dev)
    qpos = torch.arange(Lq, device=dev)
    qblk = torch.where(qpos < Li, qpos // T, torch.full_like(qpos, 10 ** 9))
    kblk = torch.where((kpos >= Lh) & (kpos < Lh + Li), (kpos - Lh) // T, torch.full_like(kpos, -1))
    mask = kblk[None, :] <= qblk[:, None]
    ref = torch.empty(Lq, H, 128, device=dev)
    mag = torch.empty(Lq, H, 128, device=dev)
    for h in range(H):
        s = (q[0, :, h] @ k[0, :, h].T) / (128 ** 0.5)
        s.masked_fill_(~mask, float("-inf"))
        p = torch.softmax(s, -1)
        ref[:, h] = p @ v[0, :, h]
        mag[:, h] = p @ v[0, :, h].abs()
    assert_close(out_img[0], ref[:Li], "config-2 image rows", mag[:Li])
    assert_close(out_txt[0], ref[Li:], "config-2 text row", mag[Li:])


def test_ring_history_rows(cuda_lib):
    """A history given through a row map (sink + sliding window in a frame ring) equals the
    same rows laid out contiguously."""
    dev = torch.device("cuda")
    T, H = 64, 2
    cache, cur, dk, dv = make_case(1, 1, 10 * T, 2 * T, 1, H, "fp8_e4m3", seed=77)
    rows = torch.cat([torch.arange(0, T), torch.arange(6 * T, 10 * T), torch.arange(2 * T, 3 * T)]).to(torch.int32)
    cdev = to_dev(cache, dev)
    out_a, _ = hatt.cached_attention_local(*(t.to(dev) for t in cur), cdev, rows.numel(),
                                           hist_rows=rows.to(dev), group_tokens=T)
    ref_img, _, (mag, _) = oatt.cached_attention(*cur, dk[:, rows.long()], dv[:, rows.long()], group_tokens=T,
                                                 return_magnitude=True)
    assert_close(out_a, ref_img, "ring rows", mag)


def test_empty_text_and_single_query(cuda_lib):
    dev = torch.device("cuda")
    cache, cur, dk, dv = make_case(1, 1, 200, 1, 0, 2, "int8", seed=9)
    out_img, out_txt = hatt.cached_attention_local(*(t.to(dev) for t in cur), to_dev(cache, dev), 200)
    ref_img, _, (mag, _) = oatt.cached_attention(*cur, dk, dv, return_magnitude=True)
    assert out_txt.shape[1] == 0
    assert_close(out_img, ref_img, "single query", mag)


def test_exp2_poly_accuracy(cuda_lib):
    """The FMA-pipe exponential (packed pairs) against exp2 in float64: relative error <= 1e-4
    wherever the result is a normal float; below -125 and for -inf a nonnegative value under
    2^-125 (the kernel decides "no visible key" from the running maximum, not from P)."""
    from hy_nomas_b200 import _lib
    dev = torch.device("cuda")
    x = torch.cat([torch.linspace(-125.0, 12.0, 2_000_001), torch.tensor([-126.0, -1e4, float("-inf")])])
    x = x.to(dev)
    y = torch.empty_like(x)
    _lib.check(cuda_lib.hyb_exp2_poly_eval(x.data_ptr(), y.data_ptr(), x.numel(),
                                           torch.cuda.current_stream().cuda_stream), "exp2 poly")
    ref = torch.exp2(x.double())
    normal = x > -125.0
    rel = ((y.double() - ref).abs() / ref)[normal]
    assert rel.max().item() <= 1e-4, rel.max().item()
    tail = y[x < -125.0]
    assert torch.all(tail >= 0) and torch.all(tail < 2.0 ** -125)


@pytest.mark.parametrize("splits", [1, 2, 5, 16])
def test_key_slices_merge_to_the_same_result(cuda_lib, splits, monkeypatch):
    """Split-KV: each pair-CTA covers one slice of its key tiles and the partial rows are merged
    by LSE; every split count gives the oracle result (masks, padded text rows, LSE)."""
    monkeypatch.setenv("HYB_KV_SPLITS", str(splits))
    dev = torch.device("cuda")
    B, Lh, Li, Lt, H, G = 1, 3000, 700, 3, 2, 175
    cache, cur, dk, dv = make_case(B, 1, Lh, Li, Lt, H, "fp8_e4m3", seed=500 + splits)
    hmask = torch.ones(1, Lh, dtype=torch.bool)
    hmask[:, 1000:1300] = False
    text_mask = torch.tensor([[True, False, True]])
    lse = torch.empty(B, H, Li + Lt, dtype=torch.float32, device=dev)
    out_img, out_txt = hatt.cached_attention_local(
        *(t.to(dev) for t in cur), to_dev(cache, dev), Lh, history_mask=hmask.to(dev),
        text_mask=text_mask.to(dev), group_tokens=G, lse=lse)
    assert hatt.workspace_layout(B, H, Lh, Li, Lt, True).kv_splits == splits
    ref_img, ref_txt, ref_lse, (mag_img, mag_txt) = oatt.cached_attention(
        *cur, dk, dv, history_mask=hmask, text_mask=text_mask, group_tokens=G, return_lse=True,
        return_magnitude=True)
    assert_close(out_img, ref_img, f"image rows, {splits} slices", mag_img)
    valid = text_mask
    assert_close(out_txt.cpu()[valid], ref_txt[valid], "text rows", mag_txt[valid])
    assert torch.all(out_txt.cpu()[~valid] == 0)
    fin = torch.isfinite(ref_lse)
    assert torch.equal(torch.isfinite(lse.cpu()), fin)
    assert (lse.cpu()[fin] - ref_lse[fin]).abs().max() < 1e-3


def test_balanced_work_list_matches_oracle(cuda_lib, monkeypatch):
    """Without a forced split count the launch planner cuts query pairs into different numbers
    of key slices; the merged result still equals the oracle."""
    import ctypes
    monkeypatch.delenv("HYB_KV_SPLITS", raising=False)
    dev = torch.device("cuda")
    B, Lh, Li, Lt, H, G = 1, 3000, 2000, 3, 2, 500
    cache, cur, dk, dv = make_case(B, 1, Lh, Li, Lt, H, "fp8_e4m3", seed=611)
    lse = torch.empty(B, H, Li + Lt, dtype=torch.float32, device=dev)
    ws = hatt.Workspace()
    out_img, out_txt = hatt.cached_attention_local(*(t.to(dev) for t in cur), to_dev(cache, dev), Lh,
                                                   group_tokens=G, lse=lse, workspace=ws)
    ks = (ctypes.c_int32 * 64)()
    n = cuda_lib.hyb_attn_work_plan(ctypes.byref(ws.attn_args), 0, ks, 64)
    assert n == (Li + Lt + 255) // 256
    assert len(set(ks[:n])) > 1 and max(ks[:n]) > 1, list(ks[:n])
    ref_img, ref_txt, ref_lse, (mag_img, mag_txt) = oatt.cached_attention(
        *cur, dk, dv, group_tokens=G, return_lse=True, return_magnitude=True)
    assert_close(out_img, ref_img, "image rows, balanced slices", mag_img)
    assert_close(out_txt, ref_txt, "text rows", mag_txt)
    assert (lse.cpu() - ref_lse).abs().max() < 1e-3


@pytest.mark.parametrize("decoded", [False, True])
@pytest.mark.parametrize("sink,keep,fmt,write_in_call", [(1, 3, "fp8_e4m3", True), (2, 2, "int8", False)])
def test_window_rollout_matches_oracle(cuda_lib, sink, keep, fmt, write_in_call, decoded):
    """Long-rollout loop: every step attends a 1-frame chunk to the sink + sliding-window ring
    through the drop-in call, then appends the frame (quantise-on-write into the recycled
    slot; with ``decoded`` also its one-time decode into the window's mirror, which the
    attention then reads in slot order).  Each step equals the oracle over the reference's slid
    history."""
    from hy_nomas_b200.window import SinkWindowKVCache
    from oracle import window as ow
    dev = torch.device("cuda")
    T, H = 96, 2
    gen = make_generator(77 + keep)
    win = SinkWindowKVCache(1, H, T, sink, keep, storage_format=fmt, device=dev, decoded=decoded)
    all_k, all_v = [], []
    for step in range(sink + keep + 4):
        q, k, v = (seeded_kv((1, T, H, 128), gen) for _ in range(3))
        tq, tk, tv = (seeded_kv((1, 0 if write_in_call else 1, H, 128), gen) for _ in range(3))
        with torch.no_grad():
            out_img, out_txt = hatt.causal_attention_with_cache_mp(
                (q.to(dev), tq.to(dev)), (k.to(dev), tk.to(dev)), (v.to(dev), tv.to(dev)), win.view(),
                cache_valid_len=win.valid_len, update_cache=write_in_call, cache_txt=not write_in_call,
                tokens_per_frame=T, seg_ar_attention_backend="b200")
            if not write_in_call:
                win.append(k.to(dev), v.to(dev))
        # oracle: history = the reference slide of every frame so far, decoded
        frames = len(all_k)
        if frames:
            hk, _ = ow.slide(torch.cat(all_k, 1), frames, sink, keep, T)
            hv, kept = ow.slide(torch.cat(all_v, 1), frames, sink, keep, T)
            hk, hv = hk[:, :kept * T], hv[:, :kept * T]
        else:
            hk = hv = k[:, :0]
        ref_img, ref_txt, _, (mag_img, mag_txt) = oatt.cached_attention(
            q, k, v, tq, tk, tv, hk, hv, attend_txt=True, return_lse=True, return_magnitude=True)
        assert_close(out_img.view(1, T, H, 128), ref_img, f"window step {step} image", mag_img)
        assert out_txt.shape == (1, tq.shape[1], H * 128)
        assert_close(out_txt.view(1, tq.shape[1], H, 128), ref_txt, f"window step {step} text", mag_txt)
        ck, sk = oq.quantize(k, fmt)
        cv, sv = oq.quantize(v, fmt)
        all_k.append(oq.dequantize(ck, sk))
        all_v.append(oq.dequantize(cv, sv))
    assert win.frames == sink + keep + 4 and win.valid_len == (sink + keep) * T


def test_graphed_call_replays_the_drop_in(cuda_lib):
    """GraphedCall: warm-up calls run eagerly, then one captured graph per input buffer set;
    replayed outputs equal the eager call's bit for bit and the cache write is repeated."""
    import os
    from hy_nomas_b200.graphs import GraphedCall
    os.environ["HYB_ASSUME_FINITE_KV"] = "1"
    try:
        dev = torch.device("cuda")
        B, Lh, Li, Lt, H, G = 1, 512, 256, 1, 2, 128
        cache, cur, _, _ = make_case(B, 1, Lh, Li, Lt, H, "fp8_e4m3", seed=812)
        cache = to_dev(cache, dev)
        bufs = [[t.to(dev) for t in cur] for _ in range(2)]

        def step(qi, ki, vi, qt, kt, vt):
            with torch.no_grad():
                return hatt.causal_attention_with_cache_mp(
                    (qi, qt), (ki, kt), (vi, vt), cache, cache_valid_len=Lh, update_cache=True,
                    tokens_per_frame=G, chunk_causal_frames=1, seg_ar_attention_backend="b200")

        ref = [t.clone() for t in step(*bufs[0])]
        call = GraphedCall(step, dev, warmup=1)
        for i in range(6):
            out = call(*bufs[i % 2])
            torch.cuda.synchronize()
            for a, b in zip(out, ref):
                assert torch.equal(a, b), i
        assert len(call._graphs) == 2
        call.release()
    finally:
        os.environ.pop("HYB_ASSUME_FINITE_KV", None)


def test_config1_drop_in_matches_reference(cuda_lib):
    """BASELINE config 1 through the drop-in (history quantised on the GPU into an E4M3 cache,
    one frame of 256 tokens, frame-causal) against the reference's own outputs."""
    from conftest import config1_inputs
    g = load_golden("attn_config1.npz")
    dev = torch.device("cuda")
    hk, hv, cur, _ = config1_inputs()
    Lh, Li, Lt, H = 1024, 256, 1, 8
    cache = kvc.make_fp8_kv_block(1, Lh + Li + Lt, H, 128, device=dev)
    kvc.quantize_kv_pair_into(cache, hk.to(dev), hv.to(dev), 0)
    c = [t.to(dev) for t in cur]
    with torch.no_grad():
        out_img, out_txt = hatt.causal_attention_with_cache_mp(
            (c[0], c[3]), (c[1], c[4]), (c[2], c[5]), cache, cache_valid_len=Lh, attn_mode="flash3",
            tokens_per_frame=256, chunk_causal_frames=1)
    for got, key in ((out_img, "out_img"), (out_txt, "out_txt")):
        ref = bf16(g[key]).float()
        o = got.reshape(ref.shape).float().cpu()
        assert ((o - ref).abs() <= ATOL + 1e-2 * ref.abs()).all(), key
        assert torch.nn.functional.cosine_similarity(o.flatten()[None], ref.flatten()[None]).item() >= COS


@pytest.mark.parametrize("name", ["basic", "batch", "nohist_update"])
def test_intra_segment_drop_in_matches_reference(cuda_lib, name):
    """Intra-segment action masks through the drop-in (head text, per-action text slices, a
    gap window, an uncovered frame, offsets past the valid text, a sample without offsets, a
    cache write) against the reference's own outputs and against the fp32 oracle."""
    g, Lh, T, offsets, windows_tok, hk, hv, cur = intra_case(name)
    dev = torch.device("cuda")
    cache = {n: torch.from_numpy(g[f"hist_{n}"]).to(dev) for n in ("k", "v")}
    cache.update({f"{n}_scale": torch.from_numpy(g[f"hist_{n}_scale"]).to(dev) for n in ("k", "v")})
    cmask = torch.from_numpy(g["cache_mask"]).to(dev)
    tmask = torch.from_numpy(g["text_mask"])
    d = [t.to(dev) for t in cur]
    with torch.no_grad():
        out_img, out_txt = hatt.causal_attention_with_cache_mp(
            (d[0], d[3]), (d[1], d[4]), (d[2], d[5]), cache, cache_valid_len=Lh, attn_mode="flash3",
            text_mask=tmask.to(dev), update_cache=bool(g["update_cache"]), cache_txt=True, cache_mask=cmask,
            intra_seg_txt_offsets=offsets, intra_seg_vid_windows=g["windows"].tolist(), tokens_per_frame=T,
            seg_ar_attention_backend="magi")
    torch.cuda.synchronize()
    B, Li, H, D = cur[0].shape
    Lt = cur[3].shape[1]
    out_img = out_img.reshape(B, Li, H, D).float().cpu()
    out_txt = out_txt.reshape(B, Lt, H, D).float().cpu()
    ref_img, ref_txt = bf16(g["out_img"]).float(), bf16(g["out_txt"]).float()
    assert ((out_img - ref_img).abs() <= ATOL + 1e-2 * ref_img.abs()).all()
    assert ((out_txt - ref_txt).abs() <= ATOL + 1e-2 * ref_txt.abs()).all()
    # rows without ranges are exactly zero, and only those
    assert torch.equal(out_img.abs().amax(dim=(2, 3)) == 0, ref_img.abs().amax(dim=(2, 3)) == 0)
    assert torch.equal(out_txt.abs().amax(dim=(2, 3)) == 0, ref_txt.abs().amax(dim=(2, 3)) == 0)
    o_img, o_txt, (m_img, m_txt) = oatt.intra_segment_attention(
        *cur, hk, hv, offsets, windows_tok, history_mask=torch.from_numpy(g["cache_mask"]), text_mask=tmask,
        return_magnitude=True)
    assert_close(out_img, o_img, f"intra {name} image", m_img)
    assert_close(out_txt, o_txt, f"intra {name} text", m_txt)


def test_intra_segment_long_history_block_causal(cuda_lib):
    """Three actions over an FP8 history of 5,000 tokens (the text rows' pass over the staged
    keys runs in key slices) with the block-causal extension, against the fp32 oracle."""
    T, frames, Lt = 160, 3, 40
    cache, cur, dk, dv = make_case(1, 1, 5000, T * frames, Lt, 2, "fp8_e4m3", seed=77)
    dev = torch.device("cuda")
    cmask = torch.zeros(1, cache["k"].shape[1], dtype=torch.bool)
    cmask[:, :5000] = True
    cmask[:, 1200:1333] = False
    tmask = torch.ones(1, Lt, dtype=torch.bool)
    tmask[:, 30:] = False
    tmask[:, 7] = False
    offsets = [[5, 12, 20, 33]]
    windows = [[0, 1, 2], [1, 2, 0], [2, 3, 1]]
    d = [t.to(dev) for t in cur]
    with torch.no_grad():
        out_img, out_txt = hatt.causal_attention_with_cache_mp(
            (d[0], d[3]), (d[1], d[4]), (d[2], d[5]), to_dev(cache, dev), cache_valid_len=5000,
            attn_mode="flash3", text_mask=tmask.to(dev), cache_txt=True, cache_mask=cmask.to(dev),
            intra_seg_txt_offsets=offsets, intra_seg_vid_windows=windows, tokens_per_frame=T,
            chunk_causal_frames=1)
    torch.cuda.synchronize()
    o_img, o_txt, (m_img, m_txt) = oatt.intra_segment_attention(
        *cur, dk, dv, offsets, [[a * T, b * T, c] for a, b, c in windows], history_mask=cmask, text_mask=tmask,
        group_tokens=T, return_magnitude=True)
    assert_close(out_img.reshape(o_img.shape), o_img, "long intra image", m_img)
    assert_close(out_txt.reshape(o_txt.shape), o_txt, "long intra text", m_txt)
    assert torch.all(out_txt.reshape(o_txt.shape).cpu()[0, 30:] == 0)



@pytest.mark.parametrize("name", ["swa_int8_evict", "swa_bf16_evict", "swa_int8_overflow"])
def test_swa_history_sequence_matches_reference(cuda_lib, name):
    """A sequence of cache-writing calls on a bounded (``swa_capacity``) history: after every
    call the outputs match the reference's, and the cache rows (bit for bit), the mask, the
    records, ``swa_valid_len`` and ``swa_evicted`` are the ones the reference's commit left."""
    g = load_golden(f"{name}.npz")
    dev = torch.device("cuda")
    cap = int(g["cap"])
    H, D = g["0_img_k"].shape[2:]
    if "int8" in name:
        cache = kvc.make_int8_kv_block(1, cap, H, D, device=dev)
    else:
        cache = {"k": torch.zeros(1, cap, H, D, dtype=torch.bfloat16, device=dev),
                 "v": torch.zeros(1, cap, H, D, dtype=torch.bfloat16, device=dev)}
    cache["swa_capacity"] = int(g["capacity"])
    mask = torch.zeros(1, cap, dtype=torch.bool, device=dev)
    valid = 0
    for i in range(int(g["steps"])):
        x = {n: bf16(g[f"{i}_{n}"]).to(dev) for n in ("img_q", "img_k", "img_v", "txt_q", "txt_k", "txt_v")}
        with torch.no_grad():
            out_img, out_txt = hatt.causal_attention_with_cache_mp(
                (x["img_q"], x["txt_q"]), (x["img_k"], x["txt_k"]), (x["img_v"], x["txt_v"]), cache,
                cache_valid_len=valid, attn_mode="flash3", text_mask=torch.from_numpy(g[f"{i}_text_mask"]).to(dev),
                update_cache=True, cache_txt=True, cache_mask=mask, tokens_per_frame=16)
        torch.cuda.synchronize()
        ref_img, ref_txt = bf16(g[f"{i}_out_img"]).float(), bf16(g[f"{i}_out_txt"]).float()
        out_img = out_img.reshape(ref_img.shape).float().cpu()
        out_txt = out_txt.reshape(ref_txt.shape).float().cpu()
        assert ((out_img - ref_img).abs() <= ATOL + 1e-2 * ref_img.abs()).all(), f"step {i} image"
        valid_t = torch.from_numpy(g[f"{i}_text_mask"])[0]
        assert ((out_txt[0, valid_t] - ref_txt[0, valid_t]).abs() <= ATOL + 1e-2 * ref_txt[0, valid_t].abs()).all()
        assert torch.all(out_txt[0, ~valid_t] == 0)
        valid = cache["swa_valid_len"]
        assert valid == int(g[f"{i}_valid_after"]) and cache["swa_evicted"] == int(g[f"{i}_evicted"])
        for key in ("k", "v", "k_scale", "v_scale"):
            if f"{i}_{key}" not in g:
                continue
            got = cache[key][:, :valid].cpu()
            got = got.view(torch.int16) if got.dtype == torch.bfloat16 else got
            assert np.array_equal(got.numpy().view(np.uint8), g[f"{i}_{key}"].view(np.uint8)), f"step {i} {key}"
        assert np.array_equal(mask.cpu().numpy(), g[f"{i}_mask"])
        recs = [[r.start, r.image_tokens, r.end, r.time_start, r.height, r.width] for r in cache["swa_video"]]
        assert recs == g[f"{i}_records"].tolist()
