#!/usr/bin/env python
"""Generate the golden fixtures of tests/golden/ by running the Hy-Nomas reference.

Run where the reference checkout is available, with ``HY_NOMAS_REF`` naming it:

    HY_NOMAS_REF=<reference checkout> python tests/golden/make_golden.py

The reference's DiT module imports ``diffusers`` only for two base classes; a 10-line
stub package written to a temporary directory stands in for it.  Every fixture stores
its inputs and the reference's outputs (bf16 as int16 bit patterns, e4m3 as uint8):

  quant_int8.npz        quantize_kv_pair_into / dequantize_kv, CPU branch
                        (hymm/models/dit/modules/int8_kv_cache.py:161-205)
  attn_<case>.npz       causal_attention_with_cache_mp(attn_mode="torch")
                        (hymm/models/dit/nomas_cpt.py:335-884): INT8 caches (O1), a bf16
                        cache of decoded E4M3 values (O2), frame-causal via one reference
                        call per query frame (O3), CFG history broadcast, cache writes
  sp_<case>.npz         all_to_all_qkv / all_to_all_4D / all_gather over 2 gloo ranks
                        (hymm/distributed/communications.py)
  ring_merge.npz        flash_attn_fwd_out_correction / _softmax_lse_correction
                        (attention/dynamic_ring_attention.py:86-105), eager bodies
  window_slide.npz      SelfForcingTrainingPipeline._slide_kv_cache sink + window eviction
                        (hymm/models/self_forcing/causal_training_pipeline.py:203-236)
  attn_config1.npz      BASELINE config 1 (8 heads, 256-token frame vs 4 cached E4M3 frames):
                        the reference's outputs only; the inputs are regenerated from the seed
                        (``config1_inputs``) and checked against the stored checksums
  intra_<case>.npz      causal_attention_with_cache_mp(attn_mode="flash3") with intra-segment
                        action masks (nomas_cpt.py:691-770 -> _intra_seg_cache_forward, :198-332,
                        ranges from _build_intra_seg_cache_ranges, :107-193).  The range kernel
                        it calls (MagiAttention / flex) runs on CUDA only; a dense stand-in with
                        the kernels' rectangle-union semantics (overlaps refused, rows without
                        ranges zero, fp32 softmax, bf16 output) takes its place, and the ranges
                        the reference built are stored as a dense visibility per sample
  swa_<fmt>_<case>.npz  bounded segment-AR history (sliding-window cache): a sequence of
                        causal_attention_with_cache_mp(attn_mode="torch", update_cache=True)
                        calls on a cache dict with ``swa_capacity`` (nomas_cpt.py:593-597,
                        :845-852 -> swa_cache.append_dense_record / commit_window), with the
                        outputs, cache rows, mask, records and lengths after every call
"""
from __future__ import annotations

import importlib
import os
import sys
import tempfile
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent


def _install_stub() -> None:
    sys.path.insert(0, str(REPO))
    from oracle.reference import install_stub
    try:
        install_stub()
    except RuntimeError as e:
        raise SystemExit(str(e))


def bf(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy()


def seeded(shape, gen):
    from hy_nomas_b200.synthetic import seeded_kv
    return seeded_kv(shape, gen)


def make_quant():
    i8 = importlib.import_module("hymm.models.dit.modules.int8_kv_cache")
    gen = torch.Generator().manual_seed(7)
    k = seeded((1, 40, 3, 128), gen)
    v = seeded((1, 40, 3, 128), gen)
    k[0, 0] = 0                        # all-zero rows -> scale 1
    v[0, 1, 1] = 0
    k[0, 2] *= 1e-30                   # tiny values (subnormal codes)
    v[0, 3] *= 4096.0                  # large values
    k[0, 4, 0, :] = torch.linspace(-127.5, 127.5, 128).to(torch.bfloat16)  # exact .5 ties
    cache = i8.make_int8_kv_block(1, 48, 3, 128, device="cpu")
    start = 5
    i8.quantize_kv_pair_into(cache, k, v, start)
    dk = i8.dequantize_kv(cache, "k", start + 40)
    dv = i8.dequantize_kv(cache, "v", start + 40)
    np.savez_compressed(
        HERE / "quant_int8.npz", k=bf(k), v=bf(v), start=start,
        k_codes=cache["k"][:, start:start + 40].numpy(), v_codes=cache["v"][:, start:start + 40].numpy(),
        k_scale=cache["k_scale"][:, start:start + 40].numpy(),
        v_scale=cache["v_scale"][:, start:start + 40].numpy(),
        k_deq=bf(dk[:, start:]), v_deq=bf(dv[:, start:]))


def _call_ref(native, **kw):
    with torch.no_grad():
        return native.causal_attention_with_cache_mp(attn_mode="torch", **kw)


def make_attention():
    native = importlib.import_module("hymm.models.dit.nomas_cpt")
    i8 = importlib.import_module("hymm.models.dit.modules.int8_kv_cache")
    sys.path.insert(0, str(REPO))
    from oracle.quant import quantize_e4m3, dequantize

    H, D = 2, 128

    def chunk(B, Li, Lt, gen):
        return [seeded((B, L, H, D), gen) for L in (Li, Lt) for _ in range(3)]

    def int8_cache(Bc, cap, Lh, gen):
        cache = i8.make_int8_kv_block(Bc, cap, H, D, device="cpu")
        hk, hv = seeded((Bc, Lh, H, D), gen), seeded((Bc, Lh, H, D), gen)
        i8.quantize_kv_pair_into(cache, hk, hv, 0)
        return cache

    def save(name, cache, args, out, extra=None):
        img_q, img_k, img_v, txt_q, txt_k, txt_v = args
        d = dict(img_q=bf(img_q), img_k=bf(img_k), img_v=bf(img_v),
                 txt_q=bf(txt_q), txt_k=bf(txt_k), txt_v=bf(txt_v),
                 out_img=bf(out[0]), out_txt=bf(out[1]))
        if cache["k"].dtype == torch.int8:
            d.update(hist_k=cache["k"].numpy(), hist_v=cache["v"].numpy(),
                     hist_k_scale=cache["k_scale"].numpy(), hist_v_scale=cache["v_scale"].numpy(),
                     fmt="int8")
        d.update(extra or {})
        np.savez_compressed(HERE / f"attn_{name}.npz", **d)

    def run_case(name, B, Bc, Lh, Li, Lt, text_mask, cache_mask_holes, update_cache, cache_txt, seed):
        gen = torch.Generator().manual_seed(seed)
        cap = Lh + Li + Lt + 16
        cache = int8_cache(Bc, cap, Lh, gen)
        args = chunk(B, Li, Lt, gen)
        cmask = torch.zeros(Bc, cap, dtype=torch.bool)
        cmask[:, :Lh] = True
        for a, b in cache_mask_holes:
            cmask[:, a:b] = False
        tmask = torch.tensor(text_mask, dtype=torch.bool).reshape(B, Lt)
        before = {k: v.clone() for k, v in cache.items()}
        mask_before = cmask.clone()
        out = _call_ref(native, q=(args[0], args[3]), k=(args[1], args[4]), v=(args[2], args[5]),
                        kv_cache=cache, cache_valid_len=Lh, text_mask=tmask,
                        update_cache=update_cache, cache_txt=cache_txt, cache_mask=cmask)
        out = (out[0].reshape(B, Li, H, D), out[1].reshape(B, Lt, H, D))
        extra = dict(Lh=Lh, cache_mask=mask_before.numpy(), text_mask=tmask.numpy(),
                     update_cache=update_cache, cache_txt=cache_txt, cap=cap,
                     cache_mask_after=cmask.numpy())
        if update_cache:
            extra.update(written_k=cache["k"].numpy(), written_v=cache["v"].numpy(),
                         written_k_scale=cache["k_scale"].numpy(), written_v_scale=cache["v_scale"].numpy())
        save(name, before, args, out, extra)

    # O1: INT8 cache, reference-exact path (kv_mask honoured in torch mode for int8).
    run_case("int8_basic", 1, 1, 96, 64, 4, [1, 1, 1, 0], [(10, 21)], False, True, 11)
    run_case("int8_update", 1, 1, 96, 64, 4, [1, 1, 0, 1], [(40, 45)], True, True, 12)
    run_case("int8_nocachetxt", 1, 1, 80, 48, 3, [1, 1, 1], [], False, False, 13)
    run_case("int8_update_nocachetxt", 1, 1, 80, 48, 3, [1, 0, 1], [], True, False, 14)
    run_case("int8_cfg", 2, 1, 64, 32, 2, [1, 1, 1, 0], [(0, 5)], False, True, 15)
    run_case("int8_empty_history", 1, 1, 0, 48, 2, [1, 1], [], False, True, 16)

    # O2: E4M3 codes (restated quantiser) decoded into a bf16 cache; torch mode ignores
    # kv_mask for a bf16 cache, so every key is valid here.
    gen = torch.Generator().manual_seed(21)
    Lh, Li, Lt, B = 128, 64, 1, 1
    hk, hv = seeded((1, Lh, H, D), gen), seeded((1, Lh, H, D), gen)
    ck, sk = quantize_e4m3(hk)
    cv, sv = quantize_e4m3(hv)
    cache = {"k": torch.zeros(1, Lh + Li + Lt, H, D, dtype=torch.bfloat16),
             "v": torch.zeros(1, Lh + Li + Lt, H, D, dtype=torch.bfloat16)}
    cache["k"][:, :Lh] = dequantize(ck, sk)
    cache["v"][:, :Lh] = dequantize(cv, sv)
    args = chunk(B, Li, Lt, gen)
    out = _call_ref(native, q=(args[0], args[3]), k=(args[1], args[4]), v=(args[2], args[5]),
                    kv_cache=cache, cache_valid_len=Lh, text_mask=None, update_cache=False,
                    cache_txt=True, cache_mask=None)
    out = (out[0].reshape(B, Li, H, D), out[1].reshape(B, Lt, H, D))
    np.savez_compressed(
        HERE / "attn_fp8_o2.npz", fmt="fp8_e4m3", Lh=Lh, hist_k=ck.view(torch.uint8).numpy(),
        hist_v=cv.view(torch.uint8).numpy(), hist_k_scale=sk.numpy(), hist_v_scale=sv.numpy(),
        hist_k_raw=bf(hk), hist_v_raw=bf(hv),
        img_q=bf(args[0]), img_k=bf(args[1]), img_v=bf(args[2]), txt_q=bf(args[3]),
        txt_k=bf(args[4]), txt_v=bf(args[5]), out_img=bf(out[0]), out_txt=bf(out[1]))

    # O3: frame-level block-causal = one reference call per query frame, history advanced
    # by the chunk's earlier frames (bf16 cache of decoded INT8 history + raw frames).
    gen = torch.Generator().manual_seed(31)
    T, F, Lh, Lt, B = 16, 3, 64, 1, 1
    Li = T * F
    cache8 = int8_cache(1, Lh + Li + Lt + 8, Lh, gen)
    args = chunk(B, Li, Lt, gen)
    hist_k = i8.dequantize_kv(cache8, "k", Lh)
    hist_v = i8.dequantize_kv(cache8, "v", Lh)
    out_img = torch.zeros(B, Li, H, D, dtype=torch.bfloat16)
    out_txt = None
    for f in range(F):
        prev = f * T
        cap = Lh + prev + T + Lt
        c = {"k": torch.zeros(1, cap, H, D, dtype=torch.bfloat16),
             "v": torch.zeros(1, cap, H, D, dtype=torch.bfloat16)}
        c["k"][:, :Lh] = hist_k
        c["v"][:, :Lh] = hist_v
        c["k"][:, Lh:Lh + prev] = args[1][:, :prev]
        c["v"][:, Lh:Lh + prev] = args[2][:, :prev]
        sl = slice(prev, prev + T)
        o = _call_ref(native, q=(args[0][:, sl], args[3]), k=(args[1][:, sl], args[4]),
                      v=(args[2][:, sl], args[5]), kv_cache=c, cache_valid_len=Lh + prev,
                      text_mask=None, update_cache=False, cache_txt=True, cache_mask=None)
        out_img[:, sl] = o[0].reshape(B, T, H, D)
        if f == F - 1:
            # text queries see every frame: take them from a call over the whole chunk
            c2 = {"k": torch.zeros(1, Lh + Li + Lt, H, D, dtype=torch.bfloat16),
                  "v": torch.zeros(1, Lh + Li + Lt, H, D, dtype=torch.bfloat16)}
            c2["k"][:, :Lh] = hist_k
            c2["v"][:, :Lh] = hist_v
            o2 = _call_ref(native, q=(args[0], args[3]), k=(args[1], args[4]), v=(args[2], args[5]),
                           kv_cache=c2, cache_valid_len=Lh, text_mask=None, update_cache=False,
                           cache_txt=True, cache_mask=None)
            out_txt = o2[1].reshape(B, Lt, H, D)
    np.savez_compressed(
        HERE / "attn_frame_causal_o3.npz", fmt="int8", Lh=Lh, tokens_per_frame=T, frames=F,
        hist_k=cache8["k"].numpy(), hist_v=cache8["v"].numpy(), hist_k_scale=cache8["k_scale"].numpy(),
        hist_v_scale=cache8["v_scale"].numpy(),
        img_q=bf(args[0]), img_k=bf(args[1]), img_v=bf(args[2]), txt_q=bf(args[3]),
        txt_k=bf(args[4]), txt_v=bf(args[5]), out_img=bf(out_img), out_txt=bf(out_txt))


def _sp_worker(rank, world, init_file, out_dir):
    import torch.distributed as dist
    _install_stub()
    comm = importlib.import_module("hymm.distributed.communications")
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world)
    H, D, B = 4, 128, 1
    res = {}
    for case, lens in (("even", (6, 6)), ("uneven", (5, 3))):
        gen = torch.Generator().manual_seed(100 + rank)
        q, k, v = (torch.randn(B, lens[rank], H, D, generator=gen).to(torch.bfloat16) for _ in range(3))
        meta = comm.prepare_sp_communication(lens[rank], H, "cpu", None)
        oq, ok, ov = comm.all_to_all_qkv(q, k, v, group=None, sequence_lengths=meta.sequence_lengths)
        o_in = torch.randn(B, sum(lens), H // world, D, generator=gen).to(torch.bfloat16)
        o_out = comm.all_to_all_4D(o_in, group=None, scatter_dim=1, gather_dim=2,
                                   sequence_lengths=meta.sequence_lengths)
        t_in = torch.randn(B, 3, H // world, D, generator=gen).to(torch.bfloat16)
        t_out = comm.all_gather(t_in, dim=2, group=None, sizes=meta.head_sizes)
        res.update({f"{case}_q": bf(q), f"{case}_k": bf(k), f"{case}_v": bf(v),
                    f"{case}_oq": bf(oq), f"{case}_ok": bf(ok), f"{case}_ov": bf(ov),
                    f"{case}_o_in": bf(o_in), f"{case}_o_out": bf(o_out),
                    f"{case}_t_in": bf(t_in), f"{case}_t_out": bf(t_out),
                    f"{case}_lens": np.array(lens)})
    np.savez_compressed(Path(out_dir) / f"sp_rank{rank}.npz", **res)
    dist.destroy_process_group()


def make_sp():
    import torch.multiprocessing as mp
    init_file = tempfile.mktemp(prefix="hyb_gloo_")
    mp.spawn(_sp_worker, args=(2, init_file, str(HERE)), nprocs=2, join=True)


def make_ring_merge():
    dra = importlib.import_module("hymm.models.dit.modules.attention.dynamic_ring_attention")
    out_fn = dra.flash_attn_fwd_out_correction.__wrapped__
    lse_fn = dra.flash_attn_fwd_softmax_lse_correction.__wrapped__
    gen = torch.Generator().manual_seed(41)
    S, H, D = 24, 3, 128
    out_a = torch.randn(1, S, H, D, generator=gen, dtype=torch.float64)
    lse_a = torch.randn(H, S, generator=gen, dtype=torch.float64) * 3
    out_b = torch.randn(1, S, H, D, generator=gen, dtype=torch.float64)
    lse_b = torch.randn(H, S, generator=gen, dtype=torch.float64) * 3
    lse_b[0, :4] = float("-inf")       # rows a step could not see
    lse = lse_a.clone()
    lse_fn(lse, lse_b)
    # The reference rescales every step's output by its own lse against the final lse.
    out = torch.zeros_like(out_a)
    out_fn(out, out_a, 1, lse, lse_a)   # bshd, seq_dim = 1 (dynamic_ring_attention.py:253-262)
    out_fn(out, out_b, 1, lse, lse_b)
    np.savez_compressed(HERE / "ring_merge.npz", out_a=out_a.numpy(), lse_a=lse_a.numpy(),
                        out_b=out_b.numpy(), lse_b=lse_b.numpy(), lse=lse.numpy(), out=out.numpy())


def make_window():
    ctp = importlib.import_module("hymm.models.self_forcing.causal_training_pipeline")
    T, frames, sink, keep = 4, 12, 1, 5
    k = torch.arange(frames * T, dtype=torch.float32).reshape(1, frames * T, 1, 1).repeat(1, 1, 2, 1)
    ns = types.SimpleNamespace(kv_cache1=[{"k": k.clone(), "v": (k + 1000).clone()}], sink_frames=sink,
                               cache_keep_frames=keep, _tokens_per_frame=T, num_max_frames=frames)
    new_count = ctp.SelfForcingTrainingPipeline._slide_kv_cache(ns, frames)
    np.savez_compressed(HERE / "window_slide.npz", tokens_per_frame=T, frames=frames, sink=sink, keep=keep,
                        new_count=new_count, k_after=ns.kv_cache1[0]["k"].numpy(),
                        v_after=ns.kv_cache1[0]["v"].numpy())


def config1_inputs():
    """BASELINE config 1 inputs, regenerated identically by the tests: B=1, 8 heads x 128, a
    256-token frame (16 x 16) against 4 cached frames (1,024 tokens) and 1 text token, seeded
    N(0, 1) with 4 outlier channels per head x8 (config seed 1235)."""
    from hy_nomas_b200.synthetic import config_seed, make_generator
    gen = make_generator(config_seed(1))
    H = 8
    hk, hv = seeded((1, 1024, H, 128), gen), seeded((1, 1024, H, 128), gen)
    cur = [seeded((1, L, H, 128), gen) for L in (256, 1) for _ in range(3)]
    return hk, hv, cur


def input_checksums(tensors):
    return np.array([t.double().sum().item() for t in tensors], dtype=np.float64)


def make_config1():
    """Config 1 through the reference: e4m3 codes of the history (restated quantiser; the
    reference has no FP8 cache) decoded into a bf16 cache, one torch-mode call.  Stores only
    the outputs and input checksums (the inputs are regenerated from the seed)."""
    native = importlib.import_module("hymm.models.dit.nomas_cpt")
    from oracle.quant import dequantize, quantize_e4m3
    hk, hv, cur = config1_inputs()
    ck, sk = quantize_e4m3(hk)
    cv, sv = quantize_e4m3(hv)
    Lh, Li, Lt, H = 1024, 256, 1, 8
    cache = {"k": torch.zeros(1, Lh + Li + Lt, H, 128, dtype=torch.bfloat16),
             "v": torch.zeros(1, Lh + Li + Lt, H, 128, dtype=torch.bfloat16)}
    cache["k"][:, :Lh] = dequantize(ck, sk)
    cache["v"][:, :Lh] = dequantize(cv, sv)
    out = _call_ref(native, q=(cur[0], cur[3]), k=(cur[1], cur[4]), v=(cur[2], cur[5]), kv_cache=cache,
                    cache_valid_len=Lh, text_mask=None, update_cache=False, cache_txt=True, cache_mask=None)
    np.savez_compressed(HERE / "attn_config1.npz", out_img=bf(out[0].reshape(1, Li, H, 128)),
                        out_txt=bf(out[1].reshape(1, Lt, H, 128)),
                        checksums=input_checksums([hk, hv, *cur]))



def _dense_range_kernel(calls):
    """Stand-in for the range attention kernel (CUDA-only in the reference): the union of the
    (q_range, k_range) rectangles is the visibility, as both backends define it (flex refuses
    overlapping rectangles, range_attention.py:97-100); softmax in fp32, rows without keys
    zero, output in the input dtype.  Every call's rectangles are appended to ``calls``."""
    def kernel(q, k, v, q_ranges, k_ranges, attn_type_map=None, backend="magi", softmax_scale=None,
               deterministic=False, **kwargs):
        nq, nk, D = q.shape[0], k.shape[0], q.shape[-1]
        cover = torch.zeros(nq, nk, dtype=torch.int32)
        for (qs, qe), (ks, ke) in zip(q_ranges.tolist(), k_ranges.tolist()):
            cover[qs:qe, ks:ke] += 1
        if nq and nk and int(cover.max()) > 1:
            raise ValueError("overlapping QK rectangles")
        vis = cover.bool()
        calls.append(vis.clone())
        qf, kf, vf = (x.float().transpose(0, 1) for x in (q, k, v))
        s = (qf @ kf.transpose(1, 2)) * (softmax_scale or 1.0 / D ** 0.5)
        s = s.masked_fill(~vis[None], float("-inf"))
        m = s.amax(-1, keepdim=True)
        m = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
        p = torch.exp(s - m)
        l = p.sum(-1, keepdim=True)
        o = (p @ vf) / torch.where(l > 0, l, torch.ones_like(l))
        return o.transpose(0, 1).to(q.dtype), None
    return kernel


def make_intra_seg():
    """Intra-segment action masks through the reference's flash3 cached path (INT8 cache)."""
    native = importlib.import_module("hymm.models.dit.nomas_cpt")
    i8 = importlib.import_module("hymm.models.dit.modules.int8_kv_cache")
    H, D = 2, 128
    calls = []
    native.range_attention = _dense_range_kernel(calls)
    native._flex_flash_attn_func = object()      # the magi branch only checks that it exists

    def run_case(name, B, Lh, holes, T, frames, text_mask, offsets, windows, update_cache, seed):
        gen = torch.Generator().manual_seed(seed)
        Li, Lt = T * frames, len(text_mask[0])
        cap = Lh + Li + Lt + 8
        cache = i8.make_int8_kv_block(B, cap, H, D, device="cpu")
        if Lh:
            i8.quantize_kv_pair_into(cache, seeded((B, Lh, H, D), gen), seeded((B, Lh, H, D), gen), 0)
        args = [seeded((B, L, H, D), gen) for L in (Li, Lt) for _ in range(3)]
        cmask = torch.zeros(B, cap, dtype=torch.bool)
        cmask[:, :Lh] = True
        for b, (a, e) in holes:
            cmask[b, a:e] = False
        tmask = torch.tensor(text_mask, dtype=torch.bool)
        before = {k: v.clone() for k, v in cache.items()}
        mask_before = cmask.clone()
        calls.clear()
        with torch.no_grad():
            out = native.causal_attention_with_cache_mp(
                (args[0], args[3]), (args[1], args[4]), (args[2], args[5]), cache, cache_valid_len=Lh,
                attn_mode="flash3", text_mask=tmask, update_cache=update_cache, cache_txt=True,
                cache_mask=cmask, intra_seg_txt_offsets=offsets, intra_seg_vid_windows=windows,
                tokens_per_frame=T, seg_ar_attention_backend="magi")
        assert len(calls) == B
        # the reference's rectangles (compact per sample) as dense [Lq, Lk] visibility
        dense = torch.zeros(B, Li + Lt, Lh + Li + Lt, dtype=torch.bool)
        for b in range(B):
            hist_idx = mask_before[b, :Lh].nonzero().flatten()
            txt_idx = tmask[b].nonzero().flatten()
            qpos = torch.cat([torch.arange(Li), Li + txt_idx])
            kpos = torch.cat([hist_idx, Lh + torch.arange(Li), Lh + Li + txt_idx])
            dense[b][qpos[:, None], kpos[None, :]] = calls[b]
        np.savez_compressed(
            HERE / f"intra_{name}.npz", Lh=Lh, T=T, frames=frames, update_cache=update_cache,
            hist_k=before["k"].numpy(), hist_v=before["v"].numpy(), hist_k_scale=before["k_scale"].numpy(),
            hist_v_scale=before["v_scale"].numpy(), cache_mask=mask_before.numpy(), text_mask=tmask.numpy(),
            offsets=np.array([-1 if o is None else len(o) for o in offsets], dtype=np.int64),
            offsets_flat=np.array([x for o in offsets if o is not None for x in o], dtype=np.int64),
            windows=np.array(windows, dtype=np.int64).reshape(-1, 3), ref_visibility=dense.numpy(),
            img_q=bf(args[0]), img_k=bf(args[1]), img_v=bf(args[2]), txt_q=bf(args[3]), txt_k=bf(args[4]),
            txt_v=bf(args[5]), out_img=bf(out[0].reshape(B, Li, H, D)), out_txt=bf(out[1].reshape(B, Lt, H, D)))

    # head text, two actions, a gap window; padded text tokens; history holes
    run_case("basic", 1, 64, [(0, (5, 9))], 16, 3, [[1, 1, 1, 0, 1, 1, 1, 0]], [[2, 4, 6]],
             [[0, 1, 0], [1, 2, -1], [2, 3, 1]], False, 41)
    # two samples: offsets past the valid text (clamped), an uncovered frame; the second sample
    # has no offsets and keeps full attention
    run_case("batch", 2, 48, [(0, (0, 4)), (1, (20, 30))], 16, 3, [[1, 1, 1, 1, 1, 0], [1, 0, 1, 1, 0, 0]],
             [[1, 3, 7], None], [[0, 1, 1], [2, 3, 0]], False, 42)
    # empty history, empty head, cache write of the chunk
    run_case("nohist_update", 1, 0, [], 16, 3, [[1, 1, 1, 1]], [[0, 2, 3]], [[0, 2, 1], [2, 3, 0]], True, 43)



def make_swa():
    """Sliding-window (bounded) history through the reference: one call per segment with
    ``update_cache=True``; every call's inputs, outputs and the cache state it leaves."""
    native = importlib.import_module("hymm.models.dit.nomas_cpt")
    i8 = importlib.import_module("hymm.models.dit.modules.int8_kv_cache")
    H, D, T, Lt = 2, 128, 16, 3

    def run(name, fmt, capacity, frames_per_call, text_masks, seed):
        gen = torch.Generator().manual_seed(seed)
        cap = capacity + 8
        if fmt == "int8":
            cache = i8.make_int8_kv_block(1, cap, H, D, device="cpu")
        else:
            cache = {"k": torch.zeros(1, cap, H, D, dtype=torch.bfloat16),
                     "v": torch.zeros(1, cap, H, D, dtype=torch.bfloat16)}
        cache["swa_capacity"] = capacity
        mask = torch.zeros(1, cap, dtype=torch.bool)
        valid = 0
        d = {"capacity": capacity, "steps": len(frames_per_call), "cap": cap}
        for i, (nf, tm) in enumerate(zip(frames_per_call, text_masks)):
            args = [seeded((1, L, H, D), gen) for L in (nf * T, Lt) for _ in range(3)]
            tmask = torch.tensor([tm], dtype=torch.bool)
            with torch.no_grad():
                out = native.causal_attention_with_cache_mp(
                    (args[0], args[3]), (args[1], args[4]), (args[2], args[5]), cache, cache_valid_len=valid,
                    attn_mode="torch", text_mask=tmask, update_cache=True, cache_txt=True, cache_mask=mask,
                    tokens_per_frame=T)
            valid_before, valid = valid, int(cache["swa_valid_len"])
            recs = [[r.start, r.image_tokens, r.end, r.time_start, r.height, r.width] for r in cache["swa_video"]]
            for j, n in enumerate(("img_q", "img_k", "img_v", "txt_q", "txt_k", "txt_v")):
                d[f"{i}_{n}"] = bf(args[j])
            d[f"{i}_text_mask"] = tmask.numpy()
            d[f"{i}_valid_before"] = valid_before
            d[f"{i}_out_img"] = bf(out[0].reshape(1, nf * T, H, D))
            d[f"{i}_out_txt"] = bf(out[1].reshape(1, Lt, H, D))
            d[f"{i}_valid_after"] = valid
            d[f"{i}_evicted"] = int(cache["swa_evicted"])
            d[f"{i}_records"] = np.array(recs, dtype=np.int64).reshape(-1, 6)
            d[f"{i}_next_frame"] = int(cache["swa_next_frame"])
            d[f"{i}_mask"] = mask.numpy().copy()
            for key in ("k", "v", "k_scale", "v_scale"):
                if key in cache:
                    t = cache[key][:, :valid]
                    d[f"{i}_{key}"] = bf(t.clone()) if t.dtype == torch.bfloat16 else t.numpy().copy()
        np.savez_compressed(HERE / f"swa_{fmt}_{name}.npz", **d)

    # whole records, then one frame of a record (its text kept), then a record and a frame
    frames, masks = [2, 2, 3, 1, 2], [[1, 1, 1], [1, 1, 0], [1, 0, 1], [1, 1, 1], [0, 1, 1]]
    run("evict", "int8", 90, frames, masks, 51)
    run("evict", "bf16", 90, frames, masks, 52)
    # a chunk larger than the budget: the cut reaches into the current chunk
    run("overflow", "int8", 40, [2, 3, 1], [[1, 1, 1], [1, 1, 0], [1, 1, 1]], 53)


def main():
    _install_stub()
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    if "--only-intra" in sys.argv:
        make_intra_seg()
        return
    if "--only-swa" in sys.argv:
        make_swa()
        return
    if "--only-late" not in sys.argv:
        make_quant()
        make_attention()
    make_ring_merge()
    make_window()
    make_sp()
    make_config1()
    make_intra_seg()
    make_swa()
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
