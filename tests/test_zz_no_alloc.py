"""The allocation-free cached attention entry point (``hyb_cached_attention_noalloc``).

It exists for callers that cannot allocate device memory when they call attention — a
framework that has already reserved the device's memory in its own pool, a decode loop that
must not risk cudaMalloc's device synchronisation, or an FFI host without an allocator — and
keeps its staging scratch in a fixed static device array instead of a caller workspace.

This file is collected last so a run that stops at the first failure has run every other test
before it.  It drives the entry point through the C ABI on two calls in a row (different
inputs, so a stale scratch would show) and compares each result with the workspace-based
entry point ``hyb_cached_attention`` under the attention tests' tolerance."""
import ctypes

import pytest
import torch

from hy_nomas_b200 import _lib
from hy_nomas_b200 import attention as hatt
from hy_nomas_b200.synthetic import make_generator, seeded_kv
from oracle import quant as oq

pytestmark = pytest.mark.gpu

ATOL = 2e-2
RTOL = 2.0 ** -7
COS = 0.9995


def _case(seed, dev, H=2, Lh=1000, Li=384, Lt=3):
    gen = make_generator(seed)
    hk, hv = seeded_kv((1, Lh, H, 128), gen), seeded_kv((1, Lh, H, 128), gen)
    cur = [seeded_kv((1, L, H, 128), gen).to(dev) for L in (Li, Lt) for _ in range(3)]
    ck, sk = oq.quantize_e4m3(hk)
    cv, sv = oq.quantize_e4m3(hv)
    cache = {"k": ck.to(dev), "v": cv.to(dev), "k_scale": sk.to(dev), "v_scale": sv.to(dev),
             "storage_format": "fp8_e4m3"}
    hmask = torch.ones(1, Lh, dtype=torch.bool, device=dev)
    hmask[:, 10:40] = False
    tmask = torch.tensor([[True, False, True]], device=dev)
    return cache, cur, hmask, tmask


def _args(cache, cur, hmask, tmask, out_img, out_txt, group_tokens):
    img_q, img_k, img_v, txt_q, txt_k, txt_v = cur
    a = _lib.CachedAttnArgs()
    a.abi_version = _lib.HYB_ABI_VERSION
    a.B, a.H, a.D = img_q.shape[0], img_q.shape[2], 128
    a.cache_batch = cache["k"].shape[0]
    a.valid_len = cache["k"].shape[1]
    a.img_len, a.txt_len = img_q.shape[1], txt_q.shape[1]
    a.attend_txt = 1
    a.group_tokens = group_tokens
    a.softmax_scale = 0.0
    a.hist_k = _lib.coded_view(cache["k"], cache["k_scale"], _lib.HYB_FMT_E4M3)
    a.hist_v = _lib.coded_view(cache["v"], cache["v_scale"], _lib.HYB_FMT_E4M3)
    a.img_q, a.img_k, a.img_v = (_lib.bf16_view(t) for t in (img_q, img_k, img_v))
    a.txt_q, a.txt_k, a.txt_v = (_lib.bf16_view(t) for t in (txt_q, txt_k, txt_v))
    a.hist_rows = None
    a.cache_mask, a.cache_mask_sb = hmask.data_ptr(), hmask.stride(0)
    a.text_mask, a.text_mask_sb = tmask.data_ptr(), tmask.stride(0)
    a.out_img = out_img.data_ptr()
    a.oi_sb, a.oi_st, a.oi_sh = out_img.stride()[:3]
    a.oi_seg, a.oi_sseg = 0, 0
    a.out_txt = out_txt.data_ptr()
    a.ot_sb, a.ot_st, a.ot_sh = out_txt.stride()[:3]
    a.lse = None
    a.workspace, a.workspace_bytes = None, 0      # ignored by the allocation-free entry point
    a.dev_status = _lib.device_status(out_img.device).data_ptr()
    return a


def _close(out, ref):
    o, r = out.float().flatten(), ref.float().flatten()
    assert ((o - r).abs() <= ATOL + RTOL * r.abs()).all()
    assert torch.nn.functional.cosine_similarity(o[None], r[None]).item() >= COS


def test_no_alloc_entry_point_matches_workspace_entry_point():
    assert torch.cuda.is_available(), "GPU test run without a CUDA device"
    lib = _lib.load()
    assert lib.hyb_device_supported() == 1
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    for call, seed in enumerate((301, 302)):
        cache, cur, hmask, tmask = _case(seed, dev)
        G = 128
        ref_img, ref_txt = hatt.cached_attention_local(*cur, cache, cache["k"].shape[1], history_mask=hmask,
                                                       text_mask=tmask, group_tokens=G)
        out_img = torch.full_like(ref_img, float("nan"))
        out_txt = torch.full_like(ref_txt, float("nan"))
        args = _args(cache, cur, hmask, tmask, out_img, out_txt, G)
        rc = lib.hyb_cached_attention_noalloc(ctypes.byref(args), stream)
        assert rc == _lib.HYB_OK, _lib.last_error()
        torch.cuda.synchronize(dev)
        _lib.check_device_status(dev)
        _close(out_img, ref_img)
        _close(out_txt, ref_txt)


def test_no_alloc_entry_point_rejects_oversized_problems():
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    cache, cur, hmask, tmask = _case(303, dev, H=1, Lh=64, Li=32, Lt=3)
    out_img = torch.empty(1, 32, 1, 128, dtype=torch.bfloat16, device=dev)
    out_txt = torch.empty(1, 3, 1, 128, dtype=torch.bfloat16, device=dev)
    args = _args(cache, cur, hmask, tmask, out_img, out_txt, 0)
    args.H = 64                      # staging for 64 heads x 1,000,000 keys exceeds the fixed scratch
    args.valid_len = 1_000_000
    rc = lib.hyb_cached_attention_noalloc(ctypes.byref(args), torch.cuda.current_stream(dev).cuda_stream)
    assert rc == _lib.HYB_ERR_WORKSPACE
    assert "fixed per-device scratch" in _lib.last_error()


def test_no_alloc_entry_point_reports_negative_sizes_as_invalid_arguments():
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    cache, cur, hmask, tmask = _case(304, dev, H=1, Lh=64, Li=32, Lt=3)
    out_img = torch.empty(1, 32, 1, 128, dtype=torch.bfloat16, device=dev)
    out_txt = torch.empty(1, 3, 1, 128, dtype=torch.bfloat16, device=dev)
    args = _args(cache, cur, hmask, tmask, out_img, out_txt, 0)
    args.valid_len = -5
    rc = lib.hyb_cached_attention_noalloc(ctypes.byref(args), torch.cuda.current_stream(dev).cuda_stream)
    assert rc == _lib.HYB_ERR_INVALID_ARG
    assert "negative sizes" in _lib.last_error()
    args.valid_len, args.D = 64, 64
    rc = lib.hyb_cached_attention_noalloc(ctypes.byref(args), torch.cuda.current_stream(dev).cuda_stream)
    assert rc == _lib.HYB_ERR_UNSUPPORTED
