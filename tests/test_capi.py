"""The C ABI without a GPU: the library loads, exports every symbol the header declares,
the ctypes mirrors have the C struct layouts, and argument errors come back as status
codes (no device work is attempted for rejected calls)."""
import ctypes
import re
import shutil
import subprocess
from pathlib import Path

import pytest
import torch

from hy_nomas_b200 import _lib

REPO = Path(__file__).resolve().parent.parent
HEADER = REPO / "include" / "hyb200.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(hyb_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_functions()
    assert len(names) >= 12
    for name in names:
        assert hasattr(lib, name), f"{name} missing from libhyb200.so"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"
    assert lib.hyb_version() == _lib.HYB_ABI_VERSION


LAYOUT_C = r"""
#include <stdio.h>
#include <stddef.h>
#include "hyb200.h"
#define F(T, m) printf(#T "." #m " %zu\n", offsetof(T, m));
int main(void) {
  printf("hyb_tensor4 %zu\n", sizeof(hyb_tensor4));
  printf("hyb_cached_attn_args %zu\n", sizeof(hyb_cached_attn_args));
  printf("hyb_attn_args %zu\n", sizeof(hyb_attn_args));
  F(hyb_tensor4, scale) F(hyb_tensor4, ss_h)
  F(hyb_cached_attn_args, softmax_scale) F(hyb_cached_attn_args, k_pos0) F(hyb_cached_attn_args, hist_k)
  F(hyb_cached_attn_args, txt_v) F(hyb_attn_args, k_pos0)
  F(hyb_cached_attn_args, hist_rows) F(hyb_cached_attn_args, cache_mask) F(hyb_cached_attn_args, oi_seg)
  F(hyb_cached_attn_args, out_txt) F(hyb_cached_attn_args, lse) F(hyb_cached_attn_args, workspace_bytes)
  F(hyb_cached_attn_args, dev_status) F(hyb_cached_attn_args, img_k_len) F(hyb_cached_attn_args, scatter)
  F(hyb_cached_attn_args, staged_k) F(hyb_cached_attn_args, staged_pitch)
  F(hyb_attn_args, q) F(hyb_attn_args, kwords) F(hyb_attn_args, qbits) F(hyb_attn_args, oi_sseg)
  F(hyb_attn_args, lse) F(hyb_attn_args, dev_status) F(hyb_attn_args, kv_splits) F(hyb_attn_args, v_f16) F(hyb_attn_args, part_lse)
  F(hyb_attn_args, img_k_len) F(hyb_attn_args, k_pos1) F(hyb_attn_args, acc_o) F(hyb_attn_args, acc_mode)
  F(hyb_attn_args, scatter)
  printf("hyb_part_scatter %zu\n", sizeof(hyb_part_scatter));
  F(hyb_part_scatter, lse) F(hyb_part_scatter, ranks) F(hyb_part_scatter, count) F(hyb_part_scatter, slices)
  printf("hyb_peer_sync %zu\n", sizeof(hyb_peer_sync));
  F(hyb_peer_sync, state) F(hyb_peer_sync, dev_status)
  printf("hyb_workspace_layout %zu\n", sizeof(hyb_workspace_layout));
  F(hyb_workspace_layout, total) F(hyb_workspace_layout, kv_splits)
  return 0;
}
"""


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_ctypes_layouts_match_c(tmp_path):
    src = tmp_path / "layout.c"
    src.write_text(LAYOUT_C)
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", str(REPO / "include"), str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    c = dict(line.rsplit(" ", 1) for line in out.strip().splitlines())
    types = {"hyb_tensor4": _lib.Tensor4, "hyb_cached_attn_args": _lib.CachedAttnArgs,
             "hyb_attn_args": _lib.AttnArgs, "hyb_workspace_layout": _lib.WorkspaceLayout,
             "hyb_peer_sync": _lib.PeerSync, "hyb_part_scatter": _lib.PartScatter}
    for key, val in c.items():
        if "." in key:
            t, m = key.split(".")
            assert getattr(types[t], m).offset == int(val), key
        else:
            assert ctypes.sizeof(types[key]) == int(val), key


def test_status_codes_for_rejected_calls():
    lib = _lib.load()
    x = _lib.Tensor4(16, _lib.HYB_FMT_BF16, 0, 8, 8, 8, None, 0, 0, 0)
    # head_dim other than 128 is unsupported
    rc = lib.hyb_kv_append_pair(_lib.HYB_FMT_E4M3, 1, 4, 1, 64, 8, 0, x, x, 0, None, None, 16, 16, 8, 8, 8,
                                16, 16, 1, 1, 1, None, None)
    assert rc == _lib.HYB_ERR_UNSUPPORTED and "head_dim" in _lib.last_error()
    # writing past the capacity is a capacity error (ValueError in Python)
    rc = lib.hyb_kv_append_pair(_lib.HYB_FMT_INT8, 1, 4, 1, 128, 8, 6, x, x, 0, None, None, 16, 16, 8, 8, 8,
                                16, 16, 1, 1, 1, None, None)
    assert rc == _lib.HYB_ERR_CAPACITY
    with pytest.raises(ValueError):
        _lib.check(rc, "KV quantization")
    # bf16 is not a quantised storage format
    rc = lib.hyb_kv_append_pair(_lib.HYB_FMT_BF16, 1, 4, 1, 128, 8, 0, x, x, 0, None, None, 16, 16, 8, 8, 8,
                                16, 16, 1, 1, 1, None, None)
    assert rc == _lib.HYB_ERR_UNSUPPORTED
    # SP head counts must divide
    rc = lib.hyb_ulysses_pack_qkv(3, 1, 4, 4, 8, 128, x, x, x, 16, None)
    assert rc == _lib.HYB_ERR_INVALID_ARG
    assert lib.hyb_cached_attention_workspace_bytes(1, 2, 64, 10, 10, 1, 1) == -1
    assert lib.hyb_cached_attention_workspace_bytes(1, 2, 128, 10, 10, 1, 1) > 0
    args = _lib.CachedAttnArgs()
    args.abi_version = 99
    assert lib.hyb_cached_attention(args, None) == _lib.HYB_ERR_INVALID_ARG


def test_partial_scatter_arguments_are_checked_before_any_launch():
    """A bad hyb_part_scatter (no slices, too few owner rows for the image queries, a ring
    accumulator at the same time) and a bad owner merge are argument errors; nothing runs."""
    lib = _lib.load()
    table = (ctypes.c_void_p * 2)(16, 32)
    a = _lib.AttnArgs()
    a.abi_version = _lib.HYB_ABI_VERSION
    a.B, a.H, a.D, a.Lq, a.Lk, a.img_len, a.img_k_len = 1, 2, 128, 300, 100, 300, 100
    a.q = a.k = a.v = 256
    a.kbits, a.kwords = 256, 4
    for ranks, rows, slices, index0, count in ((2, 150, 0, 0, 2), (2, 100, 1, 0, 2), (2, 150, 2, 1, 2)):
        sc = _lib.PartScatter(ctypes.cast(table, ctypes.c_void_p), ctypes.cast(table, ctypes.c_void_p),
                              ranks, rows, index0, count, slices, 0)
        a.scatter = ctypes.cast(ctypes.pointer(sc), ctypes.c_void_p)
        assert lib.hyb_attn_fwd(ctypes.byref(a), None) == _lib.HYB_ERR_INVALID_ARG
        assert "scatter" in _lib.last_error() or "own" in _lib.last_error()
    assert lib.hyb_merge_partials(1, 1, 2, 64, 4, 0, 256, 256, 256, 8, 8, 8, None, 0, 0, 0, None, 0, None,
                                  None) == _lib.HYB_ERR_UNSUPPORTED
    assert lib.hyb_merge_partials(0, 1, 2, 128, 4, 0, 256, 256, 256, 8, 8, 8, None, 0, 0, 0, None, 0, None,
                                  None) == _lib.HYB_ERR_INVALID_ARG
    c = _lib.CachedAttnArgs()
    c.abi_version = _lib.HYB_ABI_VERSION
    c.B, c.H, c.D, c.cache_batch, c.img_len, c.img_k_len = 1, 2, 128, 1, 64, 32
    assert lib.hyb_cached_attention(ctypes.byref(c), None) == _lib.HYB_ERR_INVALID_ARG
    assert "img_k_len" in _lib.last_error()


def test_workspace_size_formula():
    lib = _lib.load()
    B, H, Lh, Li, Lt = 1, 24, 24960, 6240, 1
    ws = lib.hyb_cached_attention_workspace_bytes(B, H, 128, Lh, Li, Lt, 1)
    Lk, Lq = Lh + Li + Lt, Li + Lt
    assert ws >= B * H * (Lq + 2 * Lk) * 128 * 2
    assert ws < B * H * (Lq + 2 * Lk) * 128 * 2 + 1 << 20


def test_staged_history_workspace_and_argument_checks():
    """A call with a pre-decoded history needs no K/V staging area, and its buffers must be
    given together, aligned, with a pitch that covers the history and the call's own keys;
    hyb_decode_rows rejects rows outside the pitch and bf16 sources.  Nothing runs."""
    lib = _lib.load()
    B, H, Lh, Li, Lt = 1, 24, 51480, 1560, 1
    full = lib.hyb_cached_attention_workspace_bytes_ex(B, H, 128, Lh, Li, Lt, 1, 0)
    staged = lib.hyb_cached_attention_workspace_bytes_ex(B, H, 128, Lh, Li, Lt, 1, 1)
    assert full == lib.hyb_cached_attention_workspace_bytes(B, H, 128, Lh, Li, Lt, 1)
    assert full - staged == 2 * B * H * (Lh + Li + Lt) * 128 * 2
    c = _lib.CachedAttnArgs()
    c.abi_version = _lib.HYB_ABI_VERSION
    c.B, c.H, c.D, c.cache_batch, c.valid_len, c.img_len, c.txt_len, c.attend_txt = 1, 2, 128, 1, 256, 64, 0, 1
    c.workspace, c.workspace_bytes = 256, 1 << 40
    c.staged_k, c.staged_v, c.staged_pitch = 256, 512, 256 + 63   # one row short of the call's keys
    assert lib.hyb_cached_attention(ctypes.byref(c), None) == _lib.HYB_ERR_INVALID_ARG
    assert "pitch" in _lib.last_error()
    c.staged_pitch, c.staged_v = 320, None
    assert lib.hyb_cached_attention(ctypes.byref(c), None) == _lib.HYB_ERR_INVALID_ARG
    codes = _lib.Tensor4()
    codes.data, codes.fmt, codes.scale = 256, _lib.HYB_FMT_E4M3, 512
    codes.s_b, codes.s_t, codes.s_h = 128 * 2 * 64, 128 * 2, 128
    assert lib.hyb_decode_rows(1, 64, 2, 128, ctypes.byref(codes), ctypes.byref(codes), 256, 512, 100, 40,
                               None) == _lib.HYB_ERR_INVALID_ARG
    bf = _lib.Tensor4()
    bf.data, bf.fmt, bf.s_b, bf.s_t, bf.s_h = 256, _lib.HYB_FMT_BF16, 128 * 2 * 64, 128 * 2, 128
    assert lib.hyb_decode_rows(1, 64, 2, 128, ctypes.byref(bf), ctypes.byref(bf), 256, 512, 128, 0,
                               None) == _lib.HYB_ERR_UNSUPPORTED


def test_no_device_is_reported_not_faked():
    lib = _lib.load()
    if torch.cuda.is_available():
        pytest.skip("CPU-only check")
    assert lib.hyb_device_supported() == 0


def test_workspace_layout_is_consistent():
    from hy_nomas_b200.attention import workspace_layout
    lib = _lib.load()
    for args in [(1, 24, 24960, 6240, 1, 1), (2, 3, 0, 130, 2, 0), (1, 1, 7, 1, 0, 1), (3, 5, 1000, 384, 9, 1),
                 (1, 3, 74880, 6240, 1, 1)]:
        B, H, Lh, Li, Lt, att = args
        lay = workspace_layout(B, H, Lh, Li, Lt, att)
        assert lay.total == lib.hyb_cached_attention_workspace_bytes(B, H, 128, Lh, Li, Lt, att)
        assert lay.Lq == Li + Lt and lay.Lk == Lh + Li + (Lt if att else 0)
        assert lay.q == 0 < lay.k < lay.v < lay.kbits < lay.qbits <= lay.part_o <= lay.part_lse <= lay.total
        assert all(x % 256 == 0 for x in (lay.k, lay.v, lay.kbits, lay.qbits, lay.part_o, lay.part_lse))
        assert 1 <= lay.kv_splits <= 16
        if lay.kv_splits > 1:
            assert lay.part_lse - lay.part_o >= lay.kv_splits * B * H * lay.Lq * 128 * 4


def _plan_args(Lh, Li, Lt, H, G, cap):
    a = _lib.AttnArgs()
    a.abi_version = _lib.HYB_ABI_VERSION
    a.B, a.H, a.D = 1, H, 128
    a.Lq, a.Lk, a.hist_len, a.img_len, a.group_tokens = Li + Lt, Lh + Li + Lt, Lh, Li, G
    a.q = a.k = a.v = a.kbits = a.out_img = a.out_txt = a.part_o = a.part_lse = 256  # never dereferenced
    a.kwords = ((a.Lk + 127) // 128) * 4
    a.oi_sb = a.oi_st = a.oi_sh = a.ot_sb = a.ot_st = a.ot_sh = 8
    a.oi_seg = max(Li, 1)
    a.kv_splits = cap
    return a


@pytest.mark.parametrize("H,cap", [(24, 4), (3, 7), (2, 1)])
def test_work_plan_is_bounded_and_covers_every_pair(H, cap, monkeypatch):
    """The host-side launch planner: one slice count per query pair, within the partial-buffer
    capacity, heavier pairs never cut into fewer slices than lighter ones of the same chunk;
    HYB_KV_SPLITS forces a uniform count."""
    monkeypatch.delenv("HYB_KV_SPLITS", raising=False)
    lib = _lib.load()
    a = _plan_args(24960, 6240, 1, H, 1560, cap)
    ks = (ctypes.c_int32 * 64)()
    n = lib.hyb_attn_work_plan(ctypes.byref(a), 148, ks, 64)
    assert n == 25
    k = list(ks[:n])
    assert all(1 <= x <= cap for x in k)
    assert k == sorted(k)            # later query pairs see more frames of the chunk
    monkeypatch.setenv("HYB_KV_SPLITS", "3")
    n = lib.hyb_attn_work_plan(ctypes.byref(a), 148, ks, 64)
    assert list(ks[:n]) == [min(3, cap)] * 25
    a.D = 64
    assert lib.hyb_attn_work_plan(ctypes.byref(a), 148, ks, 64) == _lib.HYB_ERR_UNSUPPORTED
