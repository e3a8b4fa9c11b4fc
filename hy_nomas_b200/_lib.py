"""ctypes binding of ``libhyb200.so`` (the C ABI in ``include/hyb200.h``).

The library is loaded lazily from this package directory.  Every wrapper raises the
exception type the reference raises for the same condition (ValueError for bad
shapes / capacity / non-finite values, RuntimeError otherwise).  There is no CPU
fallback: a missing library or a non-sm_100 device is an error.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = PKG_DIR / "libhyb200.so"

HYB_ABI_VERSION = 5

HYB_OK = 0
HYB_ERR_INVALID_ARG = -1
HYB_ERR_UNSUPPORTED = -2
HYB_ERR_CUDA = -3
HYB_ERR_TIMEOUT = -4
HYB_ERR_NONFINITE = -5
HYB_ERR_CAPACITY = -6
HYB_ERR_WORKSPACE = -7

HYB_FMT_BF16 = 0
HYB_FMT_E4M3 = 1
HYB_FMT_INT8 = 2

HYB_DEV_TIMEOUT = 0x1
HYB_DEV_NONFINITE = 0x2

c_i32 = ctypes.c_int32
c_i64 = ctypes.c_int64
c_ptr = ctypes.c_void_p


class Tensor4(ctypes.Structure):
    """``hyb_tensor4``: a [B, L, H, D] view with unit stride on D."""

    _fields_ = [
        ("data", c_ptr), ("fmt", c_i32), ("pad_", c_i32),
        ("s_b", c_i64), ("s_t", c_i64), ("s_h", c_i64),
        ("scale", c_ptr), ("ss_b", c_i64), ("ss_t", c_i64), ("ss_h", c_i64),
    ]


class PartScatter(ctypes.Structure):
    """hyb_part_scatter: partial rows written to their owner ranks (KV-stationary schedule)."""

    _fields_ = [("o", c_ptr), ("lse", c_ptr), ("ranks", c_i32), ("rows", c_i32), ("index0", c_i32),
                ("count", c_i32), ("slices", c_i32), ("pad_", c_i32)]


class CachedAttnArgs(ctypes.Structure):
    """``hyb_cached_attn_args``."""

    _fields_ = [
        ("abi_version", c_i32), ("B", c_i32), ("H", c_i32), ("D", c_i32),
        ("cache_batch", c_i32), ("valid_len", c_i32), ("img_len", c_i32), ("txt_len", c_i32),
        ("attend_txt", c_i32), ("group_tokens", c_i32), ("softmax_scale", ctypes.c_float),
        ("q_pos0", c_i32), ("k_pos0", c_i32),
        ("hist_k", Tensor4), ("hist_v", Tensor4),
        ("img_q", Tensor4), ("img_k", Tensor4), ("img_v", Tensor4),
        ("txt_q", Tensor4), ("txt_k", Tensor4), ("txt_v", Tensor4),
        ("hist_rows", c_ptr), ("cache_mask", c_ptr), ("cache_mask_sb", c_i64),
        ("text_mask", c_ptr), ("text_mask_sb", c_i64),
        ("out_img", c_ptr), ("oi_sb", c_i64), ("oi_st", c_i64), ("oi_sh", c_i64),
        ("oi_seg", c_i64), ("oi_sseg", c_i64),
        ("out_txt", c_ptr), ("ot_sb", c_i64), ("ot_st", c_i64), ("ot_sh", c_i64),
        ("lse", c_ptr), ("workspace", c_ptr), ("workspace_bytes", c_i64),
        ("dev_status", c_ptr), ("img_k_len", c_i32), ("scatter", c_ptr),
        ("staged_k", c_ptr), ("staged_v", c_ptr), ("staged_pitch", c_i64),
    ]


class AttnArgs(ctypes.Structure):
    """``hyb_attn_args`` (the attention kernel over staged head-major tensors)."""

    _fields_ = [
        ("abi_version", c_i32), ("B", c_i32), ("H", c_i32), ("D", c_i32), ("Lq", c_i32),
        ("Lk", c_i32), ("hist_len", c_i32), ("img_len", c_i32), ("group_tokens", c_i32),
        ("softmax_scale", ctypes.c_float), ("q_pos0", c_i32), ("k_pos0", c_i32),
        ("img_k_len", c_i32), ("q_seg", c_i32), ("q_pos1", c_i32), ("k_seg", c_i32), ("k_pos1", c_i32),
        ("pad1_", c_i32),
        ("q", c_ptr), ("k", c_ptr), ("v", c_ptr),
        ("kbits", c_ptr), ("kwords", c_i32),
        ("qbits", c_ptr), ("qwords", c_i32),
        ("out_img", c_ptr), ("oi_sb", c_i64), ("oi_st", c_i64), ("oi_sh", c_i64),
        ("oi_seg", c_i64), ("oi_sseg", c_i64),
        ("out_txt", c_ptr), ("ot_sb", c_i64), ("ot_st", c_i64), ("ot_sh", c_i64),
        ("lse", c_ptr), ("dev_status", c_ptr),
        ("kv_splits", c_i32), ("v_f16", c_i32), ("part_o", c_ptr), ("part_lse", c_ptr),
        ("acc_o", c_ptr), ("acc_lse", c_ptr), ("acc_mode", c_i32), ("pad2_", c_i32),
        ("scatter", c_ptr),
    ]


class PeerSync(ctypes.Structure):
    """``hyb_peer_sync``."""

    _fields_ = [("flags", c_ptr * 64), ("state", c_ptr), ("dev_status", c_ptr)]


class WorkspaceLayout(ctypes.Structure):
    """``hyb_workspace_layout``."""

    _fields_ = [
        ("q", c_i64), ("k", c_i64), ("v", c_i64), ("kbits", c_i64), ("qbits", c_i64),
        ("part_o", c_i64), ("part_lse", c_i64), ("total", c_i64),
        ("Lq", c_i32), ("Lk", c_i32), ("kwords", c_i32), ("qwords", c_i32), ("kv_splits", c_i32),
        ("pad_", c_i32),
    ]


# name -> (restype, argtypes); every symbol declared in include/hyb200.h
SIGNATURES = {
    "hyb_stage_head_major": (c_i32, [c_i32, c_i32, c_i32, c_i32, ctypes.POINTER(Tensor4),
                                     ctypes.POINTER(Tensor4), c_ptr, c_ptr, c_ptr]),
    "hyb_fill_key_bits": (c_i32, [c_i32, c_i32, c_i32, c_ptr, c_ptr]),
    "hyb_attn_work_plan": (c_i32, [ctypes.POINTER(AttnArgs), c_i32, ctypes.POINTER(c_i32), c_i32]),
    "hyb_peer_alloc": (c_i32, [c_i64, ctypes.POINTER(c_ptr), c_ptr]),
    "hyb_peer_push_bytes": (c_i32, [c_i32, c_i32, c_ptr, c_i64, ctypes.POINTER(c_ptr), ctypes.POINTER(PeerSync),
                                    c_ptr]),
    "hyb_peer_push_bytes_n": (c_i32, [c_i32, c_i32, c_ptr, c_i64, ctypes.POINTER(c_ptr), ctypes.POINTER(PeerSync),
                                      c_i32, c_ptr]),
    "hyb_ring_gather_stage": (c_i32, [c_i32, c_i32, c_i32, c_i32, c_i32, c_i32, ctypes.POINTER(c_ptr), c_i32,
                                      ctypes.POINTER(c_i32), ctypes.POINTER(c_i32), ctypes.POINTER(c_i32),
                                      c_ptr, c_ptr, c_i32, c_ptr]),
    "hyb_peer_open": (c_i32, [c_ptr, ctypes.POINTER(c_ptr)]),
    "hyb_peer_close": (c_i32, [c_ptr]),
    "hyb_peer_free": (c_i32, [c_ptr]),
    "hyb_ulysses_push_qkv": (c_i32, [c_i32, c_i32, c_i32, c_i32, c_i32, c_i32, ctypes.POINTER(Tensor4),
                                     ctypes.POINTER(Tensor4), ctypes.POINTER(Tensor4), ctypes.POINTER(c_ptr),
                                     ctypes.POINTER(PeerSync), c_ptr]),
    "hyb_ulysses_push_o": (c_i32, [c_i32, c_i32, c_i32, c_i32, c_i32, c_i32, c_i32, c_ptr, ctypes.POINTER(Tensor4),
                                   ctypes.POINTER(c_ptr), ctypes.POINTER(c_ptr), ctypes.POINTER(PeerSync), c_ptr]),
    "hyb_version": (c_i32, []),
    "hyb_last_error": (c_i32, [ctypes.c_char_p, ctypes.c_size_t]),
    "hyb_device_supported": (c_i32, []),
    "hyb_kv_append_pair": (c_i32, [c_i32, c_i32, c_i32, c_i32, c_i32, c_i64, c_i64,
                                   ctypes.POINTER(Tensor4), ctypes.POINTER(Tensor4),
                                   c_i32, ctypes.POINTER(Tensor4), ctypes.POINTER(Tensor4),
                                   c_ptr, c_ptr, c_i64, c_i64, c_i64,
                                   c_ptr, c_ptr, c_i64, c_i64, c_i64, c_ptr, c_ptr]),
    "hyb_check_finite": (c_i32, [ctypes.POINTER(Tensor4), c_i32, c_i32, c_i32, c_i32, c_ptr, c_ptr]),
    "hyb_kv_dequant": (c_i32, [ctypes.POINTER(Tensor4), c_i32, c_i32, c_i32, c_i32, c_ptr, c_ptr]),
    "hyb_cached_attention_workspace_bytes": (c_i64, [c_i32, c_i32, c_i32, c_i32, c_i32, c_i32, c_i32]),
    "hyb_cached_attention_workspace_bytes_ex": (c_i64, [c_i32, c_i32, c_i32, c_i32, c_i32, c_i32, c_i32, c_i32]),
    "hyb_decode_rows": (c_i32, [c_i32, c_i32, c_i32, c_i32, ctypes.POINTER(Tensor4), ctypes.POINTER(Tensor4),
                                c_ptr, c_ptr, c_i64, c_i64, c_ptr]),
    "hyb_cached_attention_workspace_layout": (c_i32, [c_i32, c_i32, c_i32, c_i32, c_i32, c_i32, c_i32,
                                                       ctypes.POINTER(WorkspaceLayout)]),
    "hyb_cached_attention": (c_i32, [ctypes.POINTER(CachedAttnArgs), c_ptr]),
    "hyb_cached_attention_noalloc": (c_i32, [ctypes.POINTER(CachedAttnArgs), c_ptr]),
    "hyb_attn_fwd": (c_i32, [ctypes.POINTER(AttnArgs), c_ptr]),
    "hyb_lse_merge": (c_i32, [c_i32, c_i32, c_i32, c_ptr, c_ptr, c_ptr, c_i32, c_ptr, c_ptr]),
    "hyb_merge_partials": (c_i32, [c_i32, c_i32, c_i32, c_i32, c_i32, c_i32, c_ptr, c_ptr,
                                   c_ptr, c_i64, c_i64, c_i64, c_ptr, c_i64, c_i64, c_i64,
                                   c_ptr, c_i64, c_ptr, c_ptr]),
    "hyb_ulysses_pack_qkv": (c_i32, [c_i32, c_i32, c_i32, c_i32, c_i32, c_i32,
                                     ctypes.POINTER(Tensor4), ctypes.POINTER(Tensor4),
                                     ctypes.POINTER(Tensor4), c_ptr, c_ptr]),
    "hyb_ulysses_pack_o": (c_i32, [c_i32, c_i32, ctypes.POINTER(c_i32), c_i32, c_i32, c_i32,
                                   ctypes.POINTER(Tensor4), c_ptr, c_ptr]),
    "hyb_ulysses_unpack_o": (c_i32, [c_i32, c_i32, c_i32, c_i32, c_i32, c_i32, c_ptr, c_ptr,
                                     c_i64, c_i64, c_i64, c_ptr]),
    "hyb_exp2_poly_eval": (c_i32, [c_ptr, c_ptr, c_i64, c_ptr]),
    "hyb_peer_barrier": (c_i32, [c_i32, c_i32, ctypes.POINTER(PeerSync), c_ptr]),
}

_LIB = None


def load(path: str | os.PathLike | None = None) -> ctypes.CDLL:
    """Load (once) and return the library; raises RuntimeError if it is missing."""
    global _LIB
    if _LIB is not None and path is None:
        return _LIB
    p = Path(path) if path is not None else LIB_PATH
    if not p.exists():
        raise RuntimeError(
            f"{p} is missing: build the CUDA extension first "
            "(python -m hy_nomas_b200.build or __graft_entry__.build())")
    lib = ctypes.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if lib.hyb_version() != HYB_ABI_VERSION:
        raise RuntimeError("libhyb200.so ABI version mismatch; rebuild the extension")
    if path is None:
        _LIB = lib
    return lib


def last_error() -> str:
    lib = load()
    buf = ctypes.create_string_buffer(1024)
    lib.hyb_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc: int, what: str) -> None:
    """Translate a C status into the reference's exception types."""
    if rc == HYB_OK:
        return
    msg = f"{what}: {last_error()}"
    if rc in (HYB_ERR_INVALID_ARG, HYB_ERR_CAPACITY, HYB_ERR_NONFINITE):
        raise ValueError(msg)
    raise RuntimeError(msg)


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def bf16_view(t: torch.Tensor) -> Tensor4:
    """[B, L, H, D] bf16 tensor -> Tensor4."""
    if t.dtype != torch.bfloat16 or t.ndim != 4:
        raise TypeError("expected a [B, L, H, D] bfloat16 tensor")
    st = t.stride()
    if st[3] != 1:
        raise ValueError("head_dim must be the contiguous dimension")
    return Tensor4(t.data_ptr(), HYB_FMT_BF16, 0, st[0], st[1], st[2], None, 0, 0, 0)


def coded_view(codes: torch.Tensor, scale: torch.Tensor, fmt: int) -> Tensor4:
    """Quantised cache (codes [B, L, H, D], fp32 scale [B, L, H, 1]) -> Tensor4."""
    st, ss = codes.stride(), scale.stride()
    if st[3] != 1:
        raise ValueError("head_dim must be the contiguous dimension")
    return Tensor4(codes.data_ptr(), fmt, 0, st[0], st[1], st[2], scale.data_ptr(), ss[0], ss[1], ss[2])


_STATUS: dict[int, torch.Tensor] = {}


def device_status(device: torch.device) -> torch.Tensor:
    """Per-device int32 status word the kernels OR HYB_DEV_* bits into."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _STATUS.get(idx)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _STATUS[idx] = t
    return t


def check_device_status(device: torch.device, reset: bool = True) -> None:
    """Synchronise with the device status word and raise on a recorded fault."""
    t = device_status(device)
    val = int(t.item())
    if reset and val:
        t.zero_()
    if val & HYB_DEV_TIMEOUT:
        raise RuntimeError("hyb200: a device-side wait timed out (kernel aborted its tile loop)")
    if val & HYB_DEV_NONFINITE:
        raise ValueError("Cannot quantize non-finite KV values")


def require_same_device(device: torch.device, what: str, *tensors) -> None:
    """Every tensor the kernels will read or write through a raw pointer must live on ``device``
    (a host tensor's pointer would be dereferenced on the GPU).  None entries are skipped; a
    CUDA device given without an index means the current one."""
    device = torch.device(device)
    if device.type == "cuda" and device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    for t in tensors:
        if t is not None and t.device != device:
            raise RuntimeError(f"{what} must be on the same device: found {t.device}, expected {device}")


def require_device(t: torch.Tensor) -> None:
    if not t.is_cuda:
        raise RuntimeError("hy_nomas_b200 kernels need CUDA tensors (no CPU path)")
    lib = load()
    with torch.cuda.device(t.device):
        if lib.hyb_device_supported() != 1:
            raise RuntimeError("hy_nomas_b200 kernels need an sm_100 (B200) device")
