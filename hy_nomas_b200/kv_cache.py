"""Quantised KV cache storage: the reference's INT8 format and the E4M3 extension.

Mirrors ``hymm/models/dit/modules/int8_kv_cache.py`` (``make_int8_kv_block`` :92-107,
``quantize_kv_into`` :125-158, ``quantize_kv_pair_into`` :161-179, ``dequantize_kv``
:182-205) and ``kv_cache_storage.py`` (``cache_format`` :6-10, ``cache_geometry``
:13-16, ``quantization_mode`` :19-23) with the same names, argument meanings and
exceptions.  The E4M3 variant keeps the reference's granularity (one fp32 scale per
token per head), its absmax rule and its API, with a 448 denominator and an RNE cast
to ``float8_e4m3fn``; a cache dict carries ``storage_format = "fp8_e4m3"``.

Every write and decode runs in the sm_100a library; there is no CPU path.
"""
from __future__ import annotations

import torch

from . import _lib

KV_KEYS = ("k", "v")
STORAGE_KEYS = ("k", "v", "k_scale", "v_scale")
FP8_FORMAT = "fp8_e4m3"
QUANTIZATION_MODES = ("none", "int8", "qvg", FP8_FORMAT)


# ----------------------------------------------------------------- format dispatch
def cache_format(cache: dict) -> str:
    """``none`` / ``int8`` / ``fp8_e4m3`` / ``qvg`` (kv_cache_storage.py:6-10)."""
    mode = cache.get("storage_format")
    if mode is not None:
        return mode
    dt = cache["k"].dtype
    if dt == torch.int8:
        return "int8"
    if dt == torch.float8_e4m3fn:
        return FP8_FORMAT
    return "none"


def cache_geometry(cache: dict):
    if cache_format(cache) == "qvg":
        return cache["shape"], cache["device"], torch.bfloat16
    return cache["k"].shape, cache["k"].device, cache["k"].dtype


def quantization_mode(inference) -> str:
    mode = getattr(inference, "kv_cache_quantization", "none")
    if mode not in QUANTIZATION_MODES:
        raise ValueError("inference.kv_cache_quantization must be none, int8, qvg, or fp8_e4m3")
    return mode


def is_int8_kv_cache(cache: dict) -> bool:
    return cache["k"].dtype == torch.int8


def is_fp8_kv_cache(cache: dict) -> bool:
    return cache["k"].dtype == torch.float8_e4m3fn


def _fmt_code(cache: dict) -> int:
    if is_int8_kv_cache(cache):
        return _lib.HYB_FMT_INT8
    if is_fp8_kv_cache(cache):
        return _lib.HYB_FMT_E4M3
    raise TypeError("INT8 or E4M3 KV data and FP32 scale are required")


# ----------------------------------------------------------------- containers
def _make_block(batch, capacity, heads, dim, dtype, device, pin_memory):
    value_shape = (batch, capacity, heads, dim)
    scale_shape = (batch, capacity, heads, 1)
    return {
        "k": torch.empty(value_shape, device=device, dtype=dtype, pin_memory=pin_memory),
        "v": torch.empty(value_shape, device=device, dtype=dtype, pin_memory=pin_memory),
        "k_scale": torch.empty(scale_shape, device=device, dtype=torch.float32, pin_memory=pin_memory),
        "v_scale": torch.empty(scale_shape, device=device, dtype=torch.float32, pin_memory=pin_memory),
    }


def make_int8_kv_block(batch: int, capacity: int, heads: int, dim: int, *,
                       device, pin_memory: bool = False, decoded: bool = False, tail_rows: int = 0) -> dict:
    """int8 codes [B, cap, H, D] + fp32 scales [B, cap, H, 1] (int8_kv_cache.py:92-107);
    ``decoded``: also keep the rows decoded (attach_decoded_mirror)."""
    block = _make_block(batch, capacity, heads, dim, torch.int8, device, pin_memory)
    return attach_decoded_mirror(block, tail_rows) if decoded else block


def make_fp8_kv_block(batch: int, capacity: int, heads: int, dim: int, *,
                      device, pin_memory: bool = False, decoded: bool = False, tail_rows: int = 0) -> dict:
    """float8_e4m3fn codes [B, cap, H, D] + fp32 scales [B, cap, H, 1]; ``decoded``: also keep
    the rows decoded (attach_decoded_mirror)."""
    block = _make_block(batch, capacity, heads, dim, torch.float8_e4m3fn, device, pin_memory)
    block["storage_format"] = FP8_FORMAT
    return attach_decoded_mirror(block, tail_rows) if decoded else block


def attach_decoded_mirror(cache: dict, tail_rows: int = 0) -> dict:
    """Keep a quantised cache decoded as well: ``cache["staged"] = (K, V, pitch)``, head-major
    bf16 K / fp16 V [B, H, cap + tail_rows, D] holding bf16(code * scale) of every row (the values
    the attention's staging pass would produce).  Every write through this module decodes the
    rows it wrote, so a call reads its history from here instead of decoding the whole cache
    (the reference's dequantize_kv per call, nomas_cpt.py:529-531, int8_kv_cache.py:182-205).
    A call stages its own keys into the rows after its history, so the capacity (or
    ``tail_rows``) must cover history + current keys.  Rows written to the codes by other means
    need refresh_decoded.  Returns the cache."""
    _fmt_code(cache)   # quantised storage only
    B, cap, H, D = cache["k"].shape
    dev = cache["k"].device
    pitch = cap + int(tail_rows)
    cache["staged"] = (torch.empty(B, H, pitch, D, dtype=torch.bfloat16, device=dev),
                       torch.empty(B, H, pitch, D, dtype=torch.float16, device=dev), pitch)
    refresh_decoded(cache, 0, cap)
    return cache


def refresh_decoded(cache: dict, start: int, n: int) -> None:
    """Decode rows [start, start + n) of the codes into the cache's decoded mirror (no-op
    without one)."""
    staged = cache.get("staged")
    if staged is None or n <= 0:
        return
    lib = _lib.load()
    fmt = _fmt_code(cache)
    k, v, ks, vs = cache["k"], cache["v"], cache["k_scale"], cache["v_scale"]
    if start < 0 or start + n > k.shape[1]:
        raise ValueError("decoded rows outside the cache")
    _lib.require_device(k)
    rows = slice(start, start + n)
    src_k = _lib.coded_view(k[:, rows], ks[:, rows], fmt)
    src_v = _lib.coded_view(v[:, rows], vs[:, rows], fmt)
    B, _, H, D = k.shape
    with torch.cuda.device(k.device):
        _lib.check(lib.hyb_decode_rows(B, n, H, D, src_k, src_v, staged[0].data_ptr(), staged[1].data_ptr(),
                                       staged[2], start, _lib.stream_ptr(k.device)), "KV decode into the mirror")


def _validate(cache: dict, key: str) -> None:
    if key not in KV_KEYS:
        raise ValueError(f"Invalid KV key: {key}")
    q = cache[key]
    scale = cache[f"{key}_scale"]
    if q.dtype not in (torch.int8, torch.float8_e4m3fn) or scale.dtype != torch.float32:
        raise TypeError("INT8 or E4M3 KV data and FP32 scale are required")
    if scale.shape != (*q.shape[:-1], 1) or scale.device != q.device:
        raise ValueError("INT8 KV scale shape/device mismatch")


def _check_values(cache: dict, key: str, values: torch.Tensor, start: int) -> None:
    q = cache[key]
    if values.ndim != 4 or values.dtype != torch.bfloat16:
        raise TypeError("KV quantization expects [B,L,H,D] BF16 values")
    batch, length, heads, dim = values.shape
    if (batch != q.shape[0] or heads != q.shape[2] or dim != q.shape[3]
            or start < 0 or start + length > q.shape[1]
            or values.device != q.device):
        raise ValueError("KV quantization shape, capacity, or device mismatch")


def _any_nonfinite(*tensors: torch.Tensor) -> bool:
    """Device-side finite check of bf16 [B, L, H, D] tensors, one host sync."""
    lib = _lib.load()
    dev = tensors[0].device
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = _lib.stream_ptr(dev)
    for t in tensors:
        if t.numel() == 0:
            continue
        view = _lib.bf16_view(t)
        _lib.check(lib.hyb_check_finite(view, t.shape[0], t.shape[1], t.shape[2], t.shape[3],
                                        status.data_ptr(), stream), "finite check")
    return bool(status.item() & _lib.HYB_DEV_NONFINITE)


def _append_pair(cache: dict, k: torch.Tensor, v: torch.Tensor, start: int,
                 k2: torch.Tensor | None = None, v2: torch.Tensor | None = None) -> None:
    """Quantise-on-write of k/v (then k2/v2, appended right after) at token ``start``."""
    lib = _lib.load()
    fmt = _fmt_code(cache)
    codes_k, codes_v = cache["k"], cache["v"]
    sk, sv = cache["k_scale"], cache["v_scale"]
    if codes_k.stride() != codes_v.stride() or sk.stride() != sv.stride():
        raise ValueError("K and V cache tensors must share strides")
    if codes_k.stride(3) != 1:
        raise ValueError("KV cache head_dim must be contiguous")
    B, L, H, D = k.shape
    L2 = 0 if k2 is None else k2.shape[1]
    dev = k.device
    with torch.cuda.device(dev):
        _lib.check(lib.hyb_kv_append_pair(
            fmt, B, L, H, D, codes_k.shape[1], start,
            _lib.bf16_view(k), _lib.bf16_view(v), L2,
            _lib.bf16_view(k2) if L2 else None, _lib.bf16_view(v2) if L2 else None,
            codes_k.data_ptr(), codes_v.data_ptr(), *codes_k.stride()[:3],
            sk.data_ptr(), sv.data_ptr(), *sk.stride()[:3],
            _lib.device_status(dev).data_ptr(), _lib.stream_ptr(dev)), "KV quantization")


def quantize_kv_into(cache: dict, key: str, values: torch.Tensor, start: int, *,
                     assume_finite: bool = False) -> None:
    """Append BF16 values into INT8 / E4M3 storage at token offset ``start``."""
    _validate(cache, key)
    _check_values(cache, key, values, start)
    if values.shape[1] == 0:
        return
    _lib.require_device(values)
    if not assume_finite and _any_nonfinite(values):
        raise ValueError("Cannot quantize non-finite KV values")
    # The pair kernel writes K and V in one launch; a single key writes the same row twice.
    other = {"k": cache[key], "v": cache[key], "k_scale": cache[f"{key}_scale"],
             "v_scale": cache[f"{key}_scale"]}
    _append_pair(other, values, values, start)
    refresh_decoded(cache, start, values.shape[1])


def quantize_kv_pair_into(cache: dict, k: torch.Tensor, v: torch.Tensor, start: int, *,
                          assume_finite: bool = False, decode: bool = True) -> None:
    """Validate K and V before writing either persistent payload or scale; with a decoded
    mirror (and ``decode``) the written rows are decoded into it too."""
    if k.shape != v.shape or k.dtype != v.dtype or k.device != v.device:
        raise ValueError("K/V shapes, dtypes, and devices must match")
    for key, values in (("k", k), ("v", v)):
        _validate(cache, key)
        q = cache[key]
        if (values.ndim != 4 or values.dtype != torch.bfloat16
                or values.shape[0] != q.shape[0]
                or values.shape[2:] != q.shape[2:]
                or start < 0 or start + values.shape[1] > q.shape[1]
                or values.device != q.device):
            raise ValueError("KV pair shape, capacity, dtype, or device mismatch")
    if k.shape[1] == 0:
        return
    _lib.require_device(k)
    if not assume_finite and _any_nonfinite(k, v):
        raise ValueError("Cannot quantize non-finite KV values")
    _append_pair(cache, k, v, start)
    if decode:
        refresh_decoded(cache, start, k.shape[1])


def quantize_kv_segments_into(cache: dict, segments_k, segments_v, start: int, *,
                              assume_finite: bool = False, decode: bool = True) -> None:
    """Append [seg_0 | seg_1] (e.g. image then text tokens) at ``start`` in one pass, with
    the validation of quantize_kv_pair_into; no concatenated copy is made.  ``decode``: as in
    quantize_kv_pair_into (a caller that stages keys into the mirror's rows first decodes later)."""
    segments_k = [s for s in segments_k if s.shape[1] > 0]
    segments_v = [s for s in segments_v if s.shape[1] > 0]
    if not segments_k:
        return
    if len(segments_k) > 2 or len(segments_k) != len(segments_v):
        raise ValueError("at most two K/V segments of matching shapes")
    total = sum(s.shape[1] for s in segments_k)
    for sk_, sv_ in zip(segments_k, segments_v):
        if sk_.shape != sv_.shape or sk_.dtype != sv_.dtype or sk_.device != sv_.device:
            raise ValueError("K/V shapes, dtypes, and devices must match")
    for key in ("k", "v"):
        _validate(cache, key)
        q = cache[key]
        for values in (segments_k if key == "k" else segments_v):
            if (values.ndim != 4 or values.dtype != torch.bfloat16
                    or values.shape[0] != q.shape[0] or values.shape[2:] != q.shape[2:]
                    or start < 0 or start + total > q.shape[1] or values.device != q.device):
                raise ValueError("KV pair shape, capacity, dtype, or device mismatch")
    _lib.require_device(segments_k[0])
    if not assume_finite and _any_nonfinite(*segments_k, *segments_v):
        raise ValueError("Cannot quantize non-finite KV values")
    if len(segments_k) == 1:
        _append_pair(cache, segments_k[0], segments_v[0], start)
    else:
        _append_pair(cache, segments_k[0], segments_v[0], start, segments_k[1], segments_v[1])
    if decode:
        refresh_decoded(cache, start, total)


def dequantize_kv(cache: dict, key: str, valid_len: int) -> torch.Tensor:
    """Decode only the valid prefix into a BF16 tensor [B, valid, H, D]."""
    _validate(cache, key)
    q = cache[key]
    scale = cache[f"{key}_scale"]
    if valid_len < 0 or valid_len > q.shape[1]:
        raise ValueError("Invalid KV valid length")
    batch, _, heads, dim = q.shape
    result = torch.empty((batch, valid_len, heads, dim), device=q.device, dtype=torch.bfloat16)
    if valid_len == 0:
        return result
    _lib.require_device(q)
    lib = _lib.load()
    with torch.cuda.device(q.device):
        _lib.check(lib.hyb_kv_dequant(_lib.coded_view(q, scale, _fmt_code(cache)), batch, valid_len,
                                      heads, dim, result.data_ptr(), _lib.stream_ptr(q.device)),
                   "KV decode")
    return result


def kv_storage_bytes(cache: dict) -> int:
    keys = STORAGE_KEYS if cache_format(cache) in ("int8", FP8_FORMAT) else KV_KEYS
    return sum(cache[key].numel() * cache[key].element_size() for key in keys)
