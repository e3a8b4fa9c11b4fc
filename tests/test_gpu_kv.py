"""Quantise-on-write and decode kernels on the GPU, bit-exact against the oracle
(and, for INT8, against the reference's own codes in tests/golden/quant_int8.npz)."""
import numpy as np
import pytest
import torch

from conftest import bf16, load_golden
from hy_nomas_b200 import kv_cache as kvc
from hy_nomas_b200.synthetic import make_generator, seeded_kv
from oracle import quant as oq

pytestmark = pytest.mark.gpu


def _block(fmt, B, cap, H, dev):
    if fmt == "int8":
        return kvc.make_int8_kv_block(B, cap, H, 128, device=dev)
    return kvc.make_fp8_kv_block(B, cap, H, 128, device=dev)


def _codes_np(t):
    return (t.view(torch.uint8) if t.dtype == torch.float8_e4m3fn else t).cpu().numpy()


def test_int8_append_matches_reference_codes(cuda_lib):
    g = load_golden("quant_int8.npz")
    dev = torch.device("cuda")
    k, v = bf16(g["k"]).to(dev), bf16(g["v"]).to(dev)
    start = int(g["start"])
    cache = _block("int8", 1, 48, 3, dev)
    kvc.quantize_kv_pair_into(cache, k, v, start)
    torch.cuda.synchronize()
    for key in ("k", "v"):
        assert np.array_equal(cache[key][:, start:start + 40].cpu().numpy(), g[f"{key}_codes"])
        got = cache[f"{key}_scale"][:, start:start + 40].cpu().numpy()
        assert np.array_equal(got.view(np.int32), g[f"{key}_scale"].view(np.int32))
        deq = kvc.dequantize_kv(cache, key, start + 40)[:, start:]
        assert np.array_equal(deq.cpu().view(torch.int16).numpy(), g[f"{key}_deq"])


@pytest.mark.parametrize("fmt", ["int8", "fp8_e4m3"])
@pytest.mark.parametrize("B,L,H,start", [(1, 1, 1, 0), (2, 333, 5, 17), (1, 6241, 24, 24960)])
def test_append_bit_exact_vs_oracle(cuda_lib, fmt, B, L, H, start):
    dev = torch.device("cuda")
    gen = make_generator(1000 + L)
    # strided source: K and V are slices of one concatenated [B, L, 2H, D] tensor
    kv = seeded_kv((B, L, 2 * H, 128), gen)
    kv[:, 0, 0] = 0
    if L > 3:
        kv[:, 2, 1] *= 1e-25
        kv[:, 3, 0] *= 1e4
    kv_dev = kv.to(dev)
    k, v = kv_dev[:, :, :H], kv_dev[:, :, H:]
    cap = start + L + 5
    cache = _block(fmt, B, cap, H, dev)
    kvc.quantize_kv_pair_into(cache, k, v, start)
    torch.cuda.synchronize()
    for key, src in (("k", kv[:, :, :H]), ("v", kv[:, :, H:])):
        codes, scale = oq.quantize(src, fmt)
        got_codes = _codes_np(cache[key][:, start:start + L])
        assert np.array_equal(got_codes, _codes_np(codes))
        got_scale = cache[f"{key}_scale"][:, start:start + L].cpu().numpy()
        assert np.array_equal(got_scale.view(np.int32), scale.numpy().view(np.int32))
        deq = kvc.dequantize_kv(cache, key, start + L)[:, start:].cpu()
        assert torch.equal(deq.view(torch.int16), oq.dequantize(codes, scale).view(torch.int16))


@pytest.mark.parametrize("fmt", ["int8", "fp8_e4m3"])
def test_nonfinite_values_rejected_before_any_write(cuda_lib, fmt):
    dev = torch.device("cuda")
    gen = make_generator(5)
    k = seeded_kv((1, 8, 2, 128), gen).to(dev)
    v = seeded_kv((1, 8, 2, 128), gen).to(dev)
    v[0, 5, 1, 7] = float("nan")
    cache = _block(fmt, 1, 16, 2, dev)
    for t in cache.values():
        if isinstance(t, torch.Tensor):
            t.view(torch.uint8).fill_(0xAB) if t.dtype != torch.float32 else t.fill_(-3.0)
    snapshot = {k2: t.clone() for k2, t in cache.items() if isinstance(t, torch.Tensor)}
    with pytest.raises(ValueError, match="non-finite"):
        kvc.quantize_kv_pair_into(cache, k, v, 4)
    for key, t in snapshot.items():
        assert torch.equal(cache[key].view(torch.uint8), t.view(torch.uint8))


def test_capacity_and_shape_errors(cuda_lib):
    dev = torch.device("cuda")
    cache = _block("fp8_e4m3", 1, 16, 2, dev)
    k = torch.zeros(1, 8, 2, 128, dtype=torch.bfloat16, device=dev)
    with pytest.raises(ValueError):
        kvc.quantize_kv_pair_into(cache, k, k, 12)
    with pytest.raises(ValueError):
        kvc.quantize_kv_pair_into(cache, k, k[:, :4], 0)
    with pytest.raises(ValueError):
        kvc.dequantize_kv(cache, "k", 17)


@pytest.mark.parametrize("fmt", ["int8", "fp8_e4m3"])
def test_append_bit_exact_on_adversarial_rows(cuda_lib, fmt):
    """Rows whose quotients x / s sit on rounding ties of the code format, rows spanning 2^-133
    .. 2^20 in magnitude, negative zeros, and rows whose absmax is a bf16 subnormal."""
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(4242)
    L, H = 512, 4
    x = torch.randn(1, L, H, 128, generator=g)
    mags = torch.pow(2.0, torch.randint(-60, 21, (1, L, H, 1), generator=g).float())
    x = x * mags
    x[:, :32] *= torch.pow(2.0, torch.randint(-133, -100, (1, 32, H, 128), generator=g).float())  # tiny, mixed
    x[:, 32:40] = 2.0 ** -130 * torch.randint(-3, 4, (1, 8, H, 128), generator=g).float()        # subnormal absmax
    x[:, 40:48] = -0.0
    x[:, 48:56, :, 5] = 1.0
    # ties: absmax 448 (s = 1) or 127 (s = 1), values halfway between neighbouring codes
    top = 448.0 if fmt == "fp8_e4m3" else 127.0
    ties = torch.tensor([1.0625, -1.0625, 2.125, 0.5 + 2 ** -5, 3.5 * 2 ** -8, -0.5, 1.5, -2.5, 100.5, 13.0])
    x[:, 56:64] = ties.repeat(13)[:128].view(1, 1, 1, 128)
    x[:, 56:64, :, 0] = top
    x[:, 64:72] = x[:, 56:64] * 2.0 ** -40   # the same ties at a power-of-two scale
    x = x.to(torch.bfloat16)
    k, v = x.to(dev), (-x).to(dev)
    cache = _block(fmt, 1, L, H, dev)
    kvc.quantize_kv_pair_into(cache, k, v, 0)
    torch.cuda.synchronize()
    for key, src in (("k", x), ("v", -x)):
        codes, scale = oq.quantize(src, fmt)
        assert np.array_equal(_codes_np(cache[key]), _codes_np(codes)), key
        assert np.array_equal(cache[f"{key}_scale"].cpu().numpy().view(np.int32), scale.numpy().view(np.int32))
