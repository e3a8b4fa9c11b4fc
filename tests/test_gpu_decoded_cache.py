"""A quantised cache that keeps a decoded mirror (kv_cache.attach_decoded_mirror / decoded=True):
every write decodes the rows it wrote, and the drop-in reads the history from the mirror
instead of decoding the whole cache per call.  The keys, their order and their values are the
ones the per-call decode stages, so a sequence of calls (denoising steps that only read the
cache, then a step that writes the chunk) gives the same outputs and LSE bit for bit, the same
cache codes, and a mirror equal to the decode of the codes."""
import pytest
import torch

from hy_nomas_b200 import attention as hatt
from hy_nomas_b200 import kv_cache as kvc
from hy_nomas_b200.synthetic import make_generator, seeded_kv

pytestmark = pytest.mark.gpu


def _run(decoded, fmt, seed):
    dev = torch.device("cuda")
    B, H, T, frames, Lt = 1, 2, 160, 2, 3
    hist_frames = 3
    Lh, Li = hist_frames * T, frames * T
    cap = Lh + 2 * (Li + Lt)
    make = kvc.make_fp8_kv_block if fmt == "fp8_e4m3" else kvc.make_int8_kv_block
    cache = make(B, cap, H, 128, device=dev, decoded=decoded)
    gen = make_generator(seed)
    with torch.no_grad():
        kvc.quantize_kv_pair_into(cache, seeded_kv((B, Lh, H, 128), gen).to(dev),
                                  seeded_kv((B, Lh, H, 128), gen).to(dev), 0)
    cmask = torch.zeros(B, cap, dtype=torch.bool, device=dev)
    cmask[:, :Lh] = True
    cmask[:, 7:11] = False
    outs = []
    valid = Lh
    for chunk in range(2):
        cur = [seeded_kv((B, L, H, 128), gen).to(dev) for L in (Li, Lt) for _ in range(3)]
        tmask = torch.tensor([[True, True, False]], device=dev)
        for step in range(3):   # two reading steps, then the step that writes the chunk
            write = step == 2
            with torch.no_grad():
                o_img, o_txt = hatt.causal_attention_with_cache_mp(
                    (cur[0], cur[3]), (cur[1], cur[4]), (cur[2], cur[5]), cache, cache_valid_len=valid,
                    text_mask=tmask, update_cache=write, cache_txt=True, cache_mask=cmask, tokens_per_frame=T,
                    seg_ar_attention_backend="b200", chunk_causal_frames=1)
            outs += [o_img.clone(), o_txt.clone()]
        valid += Li + Lt
    torch.cuda.synchronize()
    return outs, cache, valid


@pytest.mark.parametrize("fmt", ["fp8_e4m3", "int8"])
def test_decoded_mirror_matches_per_call_decode(cuda_lib, fmt):
    plain, c0, valid = _run(False, fmt, 9100)
    mirrored, c1, _ = _run(True, fmt, 9100)
    for i, (a, b) in enumerate(zip(plain, mirrored)):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16)), f"output {i} differs"
    for name in ("k", "v"):
        assert torch.equal(c0[name].view(torch.uint8), c1[name].view(torch.uint8))
        assert torch.equal(c0[f"{name}_scale"], c1[f"{name}_scale"])
    mk, mv, pitch = c1["staged"]
    want_k = kvc.dequantize_kv(c1, "k", valid)           # bf16 [B, valid, H, D]
    want_v = kvc.dequantize_kv(c1, "v", valid)
    assert torch.equal(mk[:, :, :valid].transpose(1, 2).contiguous().view(torch.int16), want_k.view(torch.int16))
    assert torch.equal(mv[:, :, :valid].transpose(1, 2).contiguous().view(torch.int16),
                       want_v.to(torch.float16).view(torch.int16))   # fp16 of the bf16 decode


def test_decoded_mirror_needs_room_for_the_call(cuda_lib):
    dev = torch.device("cuda")
    H, T = 2, 128
    cache = kvc.make_fp8_kv_block(1, 2 * T, H, 128, device=dev, decoded=True)
    gen = make_generator(3)
    q, k, v = (seeded_kv((1, T, H, 128), gen).to(dev) for _ in range(3))
    empty = q[:, :0]
    with torch.no_grad():
        kvc.quantize_kv_pair_into(cache, k, v, 0)
        with pytest.raises(ValueError, match="mirror"):
            hatt.cached_attention_local(q, k, v, empty, empty, empty, cache, 2 * T)
