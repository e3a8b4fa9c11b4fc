"""KV-stationary sequence parallelism on one GPU: every rank of the schedule runs in this process
(``kv_stationary_emulated``), each with its own sequence-sharded window cache, the attention
epilogue scattering fp32 partial rows into the owners' buffers and every owner merging them.
Each step of a rollout (1-frame chunks, sink + sliding window, quantise-on-write of every rank's
slice after the attention) must equal the oracle over the reference's slid history of whole
frames, within the north-star gate."""
import pytest
import torch

from hy_nomas_b200.kv_stationary import kv_stationary_emulated
from hy_nomas_b200.synthetic import make_generator, seeded_kv
from hy_nomas_b200.window import SinkWindowKVCache
from oracle import attention as oatt
from oracle import quant as oq
from oracle import window as ow
from parity import check_bf16

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("P,T,sink,keep,Lt,fmt,slices,decoded", [
    (4, 256, 1, 3, 1, "fp8_e4m3", None, False),   # 64 rows per owner
    (3, 300, 2, 2, 2, "int8", 2, False),          # 100 rows per owner: warps straddle owners
    (2, 512, 1, 4, 1, "fp8_e4m3", 3, False),
    (4, 256, 1, 3, 1, "fp8_e4m3", None, True),    # windows keeping their history decoded
    (3, 300, 2, 2, 2, "int8", 2, True),
])
def test_kv_stationary_rollout_matches_oracle(cuda_lib, P, T, sink, keep, Lt, fmt, slices, decoded):
    dev = torch.device("cuda")
    H = 2
    Ls = T // P
    gen = make_generator(4100 + P * 7 + keep)
    wins = [SinkWindowKVCache(1, H, Ls, sink, keep, storage_format=fmt, device=dev, decoded=decoded) for _ in range(P)]
    all_k, all_v = [], []
    for step in range(sink + keep + 3):
        q, k, v = (seeded_kv((1, T, H, 128), gen) for _ in range(3))
        tq, tk, tv = (seeded_kv((1, Lt, H, 128), gen) for _ in range(3))
        tmask = torch.ones(1, Lt, dtype=torch.bool)
        if Lt > 1:
            tmask[0, -1] = False
        with torch.no_grad():
            out_img, out_txt = kv_stationary_emulated(
                q.to(dev), k.to(dev), v.to(dev), tq.to(dev), tk.to(dev), tv.to(dev), wins,
                text_mask=tmask.to(dev), slices=slices)
        frames = len(all_k)
        if frames:
            hk, _ = ow.slide(torch.cat(all_k, 1), frames, sink, keep, T)
            hv, kept = ow.slide(torch.cat(all_v, 1), frames, sink, keep, T)
            hk, hv = hk[:, :kept * T], hv[:, :kept * T]
        else:
            hk = hv = k[:, :0]
        ref_img, ref_txt, _, _ = oatt.cached_attention(q, k, v, tq, tk, tv, hk, hv, attend_txt=True,
                                                       text_mask=tmask, return_lse=True, return_magnitude=True)
        check_bf16(out_img, ref_img, f"KV-stationary P={P} step {step} image rows")
        check_bf16(out_txt, ref_txt, f"KV-stationary P={P} step {step} text rows")
        if Lt > 1:
            assert out_txt[0, -1].float().abs().max().item() == 0.0   # padded text query
        ck, sk = oq.quantize(k, fmt)
        cv, sv = oq.quantize(v, fmt)
        all_k.append(oq.dequantize(ck, sk))
        all_v.append(oq.dequantize(cv, sv))
    assert all(w.frames == sink + keep + 3 for w in wins)

