"""The north-star parity gate, shown plainly: max-abs-err and cosine against the fp32 oracle.

(1) fp32 rows before the output rounding: every query pair is cut into two key slices
    (HYB_KV_SPLITS=2), each slice writes its normalised fp32 rows and natural-log LSE into the
    workspace (the kernel's split epilogue), and the test combines the two in float64 -- the
    combination the kernel's merge pass makes in fp32 before its single bf16 rounding.  These
    rows must meet the flat gate: max-abs <= 2e-2, cosine >= 0.9995, on BASELINE config 1 and
    on config-2 geometry (2 of the 24 heads).
(2) the bf16 outputs of the same calls: max-abs <= 2e-2 + the bf16 rounding floor of the exact
    rows (the error the reference's own bf16 output carries, tests/test_parity_floor.py),
    cosine >= 0.9995.
The measured numbers are printed (pytest -s shows them)."""
import pytest
import torch

from conftest import config1_inputs
from hy_nomas_b200 import _lib
from hy_nomas_b200 import attention as hatt
from hy_nomas_b200 import kv_cache as kvc
from oracle import attention as oatt
from oracle import quant as oq
from parity import check_bf16, check_fp32

pytestmark = pytest.mark.gpu


def kernel_rows(cur, cache, Lh, G, monkeypatch):
    """(fp32 rows before rounding [B, Lq, H, D], bf16 image rows, bf16 text rows) of one call."""
    monkeypatch.setenv("HYB_KV_SPLITS", "2")
    dev = cur[0].device
    ws = hatt.Workspace()
    out_img, out_txt = hatt.cached_attention_local(*cur, cache, Lh, group_tokens=G, workspace=ws)
    torch.cuda.synchronize()
    _lib.check_device_status(dev)
    B, Li, H, D = cur[0].shape
    Lt = cur[3].shape[1]
    lay = hatt.workspace_layout(B, H, Lh, Li, Lt, True, D)
    S, Lq = lay.kv_splits, lay.Lq
    assert S == 2
    buf = ws.buf
    po = buf[lay.part_o:lay.part_o + S * B * H * Lq * D * 4].view(torch.float32).view(S, B, H, Lq, D).double()
    pl = buf[lay.part_lse:lay.part_lse + S * B * H * Lq * 4].view(torch.float32).view(S, B, H, Lq).double()
    m = pl.max(0).values
    w = torch.where(torch.isfinite(pl), torch.exp(pl - m), torch.zeros_like(pl))
    rows = (w[..., None] * po).sum(0) / w.sum(0)[..., None]
    return rows.permute(0, 2, 1, 3).float().cpu(), out_img.float().cpu(), out_txt.float().cpu()


def fp8_cache(hk, hv, cap, dev):
    H = hk.shape[2]
    cache = kvc.make_fp8_kv_block(1, cap, H, 128, device=dev)
    with torch.no_grad():
        kvc.quantize_kv_pair_into(cache, hk.to(dev), hv.to(dev), 0)
    return cache


def test_config1_fp32_rows_and_bf16_outputs_meet_the_gate(cuda_lib, monkeypatch):
    """8 heads, one 256-token frame against 4 cached E4M3 frames + 1 text token."""
    dev = torch.device("cuda")
    hk, hv, cur, _ = config1_inputs()
    Lh, Li = hk.shape[1], cur[0].shape[1]
    cache = fp8_cache(hk, hv, Lh + Li + 1, dev)
    rows, out_img, out_txt = kernel_rows([t.to(dev) for t in cur], cache, Lh, 256, monkeypatch)
    ck, sk = oq.quantize_e4m3(hk)
    cv, sv = oq.quantize_e4m3(hv)
    assert torch.equal(cache["k"][:, :Lh].cpu().view(torch.uint8), ck.view(torch.uint8))
    ref_img, ref_txt = oatt.cached_attention(*cur, oq.dequantize(ck, sk), oq.dequantize(cv, sv), group_tokens=256)
    exact = torch.cat([ref_img, ref_txt], 1)
    check_fp32(rows, exact, "config 1 fp32 rows")
    check_bf16(torch.cat([out_img, out_txt], 1), exact, "config 1 bf16 output")


def test_config2_geometry_fp32_rows_and_bf16_outputs_meet_the_gate(cuda_lib, monkeypatch):
    """Config-2 geometry (24,960-token E4M3 history, 4-frame chunk of 1,560-token frames,
    frame-causal, 1 text token) on 2 of the 24 heads; exact reference in fp32 on the GPU."""
    from hy_nomas_b200.synthetic import make_generator, seeded_kv
    dev = torch.device("cuda")
    H, T = 2, 1560
    Lh, Li, Lt = 16 * T, 4 * T, 1
    gen = make_generator(4242)
    hk, hv = seeded_kv((1, Lh, H, 128), gen), seeded_kv((1, Lh, H, 128), gen)
    cur = [seeded_kv((1, L, H, 128), gen) for L in (Li, Lt) for _ in range(3)]
    cache = fp8_cache(hk, hv, Lh + Li + Lt, dev)
    rows, out_img, out_txt = kernel_rows([t.to(dev) for t in cur], cache, Lh, T, monkeypatch)
    dk = oq.dequantize(*oq.quantize_e4m3(hk)).to(dev).float()
    dv = oq.dequantize(*oq.quantize_e4m3(hv)).to(dev).float()
    q = torch.cat([cur[0], cur[3]], 1).to(dev).float()
    k = torch.cat([dk, cur[1].to(dev).float(), cur[4].to(dev).float()], 1)
    v = torch.cat([dv, cur[2].to(dev).float(), cur[5].to(dev).float()], 1)
    Lq, Lk = q.shape[1], k.shape[1]
    qpos, kpos = torch.arange(Lq, device=dev), torch.arange(Lk, device=dev)
    qblk = torch.where(qpos < Li, qpos // T, torch.full_like(qpos, 10 ** 9))
    kblk = torch.where((kpos >= Lh) & (kpos < Lh + Li), (kpos - Lh) // T, torch.full_like(kpos, -1))
    mask = kblk[None, :] <= qblk[:, None]
    exact = torch.empty(Lq, H, 128, device=dev)
    for h in range(H):
        s = (q[0, :, h].double() @ k[0, :, h].double().T) / (128 ** 0.5)
        s.masked_fill_(~mask, float("-inf"))
        exact[:, h] = (torch.softmax(s, -1) @ v[0, :, h].double()).float()
    exact = exact.cpu()[None]
    check_fp32(rows, exact, "config-2 geometry fp32 rows")
    check_bf16(torch.cat([out_img, out_txt], 1), exact, "config-2 geometry bf16 output")
