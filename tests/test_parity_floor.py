"""The reference's own bf16 outputs measured against the fp32 oracle on the same inputs.

Every golden fixture holds outputs of the reference's ``causal_attention_with_cache_mp``
(torch mode, tests/golden/make_golden.py).  Their distance from the exact fp32 attention is
the floor of any implementation that returns bf16, the reference's included: it is exactly
the bf16 rounding of the exact result (the reference computes the CPU path in fp32 and
rounds once).  The recorded floors pin that, and the GPU tests and the smoke check gate their
bf16 outputs at 2e-2 on top of the floor of their own inputs (tests/parity.py)."""
import pytest
import torch

from conftest import bf16, config1_inputs, e4m3, load_golden
from oracle import attention as oatt
from oracle import quant as oq
from parity import COS, metrics, rounding_floor

# max |reference bf16 output - fp32 oracle| per fixture (image and valid text rows together)
RECORDED_FLOOR = {
    "config1": 0.028821945,
    "int8_basic": 0.039699554,
    "int8_update": 0.029899597,
    "int8_nocachetxt": 0.029703140,
    "int8_update_nocachetxt": 0.053251266,
    "int8_cfg": 0.059839249,
    "int8_empty_history": 0.054517746,
    "fp8_o2": 0.030920029,
    "frame_causal_o3": 0.033270836,
}


def _case(name):
    """(exact fp32 rows, reference bf16 rows) of one fixture, valid rows only."""
    if name == "config1":
        g = load_golden("attn_config1.npz")
        hk, hv, cur, _ = config1_inputs()
        dk = oq.dequantize(*oq.quantize_e4m3(hk))
        dv = oq.dequantize(*oq.quantize_e4m3(hv))
        img, txt = oatt.cached_attention(*cur, dk, dv, group_tokens=256)
        return torch.cat([img.flatten(), txt.flatten()]), torch.cat(
            [bf16(g["out_img"]).float().flatten(), bf16(g["out_txt"]).float().flatten()])
    g = load_golden(f"attn_{name}.npz")
    Lh = int(g["Lh"])
    if name == "fp8_o2":
        hk = oq.dequantize(e4m3(g["hist_k"]), torch.from_numpy(g["hist_k_scale"]))
        hv = oq.dequantize(e4m3(g["hist_v"]), torch.from_numpy(g["hist_v_scale"]))
    else:
        hk = oq.dequantize(torch.from_numpy(g["hist_k"][:, :Lh]), torch.from_numpy(g["hist_k_scale"][:, :Lh]))
        hv = oq.dequantize(torch.from_numpy(g["hist_v"][:, :Lh]), torch.from_numpy(g["hist_v_scale"][:, :Lh]))
    cur = [bf16(g[n]) for n in ("img_q", "img_k", "img_v", "txt_q", "txt_k", "txt_v")]
    kw = {}
    valid = torch.ones(cur[3].shape[:2], dtype=torch.bool)
    if name == "frame_causal_o3":
        kw["group_tokens"] = int(g["tokens_per_frame"])
    elif name.startswith("int8"):
        valid = torch.from_numpy(g["text_mask"]).bool()
        kw.update(history_mask=torch.from_numpy(g["cache_mask"]), text_mask=valid,
                  attend_txt=bool(g["cache_txt"]) or bool(g["update_cache"]))
    img, txt = oatt.cached_attention(*cur, hk, hv, **kw)
    ref_img, ref_txt = bf16(g["out_img"]).float(), bf16(g["out_txt"]).float()
    return torch.cat([img.flatten(), txt[valid].flatten()]), torch.cat([ref_img.flatten(), ref_txt[valid].flatten()])


CASES = ["config1", "int8_basic", "int8_update", "int8_nocachetxt", "int8_update_nocachetxt", "int8_cfg",
         "int8_empty_history", "fp8_o2", "frame_causal_o3"]


@pytest.mark.parametrize("name", CASES)
def test_reference_bf16_output_is_the_rounded_exact_result(name):
    exact, ref = _case(name)
    mae, cos = metrics(ref, exact)
    floor = rounding_floor(exact)
    print(f"{name}: reference bf16 vs fp32 oracle max_abs={mae:.4e} cos={cos:.7f}; "
          f"bf16 rounding floor of the exact rows {floor:.4e}")
    assert cos >= COS
    # the reference's error is its output rounding (plus fp32 summation-order noise)
    assert mae <= floor + 2.0 ** -9 * exact.abs().max().item()
    if name in RECORDED_FLOOR:
        assert abs(mae - RECORDED_FLOOR[name]) < 1e-6, mae


def test_config1_reference_floor_exceeds_a_flat_2e_2():
    """On the benchmark distribution the flat 2e-2 gate is below the reference's own rounding."""
    exact, ref = _case("config1")
    assert metrics(ref, exact)[0] > 2e-2
