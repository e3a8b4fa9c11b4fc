"""The installer on the reference's own DiT module (CPU, where a reference checkout is named by
HY_NOMAS_REF; skipped elsewhere).  ``hymm.models.dit.nomas_cpt`` imports with a 10-line
``diffusers`` stub (``oracle/reference.py``).  An unmodified
``MMDoubleStreamBlock.forward_with_cache`` call (nomas_cpt.py:1292-1416) must reach the patched
module attribute: CPU tensors fall back to the native function with an identical result, and
an eligible call is handed to the B200 drop-in with the block's own arguments."""
import importlib
import os
from pathlib import Path

import pytest
import torch

from hy_nomas_b200 import attention as hatt
from hy_nomas_b200 import install as hinst


pytestmark = pytest.mark.skipif(
    not (os.environ.get("HY_NOMAS_REF") and (Path(os.environ["HY_NOMAS_REF"]) / "hymm").is_dir()),
    reason="HY_NOMAS_REF does not name a reference checkout")


@pytest.fixture(scope="module")
def native():
    from oracle.reference import install_stub
    install_stub()
    return importlib.import_module("hymm.models.dit.nomas_cpt")


def _block_call(native, block, cache, attn_mode="flash3"):
    gen = torch.Generator().manual_seed(11)
    B, Li, Lt, C = 1, 16, 3, 256
    img = torch.randn(B, Li, C, generator=gen).to(torch.bfloat16)
    txt = torch.randn(B, Lt, C, generator=gen).to(torch.bfloat16)
    vec = torch.randn(B, C, generator=gen).to(torch.bfloat16)
    with torch.no_grad():
        return block.forward_with_cache(img, txt, vec, kv_cache=cache, cache_valid_len=8, update_cache=False,
                                        attn_mode=attn_mode, cache_txt=True,
                                        cache_mask=torch.ones(B, 40, dtype=torch.bool))


def _cache():
    gen = torch.Generator().manual_seed(12)
    k = torch.randn(1, 40, 2, 128, generator=gen).to(torch.bfloat16)
    v = torch.randn(1, 40, 2, 128, generator=gen).to(torch.bfloat16)
    return {"k": k, "v": v}


def test_block_calls_reach_the_patch_and_cpu_falls_back_identically(native):
    torch.manual_seed(0)
    block = native.MMDoubleStreamBlock(hidden_size=256, heads_num=2, mlp_width_ratio=2.0,
                                       dtype=torch.bfloat16).eval()
    ref = _block_call(native, block, _cache(), attn_mode="torch")
    original = hinst.install(native)
    try:
        patched = native.causal_attention_with_cache_mp
        assert patched is not original and patched.original is original
        got = _block_call(native, block, _cache(), attn_mode="torch")
        assert patched.stats == {"calls": 0, "fallbacks": 1}
        for a, b in zip(ref, got):
            assert torch.equal(a, b)
    finally:
        hinst.uninstall(native)
        hatt.set_parallel_state_provider(hatt._ps.get_sequence_parallel_state, hatt._ps.nccl_info)
    assert native.causal_attention_with_cache_mp is original


def test_eligible_block_calls_are_handed_to_the_b200_drop_in(native, monkeypatch):
    torch.manual_seed(0)
    block = native.MMDoubleStreamBlock(hidden_size=256, heads_num=2, mlp_width_ratio=2.0,
                                       dtype=torch.bfloat16).eval()
    seen = []

    def drop_in(q, k, v, kv_cache, cache_valid_len, attn_mode, text_mask, update_cache, cache_txt, cache_mask,
                intra_seg_txt_offsets, intra_seg_vid_windows, tokens_per_frame, backend, sparse_context,
                sp_metadata, attention_metadata, **extra):
        seen.append(dict(cache_valid_len=cache_valid_len, attn_mode=attn_mode, update_cache=update_cache,
                         cache_txt=cache_txt, backend=backend, shapes=(q[0].shape, q[1].shape)))
        # stand in for the device path on the CPU: the reference computes the same call
        return original(q, k, v, kv_cache, cache_valid_len, "torch", text_mask, update_cache, cache_txt,
                        cache_mask, intra_seg_txt_offsets, intra_seg_vid_windows, tokens_per_frame)

    original = hinst.install(native)
    try:
        monkeypatch.setattr(hinst, "_eligible", lambda *a: True)
        monkeypatch.setattr(hinst._att, "causal_attention_with_cache_mp", drop_in)
        out = _block_call(native, block, _cache())
        patched = native.causal_attention_with_cache_mp
        assert patched.stats == {"calls": 1, "fallbacks": 0}
        assert seen == [dict(cache_valid_len=8, attn_mode="flash3", update_cache=False, cache_txt=True,
                             backend="magi", shapes=(torch.Size([1, 16, 2, 128]), torch.Size([1, 3, 2, 128])))]
        assert out[0].shape == (1, 16, 256) and out[1].shape == (1, 3, 256)
    finally:
        hinst.uninstall(native)
        hatt.set_parallel_state_provider(hatt._ps.get_sequence_parallel_state, hatt._ps.nccl_info)
