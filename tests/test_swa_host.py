"""The bounded (sliding-window) segment-AR history of hy_nomas_b200/swa.py on the CPU, against
the state the reference's own commit left after every call of a sequence
(tests/golden/make_golden.py: make_swa).  The bf16 commit is pure row movement, so it runs
here in full; the quantised commits and the attention are the GPU tests' part."""
import numpy as np
import pytest
import torch

from conftest import bf16, load_golden
from hy_nomas_b200 import swa

FIXTURES = ["swa_int8_evict", "swa_bf16_evict", "swa_int8_overflow"]
T, LT = 16, 3


def _records(cache):
    return [[r.start, r.image_tokens, r.end, r.time_start, r.height, r.width] for r in cache["swa_video"]]


@pytest.mark.parametrize("name", FIXTURES)
def test_records_and_cuts_follow_the_reference(name):
    g = load_golden(f"{name}.npz")
    cache = {"swa_capacity": int(g["capacity"])}
    valid = 0
    for i in range(int(g["steps"])):
        assert valid == int(g[f"{i}_valid_before"])
        n_img = g[f"{i}_img_k"].shape[1]
        swa.append_dense_record(cache, valid, n_img, LT, T)
        cut = swa.eviction_cut(cache["swa_video"], valid + n_img + LT, int(g["capacity"]))
        assert cut == int(g[f"{i}_evicted"])
        cache["swa_video"] = swa.trim_records(cache["swa_video"], cut)
        valid = valid + n_img + LT - cut
        assert valid == int(g[f"{i}_valid_after"])
        assert _records(cache) == g[f"{i}_records"].tolist()
        assert cache["swa_next_frame"] == int(g[f"{i}_next_frame"])


def test_bf16_commit_leaves_the_reference_cache():
    g = load_golden("swa_bf16_evict.npz")
    cap = int(g["cap"])
    H, D = g["0_img_k"].shape[2:]
    cache = {"k": torch.zeros(1, cap, H, D, dtype=torch.bfloat16), "v": torch.zeros(1, cap, H, D, dtype=torch.bfloat16),
             "swa_capacity": int(g["capacity"])}
    mask = torch.zeros(1, cap, dtype=torch.bool)
    valid = 0
    for i in range(int(g["steps"])):
        img_k, img_v = bf16(g[f"{i}_img_k"]), bf16(g[f"{i}_img_v"])
        txt_k, txt_v = bf16(g[f"{i}_txt_k"]), bf16(g[f"{i}_txt_v"])
        tm = torch.from_numpy(g[f"{i}_text_mask"])
        write_mask = torch.cat([torch.ones(1, img_k.shape[1], dtype=torch.bool), tm], dim=1)
        swa.append_dense_record(cache, valid, img_k.shape[1], LT, T)
        swa.commit_window(cache, mask, [img_k, txt_k], [img_v, txt_v], write_mask, valid)
        valid = cache["swa_valid_len"]
        assert valid == int(g[f"{i}_valid_after"]) and cache["swa_evicted"] == int(g[f"{i}_evicted"])
        for key in ("k", "v"):
            assert np.array_equal(cache[key][:, :valid].view(torch.int16).numpy(), g[f"{i}_{key}"])
        assert np.array_equal(mask.numpy(), g[f"{i}_mask"])
        assert mask._action_tail_ranges == []
        assert _records(cache) == g[f"{i}_records"].tolist()


def test_cut_is_frame_aligned_or_a_whole_record():
    recs = [swa.DenseVideo(0, 32, 35, 0, 1, 16), swa.DenseVideo(35, 48, 86, 2, 1, 16)]
    assert swa.eviction_cut(recs, 80, 90) == 0           # within the budget
    assert swa.eviction_cut(recs, 91, 90) == 16          # one frame of the first record
    assert swa.eviction_cut(recs, 110, 90) == 35         # both of its frames: the record with its text
    assert swa.eviction_cut(recs, 125, 90) == 35         # an excess of exactly its end
    assert swa.eviction_cut(recs, 126, 90) == 51         # the next record's first frame
    with pytest.raises(ValueError, match="do not cover"):
        swa.eviction_cut(recs, 200, 90)
    with pytest.raises(ValueError, match="complete video frames"):
        swa.trim_records(recs, 8)


def test_dense_record_checks():
    cache = {}
    with pytest.raises(ValueError, match="complete video frames"):
        swa.check_dense_record(cache, 0, 33, 16)
    with pytest.raises(ValueError, match="complete video frames"):
        swa.check_dense_record(cache, 0, 32, 0)
    with pytest.raises(ValueError, match="does not cover"):
        swa.check_dense_record(cache, 10, 32, 16)
    swa.append_dense_record(cache, 0, 32, 3, 16)
    swa.check_dense_record(cache, 35, 16, 16)
    assert cache["swa_next_frame"] == 2
