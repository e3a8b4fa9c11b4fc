"""Host-side logic without a GPU: the installer's fallback routing, argument validation of
the drop-in, FLOP accounting and the synthetic-input generator."""
import types

import pytest
import torch

from hy_nomas_b200 import attention as hatt
from hy_nomas_b200 import install as hinst
from hy_nomas_b200 import kv_cache as kvc
from hy_nomas_b200.flops import append_bytes, attention_flops


def _fake_native():
    calls = []

    def native(q, k, v, kv_cache, *args):
        calls.append(args)
        return "native"

    mod = types.SimpleNamespace(causal_attention_with_cache_mp=native,
                                get_sequence_parallel_state=lambda: False,
                                nccl_info=types.SimpleNamespace(sp_group=None, rank_within_spgroup=0))
    return mod, calls


def test_install_routes_cpu_and_unsupported_modes_to_native():
    mod, calls = _fake_native()
    original = hinst.install(mod)
    try:
        patched = mod.causal_attention_with_cache_mp
        assert patched.original is original
        x = torch.zeros(1, 2, 2, 128, dtype=torch.bfloat16)
        cache = {"k": torch.zeros(1, 4, 2, 128, dtype=torch.bfloat16), "v": torch.zeros(1, 4, 2, 128, dtype=torch.bfloat16)}
        assert patched((x, x), (x, x), (x, x), cache, 0, "flash3") == "native"      # CPU tensors
        assert patched((x, x), (x, x), (x, x), cache, 0, "flash3", sparse_context={}) == "native"
        qvg = {"storage_format": "qvg", "k": cache["k"], "v": cache["v"]}
        assert patched((x, x), (x, x), (x, x), qvg, 0, "flash3") == "native"
        assert patched.stats["fallbacks"] == 3 and patched.stats["calls"] == 0
        assert len(calls) == 3 and calls[0][:4] == (0, "flash3", None, False)   # positional order kept
    finally:
        hinst.uninstall(mod)
    assert mod.causal_attention_with_cache_mp is original
    hatt.set_parallel_state_provider(hatt._ps.get_sequence_parallel_state, hatt._ps.nccl_info)


def test_drop_in_validates_before_touching_the_device():
    x = torch.zeros(1, 2, 2, 128, dtype=torch.bfloat16)
    cache = {"k": torch.zeros(1, 4, 2, 128, dtype=torch.bfloat16), "v": torch.zeros(1, 4, 2, 128, dtype=torch.bfloat16)}
    with pytest.raises(ValueError, match="seg_ar_attention_backend"):
        hatt.causal_attention_with_cache_mp((x, x), (x, x), (x, x), cache, seg_ar_attention_backend="bogus")
    with pytest.raises(ValueError, match="Unsupported attn_mode for KV cache: sdpa"):
        hatt.causal_attention_with_cache_mp((x, x), (x, x), (x, x), cache, attn_mode="sdpa")
    with pytest.raises(NotImplementedError):
        hatt.causal_attention_with_cache_mp((x, x), (x, x), (x, x), cache, sparse_context={"config": {}})
    i8 = kvc.make_int8_kv_block(1, 4, 2, 128, device="cpu")
    with pytest.raises(ValueError, match="no-grad"):
        with torch.enable_grad():
            hatt.causal_attention_with_cache_mp((x, x), (x, x), (x, x), i8)
    mixed = {"k": cache["k"], "v": cache["v"].float()}
    with pytest.raises(RuntimeError, match="dtype mismatch"):
        hatt.causal_attention_with_cache_mp((x, x), (x, x), (x, x), mixed)
    with pytest.raises(RuntimeError, match="CUDA"):
        with torch.no_grad():
            hatt.causal_attention_with_cache_mp((x, x), (x, x), (x, x), cache)


def test_cache_formats_and_modes():
    assert kvc.cache_format(kvc.make_int8_kv_block(1, 2, 1, 128, device="cpu")) == "int8"
    assert kvc.cache_format(kvc.make_fp8_kv_block(1, 2, 1, 128, device="cpu")) == "fp8_e4m3"
    assert kvc.quantization_mode(types.SimpleNamespace(kv_cache_quantization="fp8_e4m3")) == "fp8_e4m3"
    with pytest.raises(ValueError):
        kvc.quantization_mode(types.SimpleNamespace(kv_cache_quantization="fp4"))
    blk = kvc.make_fp8_kv_block(2, 10, 3, 128, device="cpu")
    assert kvc.kv_storage_bytes(blk) == 2 * (2 * 10 * 3 * 128) + 2 * (2 * 10 * 3 * 4)


def test_flop_and_byte_accounting():
    assert attention_flops(24960, 6240, 1, 24, 128, True, 1560) == pytest.approx(2.2134e12, rel=1e-4)
    assert attention_flops(24960, 6240, 1, 24, 128, True, 0) == pytest.approx(2.3928e12, rel=1e-4)
    # config 1 (CPU): 8 heads, 256 queries against 1024 + 256 keys (+1 text)
    assert attention_flops(1024, 256, 1, 8) == pytest.approx(4 * 8 * 128 * (257 * 1281), rel=1e-9)
    assert append_bytes(6241, 24) == 6241 * 24 * 2 * (256 + 128 + 4)   # 116.2 MB


def test_synthetic_generator_is_seeded_and_has_outliers():
    from hy_nomas_b200.synthetic import make_generator, seeded_kv
    a = seeded_kv((1, 64, 2, 128), make_generator(5))
    b = seeded_kv((1, 64, 2, 128), make_generator(5))
    assert torch.equal(a, b)
    per_channel = a.float().abs().mean(dim=(0, 1))        # [H, D]
    for h in range(2):
        assert (per_channel[h] > 4).sum() == 4


@pytest.mark.parametrize("L,P,layout", [(32760, 8, "zigzag"), (32760, 2, "zigzag"), (1001, 3, "zigzag"),
                                        (1001, 3, "contiguous"), (5, 4, "zigzag"), (0, 2, "zigzag")])
def test_ring_plan_partitions_the_sequence(L, P, layout):
    """Every token belongs to exactly one rank, segments increase, shard/unshard round-trips,
    and zig-zag balances the frame-causal work to within one frame-row per rank pair."""
    from hy_nomas_b200.ring import RingPlan
    plan = RingPlan(L, P, layout)
    owned = []
    for r in range(P):
        n0, p0, p1 = plan.positions(r)
        segs = [(p, n) for p, n in plan.segments[r] if n > 0]
        assert all(a[0] + a[1] <= b[0] for a, b in zip(segs, segs[1:]))
        if len([1 for _, n in plan.segments[r] if n > 0]) == 2:
            assert p1 >= p0 + n0
        for p, n in segs:
            owned.extend(range(p, p + n))
    assert sorted(owned) == list(range(L))
    n = 2 * P if layout == "zigzag" else P
    align = 256 if L >= n * 1024 else 1     # large chunks start on query-pair boundaries
    assert max(plan.length(r) for r in range(P)) - min(plan.length(r) for r in range(P)) <= 2 * align
    if L:
        x = torch.arange(L).view(1, L, 1, 1)
        assert torch.equal(plan.unshard([plan.shard(x, r) for r in range(P)]), x)
    if layout == "zigzag" and L >= 1000 and P > 1:
        T = 39
        def work(r):   # visible (query, key) pairs of rank r under the frame-causal rule
            tot = 0
            for p, n in plan.segments[r]:
                for i in range(p, p + n):
                    tot += (i // T + 1) * T if (i // T + 1) * T <= L else L
            return tot
        w = [work(r) for r in range(P)]
        assert max(w) / (sum(w) / P) < 1.02


def test_ring_plan_visibility_skips_future_blocks():
    from hy_nomas_b200.ring import RingPlan
    plan = RingPlan(400, 4, "contiguous")
    assert plan.visible(0, 0, 100) and not plan.visible(0, 1, 100) and plan.visible(3, 0, 100)
    assert plan.visible(0, 3, 0)            # no causal rule: every block is computed
    zz = RingPlan(400, 4, "zigzag")
    assert all(zz.visible(r, s, 50) for r in range(4) for s in range(4))


@pytest.mark.parametrize("sink,keep,appends", [(1, 3, [1, 1, 1, 1, 1, 2, 1, 3]), (0, 2, [1, 1, 1, 1]),
                                               (2, 4, [3, 4, 1, 1, 5])])
def test_window_ring_matches_reference_slide(sink, keep, appends):
    """The frame ring read through history_rows equals the reference's memmove slide
    (restated in oracle.window): sink frames then the last `keep` frames, in order."""
    from hy_nomas_b200.window import SinkWindowKVCache
    from oracle import window as ow
    T, H = 4, 1
    win = SinkWindowKVCache(1, H, T, sink, keep, storage_format="bf16", device="cpu")
    full = []          # reference cache: every frame appended, slid like the pipeline
    count = 0
    for n in appends:
        frames = torch.arange(count, count + n, dtype=torch.float32).repeat_interleave(T)
        k = frames.view(1, n * T, 1, 1).expand(1, n * T, H, 128).to(torch.bfloat16).contiguous()
        win.append(k, k)
        full.append(k)
        count += n
        assert win.history_frames() == ow.visible_frames(count, sink, keep)
        ref_k, ref_frames = ow.slide(torch.cat(full, 1), count, sink, keep, T)
        rows = win.history_rows()
        assert rows.dtype == torch.int32 and rows.numel() == win.valid_len == ref_frames * T
        got = win.cache["k"][:, rows.long()]
        assert torch.equal(got, ref_k[:, :ref_frames * T])


@pytest.mark.parametrize("L,P,layout", [(32760, 8, "zigzag"), (1001, 3, "zigzag"), (1001, 3, "contiguous"),
                                        (7, 4, "zigzag")])
def test_gather_chunks_lay_out_the_sequence(L, P, layout):
    """The all-gather schedule's chunk table: chunks tile [0, L) in order, and chunk rows index
    each owner's block in the order the owner holds its tokens."""
    from hy_nomas_b200.ring import RingPlan
    plan = RingPlan(L, P, layout)
    chunks = plan.gather_chunks()
    pos = 0
    for start, n, owner, row0 in chunks:
        assert start == pos and n > 0
        shard = plan.shard(torch.arange(L).view(1, L), owner)
        assert torch.equal(shard[0, row0:row0 + n], torch.arange(start, start + n))
        pos += n
    assert pos == L


def test_bench_reference_arm_prints_the_contract_line():
    """bench.py --impl reference (the reference's CPU path on the host cores) prints one JSON
    line with the metric, unit, impl and the e2e / cpu_baseline objects the driver reads."""
    import json
    import subprocess
    import sys
    from conftest import REPO
    res = subprocess.run([sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "0", "--cpu-heads", "1"], capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [ln for ln in res.stdout.strip().splitlines() if ln.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "TFLOP/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["cpu_baseline"]["value"] == d["value"] and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0


@pytest.mark.parametrize("P", [2, 4, 8])
def test_large_zigzag_chunks_start_on_query_pair_boundaries(P):
    """Config 3: every chunk but the last starts and ends on a 256-token boundary, so no query
    pair of the attention kernel holds rows of both of a rank's chunks."""
    from hy_nomas_b200.ring import RingPlan
    plan = RingPlan(21 * 1560, P, "zigzag")
    for r in range(P):
        (p0, n0), (p1, n1) = plan.segments[r]
        assert p0 % 256 == 0 and n0 % 256 == 0 and p1 % 256 == 0


def test_peer_exchange_needs_equal_lengths_and_divisible_heads(monkeypatch):
    from hy_nomas_b200 import communications as comm
    monkeypatch.delenv("HYB_PEER_EXCHANGE", raising=False)
    assert comm.peer_exchange_enabled((780,) * 8, 24)
    assert not comm.peer_exchange_enabled((780, 779), 24)       # uneven: NCCL path
    assert not comm.peer_exchange_enabled((780,) * 5, 24)       # heads not divisible
    assert not comm.peer_exchange_enabled((780,), 24)           # one rank: no exchange
    monkeypatch.setenv("HYB_PEER_EXCHANGE", "0")
    assert not comm.peer_exchange_enabled((780,) * 8, 24)


def test_installer_keeps_swa_writes_on_the_b200_path_except_archived_sampling():
    fake = types.SimpleNamespace(dtype=torch.bfloat16, is_cuda=True)   # a device tensor's two attributes
    recent = {"k": fake, "v": fake, "swa_capacity": 64}
    assert hinst._eligible(recent, True, None)
    for sampling in ("uniform", "recent_mix_uniform", "temporal_context"):
        archived = dict(recent, swa_sampling=sampling)
        assert not hinst._eligible(archived, True, None)
        assert hinst._eligible(archived, False, None)     # reads of an archived history stay here
    assert not hinst._eligible(recent, True, {"config": {}})   # sparse routing goes to the native path


def test_fallback_reaches_an_original_with_the_older_signature():
    """The reactor's CacheStaging (15 parameters, no sp_metadata / attention_metadata) may be the
    function this patch wraps; fallbacks must reach it, and the frame-causal extension must not
    be dropped silently on the way."""
    calls = []

    def staging(q, k, v, kv_cache, cache_valid_len=0, attn_mode=None, text_mask=None, update_cache=False,
                cache_txt=True, cache_mask=None, intra_seg_txt_offsets=None, intra_seg_vid_windows=None,
                tokens_per_frame=0, seg_ar_attention_backend="magi", sparse_context=None):
        calls.append((cache_valid_len, attn_mode, tokens_per_frame))
        return "staging"

    mod = types.SimpleNamespace(causal_attention_with_cache_mp=staging,
                                get_sequence_parallel_state=lambda: False,
                                nccl_info=types.SimpleNamespace(sp_group=None, rank_within_spgroup=0))
    hinst.install(mod)
    try:
        patched = mod.causal_attention_with_cache_mp
        x = torch.zeros(1, 2, 2, 128, dtype=torch.bfloat16)
        cache = {"k": torch.zeros(1, 4, 2, 128, dtype=torch.bfloat16), "v": torch.zeros(1, 4, 2, 128, dtype=torch.bfloat16)}
        assert patched((x, x), (x, x), (x, x), cache, 0, "flash3", tokens_per_frame=16,
                       sp_metadata=None, attention_metadata=None) == "staging"
        assert calls == [(0, "flash3", 16)]
        with pytest.raises(NotImplementedError, match="chunk_causal_frames"):
            patched((x, x), (x, x), (x, x), cache, 0, "flash3", tokens_per_frame=16, chunk_causal_frames=1)
    finally:
        hinst.uninstall(mod)
    hatt.set_parallel_state_provider(hatt._ps.get_sequence_parallel_state, hatt._ps.nccl_info)


def test_kv_cache_errors_are_the_reference_ones_and_write_nothing():
    """Exception types and messages of the reference's INT8 cache API
    (hymm/models/dit/modules/int8_kv_cache.py:114-181), raised before anything is written."""
    cache = kvc.make_int8_kv_block(1, 8, 2, 128, device="cpu")
    before = {k: v.clone() for k, v in cache.items() if torch.is_tensor(v)}
    x = torch.zeros(1, 4, 2, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="^K/V shapes, dtypes, and devices must match$"):
        kvc.quantize_kv_pair_into(cache, x, x[:, :3], 0)
    for bad, start in ((torch.zeros(2, 4, 2, 128, dtype=torch.bfloat16), 0),   # batch
                       (x, 5),                                                   # capacity
                       (x, -1),
                       (x.float(), 0)):                                          # dtype
        with pytest.raises(ValueError, match="^KV pair shape, capacity, dtype, or device mismatch$"):
            kvc.quantize_kv_pair_into(cache, bad, bad, start)
    with pytest.raises(ValueError, match="^Invalid KV key: q$"):
        kvc.quantize_kv_into(cache, "q", x, 0)
    with pytest.raises(TypeError, match="^KV quantization expects \\[B,L,H,D\\] BF16 values$"):
        kvc.quantize_kv_into(cache, "k", x.float(), 0)
    with pytest.raises(ValueError, match="^KV quantization shape, capacity, or device mismatch$"):
        kvc.quantize_kv_into(cache, "k", x, 6)
    wrong_scale = dict(cache, k_scale=torch.ones(1, 8, 2, 2))
    with pytest.raises(ValueError, match="^INT8 KV scale shape/device mismatch$"):
        kvc.quantize_kv_into(wrong_scale, "k", x, 0)
    with pytest.raises(TypeError, match="FP32 scale are required"):
        kvc.quantize_kv_into(dict(cache, k_scale=cache["k_scale"].double()), "k", x, 0)
    with pytest.raises(ValueError, match="^Invalid KV valid length$"):
        kvc.dequantize_kv(cache, "k", 9)
    for k, v in before.items():
        assert torch.equal(cache[k], v)


def test_inputs_in_other_layouts_are_copied_once_into_kernel_rows():
    x = torch.randn(1, 6, 2, 128).to(torch.bfloat16)
    assert hatt._kernel_layout(x) is x                                   # the DiT's layout passes through
    assert hatt._kernel_layout(x[:, 2:]) is not None and hatt._kernel_layout(x[:, 2:]).data_ptr() == x[:, 2:].data_ptr()
    t = x.transpose(2, 3).contiguous().transpose(2, 3)                  # head_dim not the unit stride
    y = hatt._kernel_layout(t)
    assert y.stride(-1) == 1 and torch.equal(y, t)
    flat = torch.randn(1 * 6 * 2 * 128 + 1).to(torch.bfloat16)
    odd = flat[1:].view(1, 6, 2, 128)                                    # contiguous but 2 bytes off
    z = hatt._kernel_layout(odd)
    assert z.data_ptr() % 16 == 0 and torch.equal(z, odd)


def test_tensors_on_another_device_are_refused_before_any_kernel():
    """A tensor on another device would hand the kernels a pointer they cannot dereference;
    the reference fails on such inputs in torch's own device checks, this build before any
    launch."""
    from hy_nomas_b200 import _lib
    elsewhere = torch.empty(1, 4, dtype=torch.bool, device="meta")
    _lib.require_same_device(torch.device("cpu"), "x", torch.zeros(1), None)
    with pytest.raises(RuntimeError, match="must be on the same device"):
        _lib.require_same_device(torch.device("cpu"), "x", torch.zeros(1), elsewhere)
    x = torch.zeros(1, 16, 2, 128, dtype=torch.bfloat16)
    t = torch.zeros(1, 4, 2, 128, dtype=torch.bfloat16)
    cache = {"k": torch.zeros(1, 32, 2, 128, dtype=torch.bfloat16), "v": torch.zeros(1, 32, 2, 128, dtype=torch.bfloat16)}
    with pytest.raises(RuntimeError, match="must be on the same device"):
        hatt.cached_attention_local(x, x, x, t, t, t, cache, 0, text_mask=elsewhere)


def test_mask_shapes_are_checked_before_any_kernel():
    x = torch.zeros(1, 16, 2, 128, dtype=torch.bfloat16)
    t = torch.zeros(1, 3, 2, 128, dtype=torch.bfloat16)
    cache = {"k": torch.zeros(1, 32, 2, 128, dtype=torch.bfloat16), "v": torch.zeros(1, 32, 2, 128, dtype=torch.bfloat16)}
    with pytest.raises(ValueError, match=r"history mask must be bool \[1 or 1, >= 20\], got \(1, 10\)"):
        hatt.cached_attention_local(x, x, x, t, t, t, cache, 20, history_mask=torch.ones(1, 10, dtype=torch.bool))
    with pytest.raises(ValueError, match="history mask must be"):
        hatt.cached_attention_local(x, x, x, t, t, t, cache, 20, history_mask=torch.ones(3, 32, dtype=torch.bool))
    with pytest.raises(ValueError, match=r"history mask must be bool \[1 or 1, >= 32\]"):
        hatt.cached_attention_local(x, x, x, t, t, t, cache, 4, history_mask=torch.ones(1, 20, dtype=torch.bool),
                                    hist_rows=torch.arange(4, dtype=torch.int32))
    with pytest.raises(ValueError, match=r"text mask must be bool \[1, 3\], got \(1, 2\)"):
        hatt.cached_attention_local(x, x, x, t, t, t, cache, 20, text_mask=torch.ones(1, 2, dtype=torch.bool))


def test_a_row_map_without_its_window_must_name_cache_rows(monkeypatch):
    """The drop-in reads history through ``history_rows``; a map that does not come with its
    window cache is range-checked before the staging kernel could read a row outside the cache."""
    from hy_nomas_b200 import _lib
    monkeypatch.setattr(_lib, "require_device", lambda t: None)   # the check precedes every launch
    x = torch.zeros(1, 16, 2, 128, dtype=torch.bfloat16)
    t = torch.zeros(1, 1, 2, 128, dtype=torch.bfloat16)
    cache = {"k": torch.zeros(1, 32, 2, 128, dtype=torch.bfloat16), "v": torch.zeros(1, 32, 2, 128, dtype=torch.bfloat16),
             "history_rows": torch.tensor([0, 5, 40], dtype=torch.int32)}
    with torch.no_grad(), pytest.raises(ValueError, match="history_rows must name rows of the cache"):
        hatt.causal_attention_with_cache_mp((x, t), (x, t), (x, t), cache, cache_valid_len=3, attn_mode="flash3")


def test_kv_stationary_slice_choice():
    """Key slices per query pair of a partial-scatter launch: enough CTAs to fill the SMs,
    never fewer than 4 key tiles a slice (config 5 at P = 8: 1,561 queries x 24 heads against
    6,631 keys on each rank)."""
    from hy_nomas_b200.kv_stationary import choose_slices
    s = choose_slices(1, 24, 1561, 6631, 148)
    assert 2 <= s <= 8
    assert choose_slices(1, 24, 1561, 300, 148) == 1
    assert choose_slices(1, 2, 256, 128 * 64, 148) >= 8


def test_decoded_mirrors_are_for_quantised_caches_only():
    """A decoded mirror holds the decode of codes: a bf16 cache or window has nothing to decode,
    and asking for one is an error before any allocation or kernel."""
    from hy_nomas_b200 import kv_cache as kvc
    from hy_nomas_b200.window import SinkWindowKVCache
    plain = {"k": torch.zeros(1, 8, 2, 128, dtype=torch.bfloat16), "v": torch.zeros(1, 8, 2, 128, dtype=torch.bfloat16)}
    with pytest.raises(TypeError):
        kvc.attach_decoded_mirror(plain)
    assert "staged" not in plain
    with pytest.raises(ValueError, match="quantised"):
        SinkWindowKVCache(1, 2, 16, 1, 2, storage_format="bf16", device="cpu", decoded=True)
    win = SinkWindowKVCache(1, 2, 16, 1, 2, storage_format="fp8_e4m3", device="cpu", decoded=True, tail_rows=8)
    mk, mv, pitch = win.view()["staged"]
    assert pitch == 3 * 16 + 8 and tuple(mk.shape) == (1, 2, pitch, 128)
    assert mk.dtype == torch.bfloat16 and mv.dtype == torch.float16


@pytest.mark.parametrize("layout", ["zigzag", "contiguous"])
@pytest.mark.parametrize("world,L", [(2, 32760), (4, 32760), (8, 32760), (3, 1000), (8, 300)])
def test_overlapped_ring_groups_cover_every_other_chunk(layout, world, L):
    """The overlapped ring schedule attends each rank's own chunks, then the other ranks' chunks
    in at most two launches of at most two position segments each; together they are every
    chunk of the sequence exactly once."""
    from hy_nomas_b200.ring import RingPlan, overlap_groups, position_segments
    plan = RingPlan(L, world, layout)
    for r in range(world):
        mine, groups = overlap_groups(plan, r)
        assert len(groups) <= 2 and all(len(position_segments(g)) <= 2 for g in groups)
        seen = sorted(c for g in [mine] + groups for c in g)
        assert seen == plan.gather_chunks()
        assert sum(c[1] for c in mine) == plan.length(r)
        for g in groups:
            assert g == sorted(g) and all(c[2] != r for c in g)
