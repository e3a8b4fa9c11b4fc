#!/usr/bin/env python
"""Benchmark of the B200 chunk-causal cached attention (BASELINE config 2 at N = 1).

One step = one ``causal_attention_with_cache_mp`` call of a 4-frame chunk (4 x 1560
image tokens + 1 text token, 24 heads x 128) against a 16-frame E4M3 KV cache
(24,960 tokens) with frame-level block-causal masking, including the quantise-on-write
append of the chunk into the cache.  Metric: attention TFLOP/s, FLOPs = 4*H*D*(visible
query-key pairs) = 2.213 TFLOP per step.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

N > 1 (launched with torchrun, one rank per GPU): Ulysses sequence parallelism over the
same global chunk (strong scaling): every rank holds 6240/N image tokens and 24/N heads
of the head-sharded cache; Q/K/V and O cross NVLink through NCCL all_to_all_single.

``--impl reference`` times the reference's CPU path (restated in oracle/: decode the
INT8-style history, append the chunk, torch.cat, one SDPA call with the mask) on the
host cores, on a sample of the heads; it prints the same metric and config.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

H_TOTAL, D, T = 24, 128, 1560
HIST_FRAMES, CHUNK_FRAMES, TXT = 16, 4, 1
METRIC = "chunk-causal attn TFLOP/s (config 2: 4-frame chunk vs 16-frame FP8 KV cache, frame-causal)"
METRIC4 = "chunk-causal attn TFLOP/s (config 4: 4-frame chunk vs 48-frame FP8 KV cache, frame-causal)"
METRIC5 = "long-rollout attn TFLOP/s (config 5: 1-frame chunks vs sink + 32-frame window FP8 cache, append each step)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--cpu-heads", type=int, default=4, help="heads in the CPU baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e-timeline", action="store_true",
                    help="after the measurement, one more pass of the end-to-end loop with CUDA events around "
                         "each upload / compute / read-back, and the host link alone; printed to stderr")
    ap.add_argument("--ring-schedule", default="allgather", choices=["allgather", "allgather_overlap", "ring"],
                    help="ring workload: every block to every rank over peer memory, or neighbour passing")
    ap.add_argument("--library-comparison", action="store_true",
                    help="time this kernel and flashinfer's CUTLASS sm100a FMHA (fmha_varlen) on the same bf16 "
                         "Q/K/V of config-2 size, chunk-bidirectional, and print both (one GPU)")
    ap.add_argument("--measure-fp8-peak", action="store_true",
                    help="print the dense FP8 GEMM peak of this GPU (burst and 4 s sustained) and exit")
    ap.add_argument("--no-config3", action="store_true",
                    help="config 2: skip the config-3 ring measurement reported in the same line")
    ap.add_argument("--no-decoded-cache", action="store_true",
                    help="config 2: skip the measurement over a cache that keeps its rows decoded")
    ap.add_argument("--no-decoded-window", action="store_true",
                    help="rollout: decode the whole window on every call instead of once per appended frame")
    ap.add_argument("--no-graph", action="store_true",
                    help="time eager calls instead of replaying one captured CUDA graph of the call")
    ap.add_argument("--sp-scheme", default="auto", choices=["auto", "ulysses", "kv"],
                    help="rollout at N > 1: Ulysses over head-sharded windows, or KV-stationary over "
                         "sequence-sharded windows (Q all-gather, partial rows scattered to their owners); "
                         "auto: KV-stationary from 4 GPUs on (measured faster at N = 8, 0.30 vs 0.36 ms; "
                         "Ulysses at N = 2, 0.729 vs 0.742 ms)")
    ap.add_argument("--workload", default="config2", choices=["config2", "config4", "ring", "rollout"],
                    help="config2: 4-frame chunk vs 16-frame FP8 cache (Ulysses for N > 1); "
                         "config4: the same chunk vs a 48-frame cache; "
                         "ring: config 3, 32,760-token frame-causal sequence, ring SP over N ranks; "
                         "rollout: config 5, 1-frame chunks vs sink + 32-frame window, append each step")
    return ap.parse_args()


def load_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get("bf16_tflops", 1590.0), d.get("hbm_gbs", 6650.0), "measured"
    return 1590.0, 6650.0, "fallback"


def measure_fp8_peak(device, sustained_s=0.0):
    """Dense FP8 (e4m3) GEMM throughput on this GPU: torch._scaled_mm 8192^3 (2 N^3 FLOP),
    best of 10 launches (burst) and, with sustained_s > 0, back to back for that long.
    TFLOP/s."""
    N = 8192
    a = torch.randn(N, N, device=device).to(torch.float8_e4m3fn)
    b = torch.randn(N, N, device=device).to(torch.float8_e4m3fn).t()
    one = torch.ones((), device=device)

    def mm():
        return torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)

    for _ in range(3):
        mm()
    torch.cuda.synchronize(device)
    best = float("inf")
    for _ in range(10):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        mm()
        e1.record()
        torch.cuda.synchronize(device)
        best = min(best, e0.elapsed_time(e1))
    out = {"burst": round(2 * N ** 3 / (best * 1e-3) / 1e12, 1)}
    if sustained_s > 0:
        n = 0
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        t = time.time()
        while time.time() - t < sustained_s:
            for _ in range(20):
                mm()
            n += 20
            torch.cuda.synchronize(device)
        e1.record()
        torch.cuda.synchronize(device)
        out["sustained"] = round(2 * N ** 3 * n / (e0.elapsed_time(e1) * 1e-3) / 1e12, 1)
    del a, b
    torch.cuda.empty_cache()
    return out


def load_traffic():
    p = REPO / "profiles" / "traffic.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except Exception:
            return {}
    return {}


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.file = None

    def start(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=self.file, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.file.flush()
        rows = [r.split(",") for r in Path(self.file.name).read_text().strip().splitlines() if r.strip()]
        os.unlink(self.file.name)
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = max(mx, float(r[2]))
                for name, val in zip(names, r[5:9]):
                    if val.strip().lower() == "active":
                        reasons.add(name)
            except (ValueError, IndexError):
                continue
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def capture_step(step_fn, device):
    """CUDA graph of one call of ``step_fn`` (all kernels and NCCL collectives of one step on
    the capture stream); its replay repeats exactly that work on the same buffers.  Warm-up
    calls run first on a side stream, as graph capture requires."""
    side = torch.cuda.Stream(device=device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        for _ in range(2):
            step_fn()
    torch.cuda.current_stream(device).wait_stream(side)
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step_fn()
    torch.cuda.synchronize(device)
    return graph


def e2e_pipelined(step_fn, host_in, device, steps, warmup, world, static_outputs=False, log=None):
    """Mean ms per step through the public call with host buffers: every step copies its
    inputs from pinned host memory (H2D stream) and reads its outputs back into pinned host
    memory (D2H stream); inputs are double-buffered so that step i+1's copies overlap step
    i's compute.  With ``static_outputs`` (a graphed call returns the same output tensors for
    a buffer set) a step also waits until the read-back of step i-2 has finished.
    Device-timed on the caller's stream, max over ranks.  With ``log`` (a list), every timed
    step appends a dict of timing events around its upload, compute and read-back, and the
    region's start event is appended first."""
    import torch.distributed as dist
    compute = torch.cuda.current_stream(device)
    h2d = torch.cuda.Stream(device=device)
    d2h = torch.cuda.Stream(device=device)
    dev_in = [[torch.empty_like(t, device=device) for t in host_in] for _ in range(2)]
    host_out = [None, None]
    out_bytes = [0]

    def ev(rec, name, stream):
        if rec is not None:
            e = torch.cuda.Event(enable_timing=True)
            e.record(stream)
            rec[name] = e

    def run(n, start_event=None, timeline=None):
        free = [None, None]
        read_back = [None, None]
        for i in range(n):
            j = i % 2
            rec = {} if timeline is not None else None
            with torch.cuda.stream(h2d):
                if i == 0 and start_event is not None:
                    h2d.wait_event(start_event)
                if free[j] is not None:
                    h2d.wait_event(free[j])
                ev(rec, "up0", h2d)
                for d_, h_ in zip(dev_in[j], host_in):
                    d_.copy_(h_, non_blocking=True)
                copied = torch.cuda.Event()
                copied.record(h2d)
                ev(rec, "up1", h2d)
            compute.wait_event(copied)
            if static_outputs and read_back[j] is not None:
                compute.wait_event(read_back[j])
            ev(rec, "c0", compute)
            outs = step_fn(*dev_in[j])
            done = torch.cuda.Event()
            done.record(compute)
            ev(rec, "c1", compute)
            free[j] = done
            if host_out[j] is None:
                host_out[j] = [torch.empty(o.shape, dtype=o.dtype).pin_memory() for o in outs]
                out_bytes[0] = sum(o.numel() * o.element_size() for o in outs)
            with torch.cuda.stream(d2h):
                d2h.wait_event(done)
                ev(rec, "down0", d2h)
                for h_, o in zip(host_out[j], outs):
                    h_.copy_(o, non_blocking=True)
                    o.record_stream(d2h)
                back = torch.cuda.Event()
                back.record(d2h)
                ev(rec, "down1", d2h)
                read_back[j] = back
            if timeline is not None:
                timeline.append(rec)
        compute.wait_stream(h2d)
        compute.wait_stream(d2h)

    nwarm = max(6 if static_outputs else 2, warmup)
    if static_outputs and nwarm % 2:
        nwarm += 1   # static outputs alternate between two sets: the timed loop starts on set 0
    run(nwarm)   # a graphed call captures both buffer sets here
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(compute)
    if log is not None:
        log.append(e0)
    run(steps, start_event=e0, timeline=log)
    e1.record(compute)
    torch.cuda.synchronize(device)
    ems = e0.elapsed_time(e1) / steps
    if world > 1:
        tt = torch.tensor([ems], device=device)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ems = tt.item()
    h2d_bytes = sum(t.numel() * t.element_size() for t in host_in) * world
    return ems, h2d_bytes, out_bytes[0] * world


def dist_setup(n_gpus):
    import torch.distributed as dist
    if n_gpus <= 1:
        return 0, 1, 0
    if os.environ.get("NCCL_DEBUG", "VERSION").upper() == "VERSION":
        os.environ["NCCL_DEBUG"] = "WARN"   # keep stdout to the one JSON line
    import datetime
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    # The communicator prints a version banner on stdout during its first use; route fd 1 to
    # stderr while it is created so rank 0's stdout carries only the JSON line.
    sys.stdout.flush()
    saved = os.dup(1)
    os.dup2(2, 1)
    try:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        dist.barrier()
        torch.cuda.synchronize()
    finally:
        sys.stdout.flush()
        os.dup2(saved, 1)
        os.close(saved)
    return rank, world, local


def build_problem(rank, world, device, hist_frames=HIST_FRAMES):
    """Global chunk of config 2 (config 4: 48 history frames) split for Ulysses SP over
    `world` ranks."""
    from hy_nomas_b200 import kv_cache as kvc
    from hy_nomas_b200.synthetic import make_generator, seeded_kv
    Lh = hist_frames * T
    Li = CHUNK_FRAMES * T
    Hl = H_TOTAL // world
    gen = make_generator(1236 + rank, device=device)
    # head-sharded cache: this rank's heads for the whole history (+ room for the chunk)
    cap = Lh + Li + TXT
    cache = kvc.make_fp8_kv_block(1, cap, Hl, D, device=device)
    with torch.no_grad():
        hk = seeded_kv((1, Lh, Hl, D), gen, device=device)
        hv = seeded_kv((1, Lh, Hl, D), gen, device=device)
        kvc.quantize_kv_pair_into(cache, hk, hv, 0)
        del hk, hv
    Ls = Li // world
    img = [seeded_kv((1, Ls, H_TOTAL, D), gen, device=device) for _ in range(3)]
    # the text tokens are replicated on every rank (the reference's SP callers hold the whole
    # text and slice its heads), so they come from one generator shared by all ranks
    gen_txt = make_generator(1236 + 1000, device=device)
    txt = [seeded_kv((1, TXT, H_TOTAL, D), gen_txt, device=device) for _ in range(3)]
    cache_mask = torch.zeros(1, cap, dtype=torch.bool, device=device)
    cache_mask[:, :Lh] = True
    return dict(cache=cache, img=img, txt=txt, cache_mask=cache_mask, Lh=Lh, Li=Li, Ls=Ls, Hl=Hl)



def print_e2e_timeline(step_fn, host_in, device, steps, world, rank, static_outputs):
    """One more pass of the end-to-end loop with CUDA events around every upload, compute and
    read-back, then the host link alone (the step's uploads with nothing else running);
    printed to stderr.  Every rank runs it (the loop holds collectives)."""
    log = []
    ems, _, _ = e2e_pipelined(step_fn, host_in, device, steps, 0, world, static_outputs, log=log)
    dev_in = [torch.empty_like(t, device=device) for t in host_in]
    stream = torch.cuda.current_stream(device)

    def upload():
        for d_, h_ in zip(dev_in, host_in):
            d_.copy_(h_, non_blocking=True)

    for _ in range(3):
        upload()
    torch.cuda.synchronize(device)
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(5):
        upload()
    b.record(stream)
    torch.cuda.synchronize(device)
    up_ms = a.elapsed_time(b) / 5
    if rank != 0:
        return
    t0 = log[0]
    out = sys.stderr
    nbytes = sum(t.numel() * t.element_size() for t in host_in)
    print(f"e2e timeline: {ems:.3f} ms per step over {steps} steps; times in ms from the region's start", file=out)
    for i, r in enumerate(log[1:]):
        def at(k, r=r):
            return t0.elapsed_time(r[k])
        print(f"  step {i:3d}  upload {at('up0'):8.3f}-{at('up1'):8.3f} ({at('up1') - at('up0'):6.3f})  "
              f"compute {at('c0'):8.3f}-{at('c1'):8.3f} ({at('c1') - at('c0'):6.3f})  "
              f"read-back {at('down0'):8.3f}-{at('down1'):8.3f} ({at('down1') - at('down0'):6.3f})", file=out)
    print(f"  the step's uploads alone: {up_ms:.3f} ms for {nbytes / 1e6:.1f} MB = {nbytes / up_ms / 1e6:.1f} GB/s",
          file=out)


# ------------------------------------------------------------------------------ parity check
# Before timing, every rank checks its own output rows of a few sampled heads against the exact
# attention of the same inputs, computed in float64 with plain torch on its GPU (what the drop-in
# returns in bf16 must be within 2e-2 of it beyond the bf16 rounding any bf16 output carries,
# cosine >= 0.9995).  Inputs a rank does not hold (other ranks' sequence shards, the owner's
# history of a head) arrive over the process group, outside the timed region.
PARITY_HEADS = (0, H_TOTAL - 1)


def _exact_rows(q, k, v, vis):
    """float64 softmax(q k^T / sqrt(D)) v of q [Lq, D] over k/v [Lk, D] with visibility [Lq, Lk]."""
    s = (q.double() @ k.double().T) / (q.shape[-1] ** 0.5)
    s = s.masked_fill(~vis, float("-inf"))
    return torch.softmax(s, dim=-1) @ v.double()


def _gate(got, exact):
    """(max-abs error, cosine, bf16 floor of the exact rows) of bf16 rows against float64 rows."""
    g, e = got.double().flatten(), exact.double().flatten()
    floor = (e.float().to(torch.bfloat16).double() - e).abs().max().item()
    mae = (g - e).abs().max().item()
    cos = torch.nn.functional.cosine_similarity(g[None], e[None]).item()
    return mae, cos, floor


def _reduce_parity(rows, world, device):
    """Combine per-rank (mae, cos, floor, excess) lists: worst over heads and ranks."""
    import torch.distributed as dist
    mae = max(r[0] for r in rows)
    cos = min(r[1] for r in rows)
    excess = max(r[0] - (2e-2 + r[2]) for r in rows)
    floor = max(r[2] for r in rows)
    if world > 1:
        t = torch.tensor([mae, -cos, excess, floor], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        mae, cos, excess, floor = t[0].item(), -t[1].item(), t[2].item(), t[3].item()
    return {"max_abs": round(mae, 6), "cos": round(cos, 7), "bf16_floor": round(floor, 6),
            "gate": "max_abs <= 2e-2 + bf16 rounding floor of the exact rows, cos >= 0.9995",
            "heads_checked": list(PARITY_HEADS), "ranks_checked": world,
            "reference": "float64 torch attention of the same inputs on each rank's GPU",
            "ok": bool(excess <= 0.0 and cos >= 0.9995)}


def verify_ulysses(prob, outs, rank, world, device):
    """Parity of this rank's output rows (sequence shard ``rank``) for the sampled heads."""
    import torch.distributed as dist
    out_img, out_txt = outs
    Lh, Li, Ls, Hl = prob["Lh"], prob["Li"], prob["Ls"], prob["Hl"]
    cache, img, txt = prob["cache"], prob["img"], prob["txt"]
    out_img = out_img.reshape(1, Ls, H_TOTAL, D)
    out_txt = out_txt.reshape(1, TXT, H_TOTAL, D)
    rows = []
    for h in PARITY_HEADS:
        owner, hl = h // Hl, h % Hl
        hist = torch.empty((2, Lh, D), dtype=torch.bfloat16, device=device)
        if rank == owner:   # the owner's head-sharded history, decoded as the reference decodes it
            for i, n in enumerate("kv"):
                hist[i] = (cache[n][0, :Lh, hl].float() * cache[f"{n}_scale"][0, :Lh, hl]).to(torch.bfloat16)
        if world > 1:
            dist.broadcast(hist, src=owner)
        kv_img = []
        for x in (img[1], img[2]):
            mine = x[0, :, h].contiguous()
            if world > 1:
                parts = [torch.empty_like(mine) for _ in range(world)]
                dist.all_gather(parts, mine)
                mine = torch.cat(parts, 0)
            kv_img.append(mine)
        k = torch.cat([hist[0], kv_img[0], txt[1][0, :, h]], 0)
        v = torch.cat([hist[1], kv_img[1], txt[2][0, :, h]], 0)
        Lk = k.shape[0]
        kpos = torch.arange(Lk, device=device)
        kframe = torch.where((kpos >= Lh) & (kpos < Lh + Li), (kpos - Lh) // T, torch.full_like(kpos, -1))
        qframe = (rank * Ls + torch.arange(Ls, device=device)) // T
        vis = kframe[None, :] <= qframe[:, None]
        exact_img = _exact_rows(img[0][0, :, h], k, v, vis)
        exact_txt = _exact_rows(txt[0][0, :, h], k, v, torch.ones(TXT, Lk, dtype=torch.bool, device=device))
        got = torch.cat([out_img[0, :, h], out_txt[0, :, h]], 0)
        rows.append(_gate(got, torch.cat([exact_img, exact_txt], 0)))
    return _reduce_parity(rows, world, device)


def run_b200(args):
    from hy_nomas_b200 import _lib
    from hy_nomas_b200 import attention as hatt
    from hy_nomas_b200 import parallel_states as ps
    from hy_nomas_b200.flops import attention_flops
    import torch.distributed as dist

    rank, world, local = dist_setup(args.gpus)
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        ps.initialize_sequence_parallel_group()
    os.environ["HYB_ASSUME_FINITE_KV"] = "1"   # validation stays on the device (status word)
    hist_frames = 48 if args.workload == "config4" else HIST_FRAMES
    prob = build_problem(rank, world, device, hist_frames)
    Lh, Li, Ls, Hl = prob["Lh"], prob["Li"], prob["Ls"], prob["Hl"]
    cache, cmask = prob["cache"], prob["cache_mask"]
    img, txt = prob["img"], prob["txt"]
    flops_total = attention_flops(Lh, Li, TXT, H_TOTAL, D, True, T)
    stream = torch.cuda.current_stream(device)
    sp_metadata = None
    if world > 1:
        # Computed once per model forward and passed to every layer, as the reference's
        # forward_with_cache does (nomas_cpt.py:3486-3488).
        from hy_nomas_b200 import communications as comm
        sp_metadata = comm.prepare_sp_communication(Ls, H_TOTAL, device, ps.nccl_info.sp_group)

    def step(q_img, k_img, v_img, q_txt, k_txt, v_txt):
        with torch.no_grad():
            return hatt.causal_attention_with_cache_mp(
                (q_img, q_txt), (k_img, k_txt), (v_img, v_txt), cache, cache_valid_len=Lh,
                attn_mode="flash3", update_cache=True, cache_txt=True, cache_mask=cmask,
                tokens_per_frame=T, seg_ar_attention_backend="b200", sp_metadata=sp_metadata,
                chunk_causal_frames=1)

    for _ in range(args.warmup):
        step(*img, *txt)
    torch.cuda.synchronize(device)
    parity = verify_ulysses(prob, step(*img, *txt), rank, world, device)
    torch.cuda.synchronize(device)
    graph = None if args.no_graph else capture_step(lambda: step(*img, *txt), device)
    run_step = (lambda: step(*img, *txt)) if graph is None else graph.replay
    for _ in range(args.warmup):
        run_step()
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    sampler = ClockSampler(local)
    sampler.start()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    t0.record(stream)
    for _ in range(args.steps):
        run_step()
    t1.record(stream)
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    ms = t0.elapsed_time(t1) / args.steps
    if world > 1:
        tt = torch.tensor([ms], device=device)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = tt.item()
    _lib.check_device_status(device)
    value = flops_total / (ms * 1e-3) / 1e12

    # ---- end-to-end through the public API with pinned host buffers
    from hy_nomas_b200.graphs import GraphedCall
    host_in = [t.cpu().pin_memory() for t in (*img, *txt)]
    call = step if args.no_graph else GraphedCall(step, device)
    ems, h2d, d2h = e2e_pipelined(call, host_in, device, args.steps, args.warmup, world,
                                  static_outputs=not args.no_graph)
    if args.e2e_timeline:
        print_e2e_timeline(call, host_in, device, args.steps, world, rank, static_outputs=not args.no_graph)

    # ---- dominant kernel alone: the tcgen05 attention launch over the staged buffers
    kern = time_attention_kernel(prob, device, args.steps)
    cfg_no = 4 if args.workload == "config4" else 2
    peak_bf16, peak_hbm, peak_src = load_peaks()
    fp8 = measure_fp8_peak(device) if rank == 0 else {"burst": None}
    local_flops = attention_flops(Lh, Li, TXT, Hl, D, True, T)
    achieved = local_flops / (kern["ms"] * 1e-3) / 1e12
    tr = load_traffic() if args.workload == "config2" else {}
    traffic = tr.get("attn_fwd_config2_bytes_per_launch")
    if traffic is not None and world > 1:
        traffic = traffic * Hl / H_TOTAL

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(args.cpu_heads, reps=2)

    # ---- the same step over a cache that keeps its rows decoded (kv_cache.attach_decoded_mirror):
    # each step decodes only the chunk it writes, the history comes from the mirror.  Reported
    # beside the headline, which decodes the whole history on every call as the reference does.
    decoded = None
    if args.workload == "config2" and not args.no_decoded_cache:
        from hy_nomas_b200 import kv_cache as kvc
        kvc.attach_decoded_mirror(cache)
        parity_d = verify_ulysses(prob, step(*img, *txt), rank, world, device)
        graph_d = None if args.no_graph else capture_step(lambda: step(*img, *txt), device)
        run_d = (lambda: step(*img, *txt)) if graph_d is None else graph_d.replay
        for _ in range(args.warmup):
            run_d()
        torch.cuda.synchronize(device)
        if world > 1:
            dist.barrier()
        d0 = torch.cuda.Event(enable_timing=True)
        d1 = torch.cuda.Event(enable_timing=True)
        d0.record(stream)
        for _ in range(args.steps):
            run_d()
        d1.record(stream)
        torch.cuda.synchronize(device)
        ms_d = d0.elapsed_time(d1) / args.steps
        if world > 1:
            tt = torch.tensor([ms_d], device=device)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            ms_d = tt.item()
        _lib.check_device_status(device)
        decoded = {"value": round(flops_total / (ms_d * 1e-3) / 1e12, 2), "ms_per_step": round(ms_d, 4),
                   "parity": parity_d,
                   "what": "same step, CUDA-graph replay, over a cache keeping a decoded bf16/fp16 mirror: the step "
                           "decodes the chunk it writes (after its attention), the history is read from the mirror "
                           "(decoded when it was written, untimed prefill)"}
        del graph_d, run_d
        cache.pop("staged", None)

    del graph, run_step   # graphs holding NCCL calls are released before the process group
    if not args.no_graph:
        call.release()
    torch.cuda.synchronize(device)
    config3 = None
    if args.workload == "config2" and not args.no_config3:
        # BASELINE config 3 (ring SP over the same ranks), reported beside config 2
        del prob, cache, cmask, img, txt
        torch.cuda.empty_cache()
        config3 = ring_measurement(args, rank, world, device)
    gpus = None
    if world > 1:
        from hy_nomas_b200 import communications as comm2
        from hy_nomas_b200 import parallel_states as ps2
        comm2.release_peer_exchanges()
        ps2.destroy_sequence_parallel_group()
        gpus = _gpus_active(world, device)
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC if cfg_no == 2 else METRIC4, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None, "dtype": "bf16 Q.K^T / fp16 P.V MMAs, fp32 softmax; e4m3 KV cache",
        "data": "synthetic (seeded N(0,1), 4 outlier channels/head x8)",
        "config": {"workload": ("config 2: 1x B200 single block (N>1: Ulysses SP over the same chunk)" if cfg_no == 2
                                else "config 4: 4-frame chunk vs 48-frame FP8 cache (N>1: Ulysses SP)"),
                   "heads": H_TOTAL, "head_dim": D, "history_tokens": Lh, "chunk_image_tokens": Li,
                   "text_tokens": TXT, "tokens_per_frame": T, "mask": "frame-level block-causal (G=1)",
                   "kv_cache": "fp8_e4m3 per-token-per-head scale", "append": "quantise-on-write of the chunk each step",
                   "parallelism": f"ulysses_sp{world}" if world > 1 else "single",
                   "exchange": ("peer memory (CUDA IPC push kernels + device barrier)"
                                if world > 1 and os.environ.get("HYB_PEER_EXCHANGE", "1") != "0"
                                else ("NCCL all_to_all_single" if world > 1 else None)),
                   "timed_call": "eager" if args.no_graph else "CUDA graph replay of one drop-in call",
                   "l2": f"inputs larger than L2 ({2 * Lh * H_TOTAL * D / 1e6:.0f} MB FP8 history + 115 MB bf16 chunk "
                         "per step)",
                   "tflop_per_step": round(flops_total / 1e12, 4)},
        # per step: append, mask, stage K/V, stage Q, attention (+ split merge), and for N > 1
        # the Ulysses pack and unpack kernels
        "gpu_launches": args.steps * (4 + kern["launches"] + (2 if world > 1 else 0)),
        "e2e": {"value": round(flops_total / (ems * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
                "ms_per_step": round(ems, 4), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak_bf16, "unit": "TFLOP/s",
                     "frac": round(achieved / peak_bf16, 4), "traffic": traffic,
                     "traffic_source": tr.get("source"),
                     "kernel": "attn_fwd2_kernel (tcgen05 kind::f16: bf16 Q.K^T, fp16 P.V)",
                     "kernel_ms": round(kern["ms"], 4), "peak_source": f"{peak_src} bf16 dense (cuBLAS)",
                     "fp8_peak": fp8["burst"],
                     "frac_of_fp8_peak": round(achieved / fp8["burst"], 4) if fp8["burst"] else None,
                     "fp8_peak_source": "measured live: torch._scaled_mm e4m3 8192^3, best of 10",
                     "algorithmic_unit": "4*H*D FLOP per visible (query, key) pair"},
        "cpu_baseline": cpu,
        "clocks": clocks,
        "parity": parity,
        "decoded_cache": decoded,
        "gpus_active": gpus if gpus is not None else 1,
        "config3": config3,
    }
    print(json.dumps(line), flush=True)


def _gpus_active(world, device):
    """Distinct physical GPUs (PCI bus ids) the ranks ran on."""
    import torch.distributed as dist
    bus = torch.cuda.get_device_properties(device).pci_bus_id if hasattr(
        torch.cuda.get_device_properties(device), "pci_bus_id") else device.index
    mine = torch.tensor([int(bus), device.index], dtype=torch.int64, device=device)
    parts = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(parts, mine)
    return len({tuple(x.tolist()) for x in parts})


RING_FRAMES = 21
RING_METRIC = "chunk-causal attn TFLOP/s (config 3: ring SP, 21 x 1560-token frame-causal sequence, FP8 KV blocks)"


def _e4m3_decoded(x):
    """bf16 [L, D] rows -> the bf16 values the ring's e4m3 blocks decode to: per row
    s = absmax / 448 (1 for a zero row), codes = e4m3(x / s) (round to nearest even), value =
    bf16(code * s); the quantise-on-write rule of the KV blocks restated for the check.  It runs
    on the CPU: torch's float -> float8_e4m3fn cast on CUDA breaks some exact rounding ties
    differently from IEEE round-to-nearest-even (about 1 % of rows differ by one code), the CPU
    cast does not."""
    dev = x.device
    xf = x.float().cpu()
    amax = xf.abs().amax(-1, keepdim=True)
    sc = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))
    codes = (xf / sc).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
    return (codes.float() * sc).to(torch.bfloat16).to(dev)


def ring_measurement(args, rank, world, device):
    """Config 3: frame-causal self-attention of 21 frames x 1560 tokens (32,760), 24 heads,
    zig-zag sharded over the ranks; FP8 K/V blocks travel the ring (strong scaling).  Returns
    the measurement as a dict (the same on every rank: times are the max over ranks)."""
    from hy_nomas_b200 import _lib
    from hy_nomas_b200 import ring
    from hy_nomas_b200.flops import attention_flops
    from hy_nomas_b200.synthetic import make_generator, seeded_kv
    import torch.distributed as dist

    L = RING_FRAMES * T
    plan = ring.RingPlan(L, world, "zigzag")
    gen = make_generator(1237, device=device)
    # the same global sequence on every rank (seeded), each rank keeps its shard
    full = [seeded_kv((1, L, H_TOTAL, D), gen, device=device) for _ in range(3)]
    q, k, v = (plan.shard(x, rank).contiguous() for x in full)
    # the sampled heads of the whole sequence, for the parity check
    sampled = {h: (full[0][0, :, h].clone(), _e4m3_decoded(full[1][0, :, h]), _e4m3_decoded(full[2][0, :, h]))
               for h in PARITY_HEADS}
    del full
    torch.cuda.empty_cache()
    flops_total = attention_flops(0, L, 0, H_TOTAL, D, False, T)
    group = None
    sched = args.ring_schedule
    state = ring.ring_plan_state(q, seq_len=L, world=world, rank=rank, tokens_per_frame=T, schedule=sched,
                                 group=group)
    out = torch.empty_like(q)
    stream = torch.cuda.current_stream(device)

    def step(q_, k_, v_):
        return ring.ring_attention(q_, k_, v_, group, seq_len=L, tokens_per_frame=T, out=out, schedule=sched)

    for _ in range(args.warmup):
        step(q, k, v)
    torch.cuda.synchronize(device)
    # parity of this rank's rows (its two zig-zag chunks) for the sampled heads
    step(q, k, v)
    torch.cuda.synchronize(device)
    seg0, pos0, pos1 = plan.positions(rank)
    qpos = torch.cat([pos0 + torch.arange(seg0, device=device),
                      pos1 + torch.arange(plan.length(rank) - seg0, device=device)])
    kframe = torch.arange(L, device=device) // T
    vis = kframe[None, :] <= (qpos // T)[:, None]
    rows = []
    for h, (qh, kh, vh) in sampled.items():
        rows.append(_gate(out[0, :, h], _exact_rows(qh[qpos], kh, vh, vis)))
    parity = _reduce_parity(rows, world, device)
    del sampled, vis
    graph = None if args.no_graph else capture_step(lambda: step(q, k, v), device)
    run_step = (lambda: step(q, k, v)) if graph is None else graph.replay
    for _ in range(args.warmup):
        run_step()
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    sampler = ClockSampler(device.index)
    sampler.start()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    t0.record(stream)
    for _ in range(args.steps):
        run_step()
    t1.record(stream)
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    ms = t0.elapsed_time(t1) / args.steps
    launches_per_step = state.launches
    # attention launches alone (events on the caller's stream after each step's input is ready)
    state.event_log = []
    for _ in range(max(1, args.steps // 2)):
        step(q, k, v)
    torch.cuda.synchronize(device)
    n_timed = max(1, args.steps // 2)
    kern_ms = sum(a.elapsed_time(b) for a, b in state.event_log) / n_timed
    state.event_log = None
    if world > 1:
        tt = torch.tensor([ms, kern_ms], device=device)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms, kern_ms_max = tt.tolist()
    else:
        kern_ms_max = kern_ms
    _lib.check_device_status(device)
    value = flops_total / (ms * 1e-3) / 1e12

    # end to end: pinned host shards in, output shard back, every step
    host_in = [t.cpu().pin_memory() for t in (q, k, v)]

    def ring_call(q_, k_, v_):   # a fresh output per eager call: its read-back overlaps the next
        return (ring.ring_attention(q_, k_, v_, group, seq_len=L, tokens_per_frame=T, schedule=sched),)

    from hy_nomas_b200.graphs import GraphedCall
    rcall = ring_call if args.no_graph else GraphedCall(ring_call, device)
    ems, h2d, d2h = e2e_pipelined(rcall, host_in, device, args.steps, args.warmup, world,
                                  static_outputs=not args.no_graph)
    peak_bf16, _, peak_src = load_peaks()
    local_flops = flops_total / world
    achieved = local_flops / (kern_ms * 1e-3) / 1e12
    del graph, run_step   # graphs holding NCCL calls are released before the process group
    if not args.no_graph:
        rcall.release()
    torch.cuda.synchronize(device)
    ring.release_ring_states()
    if world > 1:
        dist.barrier()
    return {
        "metric": RING_METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world,
        "ms_per_step": round(ms, 4), "scaling": "strong",
        "config": {"workload": "config 3: ring SP, 21 frames x 1560 tokens, frame-causal", "heads": H_TOTAL,
                   "head_dim": D, "seq_len": L, "tokens_per_frame": T, "layout": "zig-zag (2N chunks)",
                   "parallelism": f"ring_sp{world}" if world > 1 else "single",
                   "schedule": (f"{sched}: " + {
                       "allgather": "every e4m3 block pushed to every rank over peer memory, one attention launch",
                       "allgather_overlap": "every e4m3 block pushed to every rank over peer memory on a side "
                                            "stream while the own-block launch runs, then the other ranks' keys "
                                            "in up to two launches merged through the fp32 accumulator",
                       "ring": "neighbour passing over NCCL send/recv, one launch per step"}[sched]),
                   "timed_call": "eager" if args.no_graph else "CUDA graph replay of one ring call",
                   "kv_block": "fp8_e4m3 codes + fp32 per-(token, head) scales, quantised each step",
                   "l2": "inputs larger than L2 (201 MB bf16 per tensor over the job)",
                   "tflop_per_step": round(flops_total / 1e12, 4)},
        "gpu_launches": launches_per_step * args.steps,
        "e2e": {"value": round(flops_total / (ems * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
                "ms_per_step": round(ems, 4), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak_bf16, "unit": "TFLOP/s",
                     "frac": round(achieved / peak_bf16, 4), "traffic": None,
                     "kernel": "attn_fwd2_kernel (tcgen05 kind::f16: bf16 Q.K^T, fp16 P.V)",
                     "kernel_ms_per_step": round(kern_ms, 4), "kernel_ms_max_rank": round(kern_ms_max, 4),
                     "peak_source": f"{peak_src} bf16 dense (cuBLAS)",
                     "algorithmic_unit": "4*H*D FLOP per visible (query, key) pair"},
        "parity": parity,
        "clocks": clocks,
    }


def run_ring(args):
    """Config 3 on its own line (``--workload ring``)."""
    import torch.distributed as dist
    rank, world, local = dist_setup(args.gpus)
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    m = ring_measurement(args, rank, world, device)
    gpus = _gpus_active(world, device) if world > 1 else 1
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return
    line = dict(m)
    line.update({"steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "vs_baseline": None,
                 "dtype": "bf16 Q.K^T / fp16 P.V MMAs, fp32 softmax; e4m3 KV blocks on the ring",
                 "data": "synthetic (seeded N(0,1), 4 outlier channels/head x8)", "cpu_baseline": None,
                 "gpus_active": gpus})
    print(json.dumps(line), flush=True)


SINK, KEEP, PREFILL = 1, 32, 64


def run_rollout(args):
    """Config 5: a 64-frame rollout history kept as first-frame sink + the last 32 frames;
    every step attends one new 1560-token frame (24 heads) to the 33 history frames and
    itself, then appends the frame into the window ring (quantise-on-write).  N > 1, Ulysses:
    each rank holds its heads' window and 1560/N of the frame's tokens.  N > 1, KV-stationary
    (--sp-scheme kv): each rank holds its 1560/N-token slice of every frame for all heads."""
    from hy_nomas_b200 import _lib
    from hy_nomas_b200 import attention as hatt
    from hy_nomas_b200 import parallel_states as ps
    from hy_nomas_b200.flops import attention_flops
    from hy_nomas_b200.synthetic import make_generator, seeded_kv
    from hy_nomas_b200.window import SinkWindowKVCache
    import torch.distributed as dist

    rank, world, local = dist_setup(args.gpus)
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        ps.initialize_sequence_parallel_group()
    os.environ["HYB_ASSUME_FINITE_KV"] = "1"
    scheme = args.sp_scheme if world > 1 else "single"
    if scheme == "auto":
        scheme = "kv" if world >= 4 else "ulysses"
    Hl = H_TOTAL // world if scheme == "ulysses" else H_TOTAL
    Ls = T // world
    Tw = Ls if scheme == "kv" else T      # tokens of each frame in this rank's window
    gen = make_generator(1238 + rank, device=device)
    # each appended frame is decoded once into the window's mirror (--no-decoded-window: every
    # call decodes the whole window, as the reference's dequantize_kv does)
    win = SinkWindowKVCache(1, Hl, Tw, SINK, KEEP, device=device, decoded=not args.no_decoded_window)
    with torch.no_grad():
        for _ in range(PREFILL):   # rollout history (untimed): 64 frames through the ring
            win.append(seeded_kv((1, Tw, Hl, D), gen, device=device), seeded_kv((1, Tw, Hl, D), gen, device=device),
                       assume_finite=True)
    img = [seeded_kv((1, Ls, H_TOTAL, D), gen, device=device) for _ in range(3)]
    txt = [img[0][:, :0] for _ in range(3)]
    Lh = (SINK + KEEP) * T
    flops_total = attention_flops(Lh, T, 0, H_TOTAL, D, True, 0)
    sp_metadata = None
    if world > 1:
        from hy_nomas_b200 import communications as comm
        sp_metadata = comm.prepare_sp_communication(Ls, H_TOTAL, device, ps.nccl_info.sp_group)
    stream = torch.cuda.current_stream(device)
    kvs = None
    if scheme == "kv":
        from hy_nomas_b200.kv_stationary import KVStationaryAttention
        kvs = KVStationaryAttention(None, 1, Ls, H_TOTAL, 0, (SINK + KEEP) * Ls, device)
        # outputs into two caller buffers used alternately (the call's out_img / out_txt), so the
        # end-to-end loop (which reads step i back while step i+1 runs) allocates nothing
        kv_outs = [(torch.empty((1, Ls, H_TOTAL, D), dtype=torch.bfloat16, device=device),
                    torch.empty((1, 0, H_TOTAL, D), dtype=torch.bfloat16, device=device)) for _ in range(2)]
        kv_calls = [0]

    def step(q_img, k_img, v_img, q_txt, k_txt, v_txt):
        with torch.no_grad():
            if kvs is not None:
                oi, ot = kv_outs[kv_calls[0] % 2]
                kv_calls[0] += 1
                return kvs(q_img, k_img, v_img, q_txt, k_txt, v_txt, win, out_img=oi, out_txt=ot)
            return hatt.causal_attention_with_cache_mp(
                (q_img, q_txt), (k_img, k_txt), (v_img, v_txt), win.view(), cache_valid_len=win.valid_len,
                update_cache=True, cache_txt=False, tokens_per_frame=T, seg_ar_attention_backend="b200",
                sp_metadata=sp_metadata, chunk_causal_frames=1)

    for _ in range(args.warmup):
        step(*img, *txt)
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    sampler = ClockSampler(local)
    sampler.start()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(device)
    t0.record(stream)
    for _ in range(args.steps):
        step(*img, *txt)
    t1.record(stream)
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    ms = t0.elapsed_time(t1) / args.steps
    if world > 1:
        tt = torch.tensor([ms], device=device)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = tt.item()
    _lib.check_device_status(device)
    value = flops_total / (ms * 1e-3) / 1e12
    host_in = [t.cpu().pin_memory() for t in (*img, *txt)]
    if kvs is not None:
        kv_calls[0] = 0   # step i of the loop below uses output buffer i % 2, as the loop expects
    ems, h2d, d2h = e2e_pipelined(lambda *x: step(*x), host_in, device, args.steps, args.warmup, world,
                                  static_outputs=kvs is not None)
    if world > 1:
        from hy_nomas_b200 import communications as comm2
        torch.cuda.synchronize(device)
        if kvs is not None:
            kvs.close()
        comm2.release_peer_exchanges()
        ps.destroy_sequence_parallel_group()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC5, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
        "dtype": "bf16 MMA / fp32 softmax; e4m3 KV cache", "data": "synthetic (seeded N(0,1), 4 outlier channels/head x8)",
        "config": {"workload": "config 5: long rollout, 1-frame chunks, sink 1 + window 32 of a 64-frame history",
                   "heads": H_TOTAL, "head_dim": D, "tokens_per_frame": T, "history_tokens": Lh,
                   "visible_keys": Lh + T, "sink_frames": SINK, "window_frames": KEEP, "prefill_frames": PREFILL,
                   "append": "quantise-on-write of each frame into its ring slot (no memmove)"
                             + ("" if args.no_decoded_window else
                                ", then its one-time decode into the window's bf16/fp16 mirror (history read in slot order)"),
                   "parallelism": (f"ulysses_sp{world}" if scheme == "ulysses" else f"kv_stationary_sp{world}")
                   if world > 1 else "single",
                   "l2": "inputs larger than L2 (155 MB FP8 window + 10 MB bf16 frame per step)",
                   "tflop_per_step": round(flops_total / 1e12, 4)},
        "gpu_launches": args.steps * ((8 if scheme == "kv" else 6 + (2 if world > 1 else 0))
                                      + (0 if args.no_decoded_window else 1)),   # + the frame's decode
        "e2e": {"value": round(flops_total / (ems * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
                "ms_per_step": round(ems, 4), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "roofline": None,
        "cpu_baseline": None,
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)


def time_attention_kernel(prob, device, iters):
    """CUDA-event time of the attention kernel launch alone on the staged workspace."""
    from hy_nomas_b200 import _lib
    from hy_nomas_b200 import attention as hatt
    Lh, Li, Ls, Hl = prob["Lh"], prob["Li"], prob["Ls"], prob["Hl"]
    gen = torch.Generator(device=device)
    gen.manual_seed(99)
    from hy_nomas_b200.synthetic import seeded_kv
    img = [seeded_kv((1, Li, Hl, D), gen, device=device) for _ in range(3)]
    txt = [seeded_kv((1, TXT, Hl, D), gen, device=device) for _ in range(3)]
    ws = hatt.Workspace()
    hatt.cached_attention_local(*img, *txt, prob["cache"], Lh, group_tokens=T, workspace=ws)
    args = ws.attn_args
    lib = _lib.load()
    stream = torch.cuda.current_stream(device)
    for _ in range(3):
        _lib.check(lib.hyb_attn_fwd(args, stream.cuda_stream), "attention")
    torch.cuda.synchronize(device)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(iters):
        _lib.check(lib.hyb_attn_fwd(args, stream.cuda_stream), "attention")
    e1.record(stream)
    torch.cuda.synchronize(device)
    import ctypes
    ks = (ctypes.c_int32 * 4096)()
    npairs = lib.hyb_attn_work_plan(ctypes.byref(args), 0, ks, 4096)
    merge = npairs > 0 and max(ks[:npairs]) > 1
    return {"ms": e0.elapsed_time(e1) / iters, "launches": 2 if merge else 1}


def cpu_problem(heads, seed=1236):
    from hy_nomas_b200.synthetic import make_generator, seeded_kv
    from oracle import quant as oq
    gen = make_generator(seed)
    Lh, Li = HIST_FRAMES * T, CHUNK_FRAMES * T
    hk = seeded_kv((1, Lh, heads, D), gen)
    hv = seeded_kv((1, Lh, heads, D), gen)
    ck, sk = oq.quantize_e4m3(hk)
    cv, sv = oq.quantize_e4m3(hv)
    cur = [seeded_kv((1, L, heads, D), gen) for L in (Li, TXT) for _ in range(3)]
    return dict(ck=ck, sk=sk, cv=cv, sv=sv, cur=cur, Lh=Lh, Li=Li)


def cpu_step(p):
    """The reference CPU path for one chunk: decode history, quantise-on-write the chunk,
    compose and run SDPA with the frame-causal mask (oracle restatement)."""
    from oracle import attention as oatt
    from oracle import quant as oq
    hk = oq.dequantize(p["ck"], p["sk"])
    hv = oq.dequantize(p["cv"], p["sv"])
    cur = p["cur"]
    oq.quantize_e4m3(torch.cat([cur[1], cur[4]], 1))
    oq.quantize_e4m3(torch.cat([cur[2], cur[5]], 1))
    return oatt.reference_sdpa_path(*cur, hk, hv, group_tokens=T)


def cpu_baseline(heads, reps=2):
    from hy_nomas_b200.flops import attention_flops
    torch.set_num_threads(os.cpu_count() or 1)
    p = cpu_problem(heads)
    cpu_step(p)
    t = time.perf_counter()
    for _ in range(reps):
        cpu_step(p)
    dt = (time.perf_counter() - t) / reps
    fl = attention_flops(p["Lh"], p["Li"], TXT, heads, D, True, T)
    return {"value": round(fl / dt / 1e12, 4), "unit": "TFLOP/s", "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"config 2 with {heads} of {H_TOTAL} heads per step (decode + append + SDPA), "
                      f"{reps} reps, {dt:.2f} s per step"}


def reference_problem(heads, seed=1236):
    """Config 2 for the reference's own function: the history quantised into an INT8 cache by
    the reference quantiser (int8_kv_cache.py:161-179), the chunk's Q/K/V in bf16."""
    import importlib
    from hy_nomas_b200.synthetic import make_generator, seeded_kv
    i8 = importlib.import_module("hymm.models.dit.modules.int8_kv_cache")
    gen = make_generator(seed)
    Lh, Li = HIST_FRAMES * T, CHUNK_FRAMES * T
    cap = Lh + Li + TXT
    cache = i8.make_int8_kv_block(1, cap, heads, D, device="cpu")
    i8.quantize_kv_pair_into(cache, seeded_kv((1, Lh, heads, D), gen), seeded_kv((1, Lh, heads, D), gen), 0)
    cur = [seeded_kv((1, L, heads, D), gen) for L in (Li, TXT) for _ in range(3)]
    return dict(cache=cache, cur=cur, Lh=Lh, Li=Li)


def reference_step(native, p):
    """One config-2 chunk through the reference's causal_attention_with_cache_mp (torch mode,
    nomas_cpt.py:335-884): one call per query frame, frame f attending the history, the
    chunk's earlier frames (written into the INT8 cache by the previous call's update_cache)
    and itself, which is the frame-level block-causal rule."""
    cache = {k: (t.clone() if isinstance(t, torch.Tensor) else t) for k, t in p["cache"].items()}
    iq, ik, iv, tq, tk, tv = p["cur"]
    with torch.no_grad():
        for f in range(CHUNK_FRAMES):
            sl = slice(f * T, (f + 1) * T)
            native.causal_attention_with_cache_mp(
                (iq[:, sl], tq), (ik[:, sl], tk), (iv[:, sl], tv), cache, cache_valid_len=p["Lh"] + f * T,
                attn_mode="torch", text_mask=None, update_cache=True, cache_txt=False, cache_mask=None)


def run_reference(args):
    """The reference arm: the reference's own CPU implementation of the path on the host cores.
    Where HY_NOMAS_REF names a reference checkout, its causal_attention_with_cache_mp itself
    (kind "reference"); elsewhere (the GPU boxes carry no checkout) the oracle restatement of
    the same path (kind "port")."""
    if args.gpus > 1:
        rank = int(os.environ.get("RANK", "0"))
        if rank != 0:
            return
    from hy_nomas_b200.flops import attention_flops
    from oracle import reference as oref
    torch.set_num_threads(os.cpu_count() or 1)
    heads = args.cpu_heads
    if oref.checkout() is not None:
        import importlib
        oref.install_stub()
        native = importlib.import_module("hymm.models.dit.nomas_cpt")
        p = reference_problem(heads)
        kind = "reference"
        sample = (f"config 2 with {heads} of {H_TOTAL} heads per step: causal_attention_with_cache_mp "
                  f"(attn_mode='torch', INT8 cache, update_cache per frame), one call per query frame")
        step = lambda: reference_step(native, p)  # noqa: E731
    else:
        p = cpu_problem(heads)
        kind = "port"
        sample = f"config 2 with {heads} of {H_TOTAL} heads per step (decode + append + SDPA)"
        step = lambda: cpu_step(p)  # noqa: E731
    for _ in range(args.warmup):
        step()
    t = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t) / args.steps
    fl = attention_flops(p["Lh"], p["Li"], TXT, heads, D, True, T)
    value = fl / dt / 1e12
    line = {
        "metric": METRIC, "value": round(value, 4), "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16 (CPU SDPA)",
        "data": "synthetic (seeded N(0,1), 4 outlier channels/head x8)", "impl": "reference",
        "config": {"workload": "config 2: 1x B200 single block", "heads_sampled": heads,
                   "history_tokens": p["Lh"], "chunk_image_tokens": p["Li"], "tokens_per_frame": T},
        "cpu_baseline": {"value": round(value, 4), "unit": "TFLOP/s", "cores": torch.get_num_threads(),
                         "kind": kind, "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def library_comparison(steps):
    """Config-2 shapes (24 heads x 128, 6,241 queries against 31,201 keys), every key visible
    (chunk-bidirectional: a frame-causal mask is not expressible in the library call), bf16
    Q/K/V resident in HBM: device time of this library's attention launch (hyb_attn_fwd on the
    staged operands) and of flashinfer's CUTLASS sm100a FMHA (fmha_varlen), the Blackwell
    library kernel closest to the incumbent FA4 / MagiAttention kernels (not installed here).
    A comparison column only: the library kernel is never on this repository's path."""
    import flashinfer
    from hy_nomas_b200 import _lib
    from hy_nomas_b200 import attention as hatt
    from hy_nomas_b200.synthetic import make_generator, seeded_kv
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    H, Lh, Li, Lt = H_TOTAL, HIST_FRAMES * T, CHUNK_FRAMES * T, TXT
    gen = make_generator(77, device=dev)
    hist = {"k": seeded_kv((1, Lh, H, D), gen, device=dev), "v": seeded_kv((1, Lh, H, D), gen, device=dev)}
    cur = [seeded_kv((1, L, H, D), gen, device=dev) for L in (Li, Lt) for _ in range(3)]
    ws = hatt.Workspace()
    hatt.cached_attention_local(*cur, hist, Lh, group_tokens=0, workspace=ws)
    lib = _lib.load()
    args = ws.attn_args
    stream = torch.cuda.current_stream(dev)

    def ours():
        _lib.check(lib.hyb_attn_fwd(args, stream.cuda_stream), "attention")

    q = torch.cat([cur[0], cur[3]], 1)[0].contiguous()                      # [Lq, H, D]
    k = torch.cat([hist["k"], cur[1], cur[4]], 1)[0].contiguous()           # [Lk, H, D]
    v = torch.cat([hist["v"], cur[2], cur[5]], 1)[0].contiguous()
    qo = torch.tensor([0, q.shape[0]], dtype=torch.int32, device=dev)
    kvo = torch.tensor([0, k.shape[0]], dtype=torch.int32, device=dev)
    out = torch.empty_like(q)

    def theirs():
        flashinfer.prefill.fmha_varlen(q, k, v, qo, kvo, out=out, causal=False, sm_scale=D ** -0.5)

    def timed(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / steps

    from hy_nomas_b200.flops import attention_flops
    fl = attention_flops(Lh, Li, Lt, H, D, True, 0)
    ms_ours, ms_lib = timed(ours), timed(theirs)
    o_ours = ws.keep[0]
    ref_rows = out[:Li].float()
    agree = (o_ours[0].float() - ref_rows).abs().max().item()
    return {"workload": "config-2 shapes, chunk-bidirectional, bf16 Q/K/V resident", "tflop": round(fl / 1e12, 4),
            "this_kernel": {"ms": round(ms_ours, 4), "tflops": round(fl / ms_ours / 1e9, 1),
                            "kernel": "attn_fwd2_kernel (bf16 Q.K^T, fp16 P.V; operands staged by the call)"},
            "flashinfer_fmha_varlen": {"ms": round(ms_lib, 4), "tflops": round(fl / ms_lib / 1e9, 1),
                                       "version": flashinfer.__version__,
                                       "kernel": "CUTLASS sm100a FMHA (bf16, non-causal)"},
            "max_abs_difference_image_rows": round(agree, 5)}


def main():
    args = parse()
    if args.library_comparison:
        print(json.dumps(library_comparison(max(args.steps, 10))), flush=True)
        return
    if args.measure_fp8_peak:
        print(json.dumps({"fp8_e4m3_gemm_tflops": measure_fp8_peak(torch.device("cuda", 0), sustained_s=4.0),
                          "how": "torch._scaled_mm e4m3 8192^3, best of 10 (burst) and back to back for 4 s"}))
        return
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "ring":
        run_ring(args)
    elif args.workload == "rollout":
        run_rollout(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
