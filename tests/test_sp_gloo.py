"""Ulysses sequence-parallel host logic on 2 CPU ranks (gloo): metadata exchange, the
collective step with the reference's buffer layouts, the head all-gather, and failure
detection when a rank dies before a collective.  The CUDA pack/unpack kernels are tested on
one GPU in test_gpu_comm.py; here the send buffers are built by the oracle layouts."""
import os
import tempfile
import time
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import GOLDEN, REPO


def _init(rank, world, init_file, timeout_s=60):
    import datetime
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _worker_layouts(rank, world, init_file, result_dir):
    import sys
    sys.path.insert(0, str(REPO))
    sys.path.insert(0, str(REPO / "tests"))
    status = "ok"
    try:
        import numpy as np
        from conftest import bf16, load_golden
        from hy_nomas_b200 import communications as comm
        from oracle import sp as osp
        _init(rank, world, init_file)
        g = load_golden(f"sp_rank{rank}.npz")
        for case in ("even", "uneven"):
            lens = tuple(int(x) for x in g[f"{case}_lens"])
            q, k, v = (bf16(g[f"{case}_{n}"]) for n in "qkv")
            meta = comm.prepare_sp_communication(q.shape[1], q.shape[2], "cpu", None)
            assert meta.sequence_lengths == lens and meta.head_sizes == (2, 2)
            send = osp.pack_seq_to_heads([q, k, v], world, max(lens))
            recv = comm.exchange(send, None)
            outs = osp.unpack_seq_to_heads(recv, lens, 3)
            for name, t in zip(("oq", "ok", "ov"), outs):
                assert torch.equal(t.view(torch.int16), torch.from_numpy(g[f"{case}_{name}"])), name
            send_o = osp.pack_heads_to_seq(bf16(g[f"{case}_o_in"]), lens)
            out_o = osp.unpack_heads_to_seq(comm.exchange(send_o, None), lens[rank])
            assert torch.equal(out_o.view(torch.int16), torch.from_numpy(g[f"{case}_o_out"]))
            t_out = comm.all_gather(bf16(g[f"{case}_t_in"]), dim=2, group=None, sizes=meta.head_sizes)
            assert torch.equal(t_out.view(torch.int16), torch.from_numpy(g[f"{case}_t_out"]))
        # metadata validation errors are raised on every rank, with the reference's message
        try:
            comm.prepare_sp_communication(4, 3, "cpu", None)
            status = "no error for 3 heads on 2 ranks"
        except ValueError as e:
            assert "divisible" in str(e)
        dist.destroy_process_group()
    except Exception:
        status = traceback.format_exc()
    with open(os.path.join(result_dir, f"r{rank}"), "w") as f:
        f.write(status)


def _worker_dead_peer(rank, world, init_file, result_dir):
    import sys
    sys.path.insert(0, str(REPO))
    status = "ok"
    try:
        from hy_nomas_b200 import communications as comm
        _init(rank, world, init_file, timeout_s=5)
        if rank == 1:
            # this rank fails between steps: it leaves before the next collective
            dist.destroy_process_group()
            os._exit(0)
        send = torch.zeros(world, 4, 2, 1, 128, dtype=torch.bfloat16)
        t0 = time.time()
        try:
            comm.exchange(send, None)
            status = "collective with a dead peer returned"
        except Exception as e:  # gloo reports the closed peer / timeout as an error
            elapsed = time.time() - t0
            status = "ok" if elapsed < 60 else f"error only after {elapsed:.0f}s: {e}"
    except Exception:
        status = traceback.format_exc()
    with open(os.path.join(result_dir, f"r{rank}"), "w") as f:
        f.write(status)


def _run(worker, world=2):
    ctx = mp.get_context("spawn")
    with tempfile.TemporaryDirectory() as d:
        init_file = os.path.join(d, "init")
        procs = [ctx.Process(target=worker, args=(r, world, init_file, d)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=180)
            if p.is_alive():
                p.kill()
        results = {}
        for r in range(world):
            path = os.path.join(d, f"r{r}")
            results[r] = open(path).read() if os.path.exists(path) else "no result"
    return results


def test_ulysses_layouts_over_gloo_match_reference():
    res = _run(_worker_layouts)
    assert res == {0: "ok", 1: "ok"}, res


def test_dead_peer_is_reported_not_hung():
    res = _run(_worker_dead_peer)
    assert res[0] == "ok", res[0]


def _worker_size_agreement(rank, world, init_file, result_dir):
    import sys
    sys.path.insert(0, str(REPO))
    status = "ok"
    try:
        from hy_nomas_b200 import communications as comm
        _init(rank, world, init_file)
        # the same sizes on every rank pass
        comm.require_same_on_every_rank(None, [4096, 4096, 256, 1, 780, 24, 1], "peer buffers")
        # one rank with another geometry: every rank raises before any buffer exists
        mine = [4096, 256, 780 if rank == 0 else 781]
        try:
            comm.require_same_on_every_rank(None, mine, "peer buffers")
            status = "no error for disagreeing sizes"
        except ValueError as e:
            assert "disagree" in str(e), str(e)
        # a different number of sizes is caught as well, without a mismatched collective
        try:
            comm.require_same_on_every_rank(None, [1, 2, 3][:2 + rank], "peer buffers")
            status = "no error for a different count"
        except ValueError as e:
            assert "number of sizes" in str(e), str(e)
        dist.destroy_process_group()
    except Exception:
        status = traceback.format_exc()
    with open(os.path.join(result_dir, f"r{rank}"), "w") as f:
        f.write(status)


def test_peer_buffer_sizes_are_checked_on_every_rank():
    """Peer buffers are sized from each rank's own geometry; ranks that disagree raise
    ValueError on every rank before anything is allocated (a write past a peer's buffer would
    be a device fault)."""
    res = _run(_worker_size_agreement)
    assert res == {0: "ok", 1: "ok"}, res


def _worker_kv_stationary(rank, world, init_file, result_dir):
    import sys
    sys.path.insert(0, str(REPO))
    status = "ok"
    try:
        from oracle import sp as osp
        from oracle import attention as oatt
        _init(rank, world, init_file)
        g = torch.Generator().manual_seed(99)
        B, H, D, Ls, Lt, frames = 1, 2, 128, 24, 1, 3
        T = Ls * world
        q, k, v = (torch.randn(B, T, H, D, generator=g).to(torch.bfloat16) for _ in range(3))
        tq, tk, tv = (torch.randn(B, Lt, H, D, generator=g).to(torch.bfloat16) for _ in range(3))
        hk, hv = (torch.randn(B, frames * T, H, D, generator=g).to(torch.bfloat16) for _ in range(2))
        # this rank's slice of every history frame and of the current frame
        mine = torch.cat([torch.arange(f * T + rank * Ls, f * T + (rank + 1) * Ls) for f in range(frames)])
        sl = slice(rank * Ls, (rank + 1) * Ls)
        o_img, o_txt = osp.kv_stationary_step(q[:, sl], k[:, sl], v[:, sl], tq, tk, tv, hk[:, mine], hv[:, mine])
        ref_img, ref_txt = oatt.cached_attention(q, k, v, tq, tk, tv, hk, hv, attend_txt=True)
        err = max((o_img - ref_img[:, sl].double()).abs().max().item(), (o_txt - ref_txt.double()).abs().max().item())
        assert err < 1e-4, err
        dist.destroy_process_group()
    except Exception:
        status = traceback.format_exc()
    with open(os.path.join(result_dir, f"r{rank}"), "w") as f:
        f.write(status)


def test_kv_stationary_protocol_over_gloo():
    """The KV-stationary schedule's protocol on 2 CPU ranks: Q all-gathered, every rank's
    partial over its own slice of every frame (text keys on rank 0 only), each owner merging its
    rows and every rank the text rows, equals attention over the whole history."""
    res = _run(_worker_kv_stationary)
    assert res == {0: "ok", 1: "ok"}, res
