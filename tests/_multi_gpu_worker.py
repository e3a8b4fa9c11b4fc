"""Worker for test_gpu_multi.py (launched with torch.distributed.run, one rank per GPU).

Runs the drop-in with Ulysses sequence parallelism over all ranks and checks, on rank 0, that
the gathered result (and the head-sharded cache writes) equal a single-GPU call on the whole
problem; then the ring schedules and the KV-stationary schedule against their one-process
emulations.  Prints "MULTI_GPU_OK" on success."""
import datetime
import os
import sys

import torch
import torch.distributed as dist

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, REPO)

from hy_nomas_b200 import attention as hatt          # noqa: E402
from hy_nomas_b200 import kv_cache as kvc            # noqa: E402
from hy_nomas_b200 import parallel_states as ps      # noqa: E402
from hy_nomas_b200.synthetic import make_generator, seeded_kv  # noqa: E402


def main():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    H, D, T, frames, Lh, Lt = 8, 128, 64, 4, 512, 2
    Li = T * frames
    assert H % world == 0 and Li % world == 0
    gen = make_generator(4242)
    hk, hv = seeded_kv((1, Lh, H, D), gen), seeded_kv((1, Lh, H, D), gen)
    img = [seeded_kv((1, Li, H, D), gen) for _ in range(3)]
    txt = [seeded_kv((1, Lt, H, D), gen) for _ in range(3)]
    tmask = torch.tensor([[True, False]], device=dev)
    cap = Lh + Li + Lt + 8

    def make_cache(heads):
        c = kvc.make_fp8_kv_block(1, cap, len(heads), D, device=dev)
        with torch.no_grad():
            kvc.quantize_kv_pair_into(c, hk[:, :, heads].to(dev).contiguous(),
                                      hv[:, :, heads].to(dev).contiguous(), 0)
        m = torch.zeros(1, cap, dtype=torch.bool, device=dev)
        m[:, :Lh] = True
        m[:, 100:130] = False
        return c, m

    # ---- Ulysses SP over all ranks
    ps.initialize_sequence_parallel_group()
    hl = list(range(rank * H // world, (rank + 1) * H // world))
    cache, mask = make_cache(hl)
    Ls = Li // world
    sl = slice(rank * Ls, (rank + 1) * Ls)
    with torch.no_grad():
        out_img, out_txt = hatt.causal_attention_with_cache_mp(
            (img[0][:, sl].to(dev), txt[0].to(dev)), (img[1][:, sl].to(dev), txt[1].to(dev)),
            (img[2][:, sl].to(dev), txt[2].to(dev)), cache, cache_valid_len=Lh, attn_mode="flash3",
            text_mask=tmask, update_cache=True, cache_txt=True, cache_mask=mask, tokens_per_frame=T,
            seg_ar_attention_backend="b200", chunk_causal_frames=1)
    # the same call over NCCL collectives (HYB_PEER_EXCHANGE=0) gives the same bytes; the cache
    # write is repeated with identical values
    from hy_nomas_b200 import communications as comm
    os.environ["HYB_PEER_EXCHANGE"] = "0"
    with torch.no_grad():
        nccl_img, nccl_txt = hatt.causal_attention_with_cache_mp(
            (img[0][:, sl].to(dev), txt[0].to(dev)), (img[1][:, sl].to(dev), txt[1].to(dev)),
            (img[2][:, sl].to(dev), txt[2].to(dev)), cache, cache_valid_len=Lh, attn_mode="flash3",
            text_mask=tmask, update_cache=True, cache_txt=True, cache_mask=mask, tokens_per_frame=T,
            seg_ar_attention_backend="b200", chunk_causal_frames=1)
    os.environ.pop("HYB_PEER_EXCHANGE", None)
    peer_ok = torch.equal(nccl_img, out_img) and torch.equal(nccl_txt, out_txt)
    if not peer_ok:
        print("peer exchange differs from NCCL on rank", rank)
    gathered = [torch.empty_like(out_img) for _ in range(world)]
    dist.all_gather(gathered, out_img.contiguous())
    codes = [torch.empty_like(cache["k"]) for _ in range(world)]
    dist.all_gather(codes, cache["k"].contiguous())
    ok = peer_ok
    if rank == 0:
        ps.set_sequence_parallel_state(False)
        full_cache, full_mask = make_cache(list(range(H)))
        with torch.no_grad():
            ref_img, ref_txt = hatt.causal_attention_with_cache_mp(
                tuple(t.to(dev) for t in (img[0], txt[0])), tuple(t.to(dev) for t in (img[1], txt[1])),
                tuple(t.to(dev) for t in (img[2], txt[2])), full_cache, cache_valid_len=Lh,
                attn_mode="flash3", text_mask=tmask, update_cache=True, cache_txt=True,
                cache_mask=full_mask, tokens_per_frame=T, seg_ar_attention_backend="b200",
                chunk_causal_frames=1)
        sp_img = torch.cat(gathered, dim=1)
        if not torch.equal(sp_img, ref_img):
            print("image mismatch", (sp_img.float() - ref_img.float()).abs().max().item())
            ok = False
        if not torch.equal(out_txt, ref_txt):
            print("text mismatch", (out_txt.float() - ref_txt.float()).abs().max().item())
            ok = False
        sp_codes = torch.cat(codes, dim=2)
        if not torch.equal(sp_codes[:, :Lh + Li + Lt].view(torch.uint8),
                           full_cache["k"][:, :Lh + Li + Lt].view(torch.uint8)):
            print("cache write mismatch")
            ok = False
        if not torch.equal(mask, full_mask):
            print("cache mask mismatch")
            ok = False
    # ---- ring (KV passing) over all ranks: equals the emulated single-process schedule
    from hy_nomas_b200 import ring
    Lr, Tr = 8 * 96 + 5, 96
    # two inputs, called back to back with no host synchronisation between the calls: the
    # second call's block push must wait (entry barrier) for every peer's decode of the first
    inputs = [tuple(seeded_kv((1, Lr, 4, D), make_generator(77 + 10 * c + i)).to(dev) for i in range(3))
              for c in range(2)]
    for schedule, layout in (("ring", "zigzag"), ("ring", "contiguous"), ("allgather", "zigzag"),
                             ("allgather", "contiguous"), ("allgather_overlap", "zigzag"),
                             ("allgather_overlap", "contiguous")):
        plan = ring.RingPlan(Lr, world, layout)
        emus = [ring.ring_attention_emulated(*x, world, tokens_per_frame=Tr, layout=layout, schedule=schedule)
                for x in inputs]
        outs = []
        for rep in range(2):   # the second round reuses the cached plan and buffers
            for rq, rk, rv in inputs:
                outs.append(ring.ring_attention(plan.shard(rq, rank).contiguous(), plan.shard(rk, rank).contiguous(),
                                                plan.shard(rv, rank).contiguous(), None, seq_len=Lr,
                                                tokens_per_frame=Tr, layout=layout, schedule=schedule))
        for i, out_ring in enumerate(outs):
            want = plan.shard(emus[i % 2], rank)
            if not torch.equal(out_ring, want):
                print("ring mismatch on rank", rank, schedule, layout, "call", i,
                      (out_ring.float() - want.float()).abs().max().item())
                ok = False
    ring.release_ring_states()
    # ---- KV-stationary schedule (Q all-gather, partial rows scattered by the attention epilogue
    # to their owners over peer memory) over all ranks: equals the emulated single-process
    # schedule bit for bit, over a rollout that wraps the window
    from hy_nomas_b200.kv_stationary import KVStationaryAttention, kv_stationary_emulated
    from hy_nomas_b200.window import SinkWindowKVCache
    Hk, Ltk = 4, 1
    Lsk = 96
    Tk = Lsk * world
    kvs = KVStationaryAttention(None, 1, Lsk, Hk, Ltk, 3 * Lsk, dev)
    sl2 = slice(rank * Lsk, (rank + 1) * Lsk)
    for decoded in (False, True):   # windows decoding per call / keeping their history decoded
        win = SinkWindowKVCache(1, Hk, Lsk, 1, 2, device=dev, decoded=decoded)
        wins = [SinkWindowKVCache(1, Hk, Lsk, 1, 2, device=dev, decoded=decoded) for _ in range(world)]
        gk = make_generator(515)
        for step in range(4):
            fq, fk, fv = (seeded_kv((1, Tk, Hk, D), gk).to(dev) for _ in range(3))
            tq2, tk2, tv2 = (seeded_kv((1, Ltk, Hk, D), gk).to(dev) for _ in range(3))
            with torch.no_grad():
                o_img, o_txt = kvs(fq[:, sl2], fk[:, sl2], fv[:, sl2], tq2, tk2, tv2, win)
                e_img, e_txt = kv_stationary_emulated(fq, fk, fv, tq2, tk2, tv2, wins, slices=kvs.slices)
            if not (torch.equal(o_img, e_img[:, sl2]) and torch.equal(o_txt, e_txt)):
                print("KV-stationary mismatch on rank", rank, "step", step, "decoded", decoded,
                      (o_img.float() - e_img[:, sl2].float()).abs().max().item())
                ok = False
    kvs.close()
    ok_t = torch.tensor([1 if ok else 0], device=dev)
    dist.all_reduce(ok_t, op=dist.ReduceOp.MIN)
    ok = bool(ok_t.item())
    flag = torch.tensor([1 if ok else 0], device=dev)
    dist.broadcast(flag, 0)
    comm.release_peer_exchanges()
    ps.destroy_sequence_parallel_group()
    dist.destroy_process_group()
    if rank == 0 and flag.item() == 1:
        print("MULTI_GPU_OK")


if __name__ == "__main__":
    main()
