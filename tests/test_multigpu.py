"""Two-GPU partitioning on real devices (NCCL): query-block shards, head
shards, the frame all-gather and the sequence-parallel (frame-sharded) layer
reproduce the single-GPU layer exactly.
Skipped unless at least two GPUs are visible."""
import datetime
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_q):
    import torch.distributed as dist
    # one CTA per work item, so shard and full layer sum in the same order
    os.environ["VGGT_ATTN_SPLIT"] = "1"
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    try:
        import vggt_sparse
        from vggt_sparse import distributed as vd
        from vggt_sparse.synthetic import clustered_layer
        dev = torch.device("cuda", rank)
        x = clustered_layer(4, centres=64, seed=2, device=dev)
        kw = dict(mode="topk", retention=0.25, dense_heads=(0, 5))
        ref = vggt_sparse.SparseGlobalLayer(16, **kw)
        ref.topk = vggt_sparse.topk_budget(0.25, x.shape.n_tokens, x.shape.n_special,
                                           x.shape.n_blocks, 64)
        full = ref(x.q, x.kp, x.vp, x.ks, x.vs)
        ok = {}
        # query-block shards
        qs = vd.QBlockShardedLayer(16, world, rank, **kw)
        rows_out, (r0, r1) = qs(x.q, x.kp, x.vp, x.ks, x.vs)
        ok["qblocks"] = bool(torch.equal(rows_out, full[:, r0:r1]))
        # head shards
        hs = vd.HeadShardedLayer(16, world, rank, dense_heads=(0, 5), mode="topk",
                                 retention=0.25)
        h_out, heads = hs(x.q, x.kp, x.vp, x.ks, x.vs)
        ok["heads"] = bool(torch.equal(h_out, full[heads]))
        # frame-sharded K/V all-gather over NCCL
        f0, f1 = vd.frame_range(4, world, rank)
        ppf = 37 * 37
        kp_full = vd.allgather_frames(x.kp[:, f0 * ppf:f1 * ppf].contiguous(), world)
        ok["allgather"] = bool(torch.equal(kp_full, x.kp))
        # sequence-parallel layer: this rank's query rows and its own frames'
        # K/V in, NCCL all-gathers of K/V inside the call (keys first)
        fs = vd.FrameShardedLayer(16, world, rank, 4, **kw)
        s0, s1 = fs.rows(x.shape.n_tokens)
        spf = 5
        shards = [t[:, f0 * ppf:f1 * ppf].contiguous() for t in (x.kp, x.vp)] + \
                 [t[:, f0 * spf:f1 * spf].contiguous() for t in (x.ks, x.vs)]
        fs_out = fs(x.q[:, s0:s1].contiguous(), *shards)
        ok["frames"] = bool(torch.equal(fs_out, full[:, s0:s1]))
        # the other schedule: one layer per head group (dense heads first)
        fsg = vd.FrameShardedLayer(16, world, rank, 4, schedule="groups", **kw)
        out_g = fsg(x.q[:, s0:s1].contiguous(), *shards)
        ok["frames_groups"] = bool(torch.equal(out_g, full[:, s0:s1]))
        # bulk gathers (one all-gather per tensor, then a copy into place)
        # with both schedules; the groups need consecutive heads
        kwc = dict(mode="topk", retention=0.25, dense_heads=(0, 1))
        refc = vggt_sparse.SparseGlobalLayer(16, **kwc)
        refc.topk = ref.topk
        fullc = refc(x.q, x.kp, x.vp, x.ks, x.vs)
        for sched in ("kfirst", "groups"):
            fsb = vd.FrameShardedLayer(16, world, rank, 4, schedule=sched, gather="bulk", **kwc)
            out_b = fsb(x.q[:, s0:s1].contiguous(), *shards)
            ok["frames_bulk_" + sched] = bool(torch.equal(out_b, fullc[:, s0:s1]))
        # the exchange over NVLink peer memory (two calls: two epochs)
        fsp = vd.FrameShardedLayer(16, world, rank, 4, gather="push", **kwc)
        for i in range(2):
            out_p = fsp(x.q[:, s0:s1].contiguous(), *shards)
            ok["frames_push_%d" % i] = bool(torch.equal(out_p, fullc[:, s0:s1]))
        fsp.check_status()
        torch.cuda.synchronize()
        result_q.put((rank, ok))
    except Exception as e:  # report instead of leaving the peer waiting
        result_q.put((rank, {"error": repr(e)}))
    finally:
        dist.destroy_process_group()


def test_two_gpu_shards_match_single_gpu_layer():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    for rank, ok in results.items():
        assert ok == {"qblocks": True, "heads": True, "allgather": True, "frames": True,
                      "frames_groups": True, "frames_bulk_kfirst": True,
                      "frames_bulk_groups": True, "frames_push_0": True,
                      "frames_push_1": True}, \
            (rank, ok)


def _push_worker(rank, world, port, result_q):
    import torch.distributed as dist
    os.environ["VGGT_ATTN_SPLIT"] = "1"
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    try:
        import vggt_sparse
        from vggt_sparse import distributed as vd
        from vggt_sparse.synthetic import clustered_layer
        dev = torch.device("cuda", rank)
        x = clustered_layer(4, centres=64, seed=3, device=dev)
        kw = dict(mode="mass", tau=0.9, dense_heads=(0, 1))
        full = vggt_sparse.SparseGlobalLayer(16, **kw)(x.q, x.kp, x.vp, x.ks, x.vs)
        fs = vd.FrameShardedLayer(16, world, rank, 4, gather="push", **kw)
        s0, s1 = fs.rows(x.shape.n_tokens)
        f0, f1 = vd.frame_range(4, world, rank)
        ppf, spf = 37 * 37, 5
        shards = [t[:, f0 * ppf:f1 * ppf].contiguous() for t in (x.kp, x.vp)] + \
                 [t[:, f0 * spf:f1 * spf].contiguous() for t in (x.ks, x.vs)]
        ok = {}
        for i in range(3):
            out = fs(x.q[:, s0:s1].contiguous(), *shards)
            ok[i] = bool(torch.equal(out, full[:, s0:s1]))
        kp_full = fs._buffers(shards[0], shards[2])[0]
        ok["kp"] = bool(torch.equal(kp_full, x.kp))
        fs.check_status()
        torch.cuda.synchronize()
        result_q.put((rank, ok))
    except Exception as e:  # report instead of leaving the peer waiting
        result_q.put((rank, {"error": repr(e)}))
    finally:
        dist.destroy_process_group()


def test_push_exchange_on_one_gpu():
    """The peer-memory exchange with a single rank (its own buffers only):
    the layer equals the single-GPU layer on three calls in a row."""
    if torch.cuda.device_count() < 1:
        pytest.skip("needs a GPU")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_push_worker, args=(0, 1, _free_port(), q))
    p.start()
    rank, ok = q.get(timeout=300)
    p.join(timeout=60)
    assert ok == {0: True, 1: True, 2: True, "kp": True}, ok
