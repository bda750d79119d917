"""Partitioning host logic on CPU: shard ranges, head balancing, the frame
all-gather and the head-wise gathers of FrameShardedLayer (world 2, gloo), and
that per-rank query-block shards of the oracle layer reassemble the full-layer
result."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from vggt_sparse import distributed as vd


def test_qblock_ranges_cover_every_block_once():
    for n, w in ((687, 8), (86, 2), (5496, 8), (3, 4)):
        seen = []
        for r in range(w):
            b0, b1 = vd.qblock_range(n, w, r)
            assert 0 <= b0 <= b1 <= n
            seen.extend(range(b0, b1))
        assert seen == list(range(n))


def test_head_assignment_balances_dense_heads():
    a = vd.head_assignment(16, 8, dense_heads=(0, 1, 2, 3), sparse_cost=0.3)
    assert sorted(sum(a, [])) == list(range(16))
    dense_per_rank = [sum(h < 4 for h in x) for x in a]
    assert max(dense_per_rank) == 1
    load = [sum(1.0 if h < 4 else 0.3 for h in x) for x in a]
    assert max(load) - min(load) <= 1.0
    assert [len(x) for x in vd.head_assignment(16, 8)] == [2] * 8
    b = vd.head_assignment(16, 4)
    assert [len(x) for x in b] == [4, 4, 4, 4]


def test_frame_ranges():
    assert [vd.frame_range(256, 8, r) for r in range(8)] == [(32 * r, 32 * r + 32) for r in range(8)]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        _work(rank, world, result_q)
    except Exception as e:  # report instead of leaving the peer waiting
        result_q.put((False, repr(e)))
    finally:
        dist.destroy_process_group()


def _work(rank, world, result_q):
    import oracle
    from vggt_sparse.synthetic import clustered_layer
    x = clustered_layer(4, centres=16, heads=2, dim=32, patch_h=6, patch_w=6, seed=3,
                        dtype=torch.float32)
    per_frame_patch = 36
    # frame-sharded K/V -> all-gather -> the full patch keys in frame-major order
    f0, f1 = vd.frame_range(4, world, rank)
    kp_local = x.kp[:, f0 * per_frame_patch:f1 * per_frame_patch]
    kp_full = vd.allgather_frames(kp_local, world)
    # the asynchronous form (the transfer overlaps work queued before result())
    pending = vd.allgather_frames_async(x.vp[:, f0 * per_frame_patch:f1 * per_frame_patch], world)
    vp_full = pending.result()
    gather_ok = torch.equal(kp_full, x.kp) and torch.equal(vp_full, x.vp)
    # head-wise gathers straight into head-major buffers, two head groups in
    # reverse order (what FrameShardedLayer enqueues)
    spf = 5
    locals_ = [x.kp[:, f0 * per_frame_patch:f1 * per_frame_patch].contiguous(),
               x.vp[:, f0 * per_frame_patch:f1 * per_frame_patch].contiguous(),
               x.ks[:, f0 * spf:f1 * spf].contiguous(), x.vs[:, f0 * spf:f1 * spf].contiguous()]
    bufs = [torch.full_like(t, float("nan")) for t in (x.kp, x.vp, x.ks, x.vs)]
    pairs = list(zip(locals_, bufs))
    works = [vd.gather_heads_async(pairs, g, world) for g in ([1], [0])]
    for w in works:
        w.wait()
    gather_ok = gather_ok and all(torch.equal(b, t) for b, t in zip(bufs, (x.kp, x.vp, x.ks, x.vs)))
    # bulk gathers: one collective per tensor into rank-major staging, then
    # the copy into head-major place (each head range of two groups)
    bufs = [torch.full_like(t, float("nan")) for t in (x.kp, x.vp, x.ks, x.vs)]
    pairs = list(zip(locals_, bufs))
    works = []
    for h0, h1 in ((1, 2), (0, 1)):
        stg = [torch.empty((world, h1 - h0) + tuple(l.shape[1:]), dtype=l.dtype)
               for l in locals_]
        works.append(vd.gather_bulk_async(pairs, h0, h1, world, stg))
    for w in works:
        w.wait()
    gather_ok = gather_ok and all(torch.equal(b, t) for b, t in zip(bufs, (x.kp, x.vp, x.ks, x.vs)))
    # the transfer a gloo group gets by default: NCCL-free bulk all-gathers
    gather_ok = gather_ok and vd.FrameShardedLayer(2, world, rank, 4).gather_mode == "bulk"
    # query-block shard of the oracle layer
    n = x.shape.n_tokens
    b0, b1 = vd.qblock_range(-(-n // 64), world, rank)
    r0, r1 = b0 * 64, min(n, b1 * 64)
    idx, cnt, _ = oracle.estimate_masks(x.q[:, r0:r1].numpy(), x.kp.numpy(), [0, 1], 64, 64,
                                        "topk", 2, 32 ** -0.5)
    out, _ = oracle.block_sparse_attention(x.q[:, r0:r1].numpy(), x.kp.numpy(),
                                           x.vp.numpy(), x.ks.numpy(), x.vs.numpy(), idx, cnt,
                                           [0, 1])
    rows = torch.tensor(out)
    sizes = [torch.zeros(1, dtype=torch.long) for _ in range(world)]
    dist.all_gather(sizes, torch.tensor([rows.shape[1]]))
    padded = torch.zeros(2, max(int(s) for s in sizes), 32)
    padded[:, :rows.shape[1]] = rows
    parts = [torch.zeros_like(padded) for _ in range(world)]
    dist.all_gather(parts, padded)
    if rank == 0:
        full = torch.cat([p[:, :int(s)] for p, s in zip(parts, sizes)], 1)
        ref_idx, ref_cnt, _ = oracle.estimate_masks(x.q.numpy(), x.kp.numpy(), [0, 1], 64, 64,
                                                    "topk", 2, 32 ** -0.5)
        ref, _ = oracle.block_sparse_attention(x.q.numpy(), x.kp.numpy(), x.vp.numpy(),
                                               x.ks.numpy(), x.vs.numpy(), ref_idx, ref_cnt,
                                               [0, 1])
        result_q.put((gather_ok, float(np.abs(full.numpy() - ref).max())))
    else:
        result_q.put((gather_ok, None))


def test_frame_sharded_transfer_choice():
    """Without an NCCL group the layer moves K/V with bulk all-gathers; the
    peer-memory exchange runs only with the keys-first schedule."""
    assert vd.FrameShardedLayer(2, 2, 0, 4).gather_mode == "bulk"
    assert vd.FrameShardedLayer(2, 2, 0, 4, gather="push").gather_mode == "push"
    with pytest.raises(ValueError, match="kfirst"):
        vd.FrameShardedLayer(2, 2, 0, 4, schedule="groups", gather="push")
    with pytest.raises(ValueError, match="gather must be"):
        vd.FrameShardedLayer(2, 2, 0, 4, gather="ring")


def test_two_rank_gloo_sharding_reassembles_the_layer():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(r[0] for r in results), results
    err = [r[1] for r in results if r[1] is not None][0]
    assert err < 1e-6
