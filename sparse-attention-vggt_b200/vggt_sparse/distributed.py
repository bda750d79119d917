"""Partitioning one global-attention layer over the GPUs of a box.

One process per GPU (``torch.distributed``, NCCL over NVLink).  The reference
runs one process per GPU on whole scenes and has no intra-layer partitioning
(SAF3R shards scenes across GPUs with CUDA_VISIBLE_DEVICES, e.g.
scripts/run_scannet50_all_gpus.sh:9); the layouts here are new:

* query-block sharding: rank r owns a contiguous range of 64-row query blocks
  (all heads).  With the layer's K/V replicated on every rank nothing crosses
  NVLink inside the layer; with K/V sharded by frames (each rank computed
  only its own tokens' K/V) one all-gather of K and V precedes the layer.
* head sharding: rank r owns a set of heads (all tokens), balanced by cost so
  dense-profiled heads are spread out.  No collective inside attention.
* frame sharding (sequence parallel, ``FrameShardedLayer``): rank r owns the
  query blocks of its rows and the K/V of its frames; every call all-gathers
  K/V head by head straight into the layout the kernels read, pipelined by
  head groups so later groups' transfers overlap earlier groups' compute.
"""
import math

import torch

from .layer import SparseGlobalLayer


def qblock_range(n_qblocks, world, rank):
    """[b0, b1) query blocks of `rank`; ranges are contiguous and cover all blocks."""
    per = math.ceil(n_qblocks / world)
    b0 = min(n_qblocks, rank * per)
    return b0, min(n_qblocks, b0 + per)


def head_assignment(n_heads, world, dense_heads=(), sparse_cost=0.3):
    """Heads per rank, greedy longest-first by cost (dense head = 1.0, sparse =
    ``sparse_cost``), each rank's list ascending.  Ties go to the lower rank."""
    dense = set(int(h) for h in dense_heads)
    order = sorted(range(n_heads), key=lambda h: (-(1.0 if h in dense else sparse_cost), h))
    load = [0.0] * world
    out = [[] for _ in range(world)]
    for h in order:
        r = min(range(world), key=lambda i: (load[i], len(out[i]), i))
        out[r].append(h)
        load[r] += 1.0 if h in dense else sparse_cost
    return [sorted(x) for x in out]


def frame_range(frames, world, rank):
    """[f0, f1) frames whose tokens rank `rank` owns under frame sharding."""
    per = math.ceil(frames / world)
    f0 = min(frames, rank * per)
    return f0, min(frames, f0 + per)


def allgather_frames(local, world, group=None):
    """All-gather a frame-sharded [H, n_local, d] tensor into [H, world * n_local, d].

    Every rank must hold the same n_local (frames divisible by world).  One
    all-gather over NCCL (gloo on CPU) lands the shards rank-major in a
    [world, H, n_local, d] buffer; one copy reorders them head-major, which is
    the layout the attention kernels read."""
    import torch.distributed as dist
    h, n, d = local.shape
    buf = torch.empty((world, h, n, d), device=local.device, dtype=local.dtype)
    dist.all_gather_into_tensor(buf.view(-1), local.contiguous().view(-1), group=group)
    return buf.permute(1, 0, 2, 3).reshape(h, world * n, d)


class PendingGather:
    """An all-gather of frame shards in flight (``allgather_frames_async``).
    ``result()`` makes the current stream wait for it and returns the
    head-major [H, world * n_local, d] tensor."""

    def __init__(self, buf, work):
        self._buf, self._work = buf, work

    def result(self):
        self._work.wait()
        w, h, n, d = self._buf.shape
        return self._buf.permute(1, 0, 2, 3).reshape(h, w * n, d)


def allgather_frames_async(local, world, group=None):
    """``allgather_frames`` started asynchronously (NCCL runs it on its own
    stream): work queued on the current stream before ``result()`` overlaps
    the transfer."""
    import torch.distributed as dist
    h, n, d = local.shape
    buf = torch.empty((world, h, n, d), device=local.device, dtype=local.dtype)
    work = dist.all_gather_into_tensor(buf.view(-1), local.contiguous().view(-1), group=group,
                                       async_op=True)
    return PendingGather(buf, work)


class QBlockShardedLayer:
    """The layer restricted to this rank's query blocks.

    ``__call__(q, kp, vp, ks, vs)`` takes the FULL q (or only this rank's rows
    when ``q_is_local``) and full K/V; it returns this rank's output rows
    [H, rows, d] and their global row range."""

    def __init__(self, heads, world, rank, **layer_kwargs):
        self.world, self.rank = world, rank
        self.layer = SparseGlobalLayer(heads, **layer_kwargs)

    def rows(self, n_tokens):
        b0, b1 = qblock_range(math.ceil(n_tokens / self.layer.block), self.world, self.rank)
        return b0 * self.layer.block, min(n_tokens, b1 * self.layer.block)

    def __call__(self, q, kp, vp, ks, vs, n_tokens=None, q_is_local=False, out=None):
        n = n_tokens if n_tokens is not None else q.shape[1]
        r0, r1 = self.rows(n)
        if self.layer.mode == "topk" and self.layer.topk is None:
            # the budget follows the FULL layer, as the reference computes it
            from .layer import topk_budget
            nb = math.ceil(kp.shape[1] / self.layer.block)
            self.layer.topk = topk_budget(self.layer.retention, n, ks.shape[1], nb,
                                          self.layer.block)
        ql = q if q_is_local else q[:, r0:r1].contiguous()
        return self.layer(ql, kp, vp, ks, vs, out=out), (r0, r1)


class HeadShardedLayer:
    """The layer restricted to this rank's heads (``head_assignment``)."""

    def __init__(self, heads, world, rank, dense_heads=(), **layer_kwargs):
        self.heads = head_assignment(heads, world, dense_heads)[rank]
        local_dense = [i for i, h in enumerate(self.heads) if h in set(dense_heads)]
        self.layer = SparseGlobalLayer(len(self.heads), dense_heads=local_dense, **layer_kwargs)

    def __call__(self, q, kp, vp, ks, vs, out=None):
        idx = torch.tensor(self.heads, device=q.device)
        sel = [t.index_select(0, idx).contiguous() for t in (q, kp, vp, ks, vs)]
        if self.layer.mode == "topk" and self.layer.topk is None:
            from .layer import topk_budget
            nb = math.ceil(kp.shape[1] / self.layer.block)
            self.layer.topk = topk_budget(self.layer.retention, q.shape[1], ks.shape[1], nb,
                                          self.layer.block)
        return self.layer(*sel, out=out), self.heads


def gather_heads_async(pairs, heads, world, group=None):
    """All-gather, for each head h in ``heads`` and each (local, full) pair,
    the frame shard local[h] ([n_local, d]) into full[h] ([world * n_local,
    d]): ranks' shards land rank-major, which for frame-major rows is the
    layer's row order, so full[h] needs no reordering.  With NCCL the calls
    of one invocation are coalesced into one launch on NCCL's stream; returns
    a handle whose ``wait()`` makes the current stream wait for them."""
    import torch.distributed as dist
    backend = dist.get_backend(group)
    calls = [(full[h], local[h]) for h in heads for local, full in pairs]
    if backend == "nccl":
        dev = calls[0][1].device if calls else None
        with dist._coalescing_manager(group=group, device=dev, async_ops=True) as cm:
            for dst, src in calls:
                dist.all_gather_into_tensor(dst, src, group=group)
        return cm
    works = [dist.all_gather_into_tensor(dst, src, group=group, async_op=True)
             for dst, src in calls]

    class _Works:
        def wait(self):
            for w in works:
                w.wait()
    return _Works()


def gather_bulk_async(pairs, h0, h1, world, staging, group=None):
    """All-gather heads [h0, h1) of every (local, full) pair with one
    collective per tensor: each rank's local[h0:h1] ([h1 - h0, n_local, d],
    contiguous in the head-major layout) lands rank-major in the matching
    ``staging`` buffer ([world, h1 - h0, n_local, d]).  The handle's
    ``wait()`` makes the current stream wait for the transfer, then copies
    staging into full[h0:h1] ([h1 - h0, world * n_local, d]), the layer's
    head-major row order.  One large message per tensor and rank instead of
    one per head keeps NCCL near its bulk rate as the rank count grows."""
    import torch.distributed as dist
    # the output as [world * (h1 - h0), n_local, d]: rank-major, the form
    # every backend accepts
    calls = [(stg.view((-1,) + tuple(stg.shape[2:])), local[h0:h1])
             for (local, _), stg in zip(pairs, staging)]
    if dist.get_backend(group) == "nccl":
        with dist._coalescing_manager(group=group, device=calls[0][1].device,
                                      async_ops=True) as cm:
            for dst, src in calls:
                dist.all_gather_into_tensor(dst, src, group=group)
        works = [cm]
    else:
        works = [dist.all_gather_into_tensor(dst, src, group=group, async_op=True)
                 for dst, src in calls]

    class _Bulk:
        def wait(self):
            for w in works:
                w.wait()
            for (_, full), stg in zip(pairs, staging):
                hg, n, d = h1 - h0, stg.shape[2], stg.shape[3]
                full[h0:h1].view(hg, world, n, d).copy_(stg.permute(1, 0, 2, 3))
    return _Bulk()


def _backend(group):
    import torch.distributed as dist
    return dist.get_backend(group) if dist.is_available() and dist.is_initialized() else None


class _EventWait:
    """A transfer handle: ``wait()`` orders the current stream after ``event``."""

    def __init__(self, event):
        self.event = event

    def wait(self):
        torch.cuda.current_stream().wait_event(self.event)


class _PushExchange:
    """The frame-shard exchange over NVLink peer memory (``vggt_kv_push``).

    The full head-major kp, vp, ks, vs ([heads, world * n_local, d] each) and
    the kernel's flag words sit in one symmetric allocation
    (``torch.distributed._symmetric_memory``): the same size and layout on
    every rank, every rank's mapped into every other's address space.  Each
    exchange runs two launches on a side stream: the patch keys (with the
    start handshake), then V and the special keys and values.  Every launch
    stores this rank's shards into all ranks' buffers and returns once this
    rank's buffers hold every rank's rows."""

    def __init__(self, kp_local, ks_local, world, rank, group):
        import ctypes

        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem

        from . import _lib
        h, npl, d = kp_local.shape
        nsl = ks_local.shape[1]
        es = kp_local.element_size()
        dev = kp_local.device
        rows = (npl, npl, nsl, nsl)
        sizes = [h * world * n * d * es for n in rows]
        self.offsets, off = [], 0
        for b in sizes:
            self.offsets.append(off)
            off += (b + 255) // 256 * 256
        self.lib = _lib.load()
        flag_bytes = self.lib.vggt_kv_push_flag_bytes(world)
        if flag_bytes <= 0:
            raise ValueError("the peer-memory exchange supports at most 16 ranks, not %d" % world)
        self.flags_off = off
        buf = symm_mem.empty(off + flag_bytes, dtype=torch.uint8, device=dev)
        buf[off:].zero_()
        grp = group if group is not None else dist.group.WORLD
        self.handle = symm_mem.rendezvous(buf, grp)
        # the peers' addresses of this allocation, in rank order
        delta = buf.data_ptr() - int(self.handle.buffer_ptrs[rank])
        self.bases = (ctypes.c_void_p * world)(*[int(b) + delta for b in self.handle.buffer_ptrs])
        self.buf = buf
        self.full = tuple(buf[o:o + b].view(kp_local.dtype).view(h, world * n, d)
                          for o, b, n in zip(self.offsets, sizes, rows))
        self.world, self.rank, self.heads, self.dim = world, rank, h, d
        self.elem = es
        self.epoch = 0
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.stream = torch.cuda.Stream(device=dev)
        self.grid = 0
        # every rank's flag words are zero before any rank signals
        torch.cuda.synchronize(dev)
        dist.barrier(group=grp)

    def _push(self, shards, which, phase, handshake):
        import ctypes

        from . import _lib
        n = len(shards)
        ptrs = (ctypes.c_void_p * n)(*[t.data_ptr() for t in shards])
        rows = (ctypes.c_int64 * n)(*[t.shape[1] for t in shards])
        offs = (ctypes.c_int64 * n)(*[self.offsets[w] for w in which])
        rc = self.lib.vggt_kv_push(ptrs, rows, offs, n, self.heads, self.dim, self.elem,
                                   self.bases, self.world, self.rank, self.flags_off, phase,
                                   self.epoch, handshake, self.grid, self.status.data_ptr(),
                                   self.stream.cuda_stream)
        _lib.check(rc)

    def exchange(self, kp_local, vp_local, ks_local, vs_local):
        """Enqueues one exchange; returns the handles of the keys and of the rest."""
        shards = [t.contiguous() for t in (kp_local, vp_local, ks_local, vs_local)]
        self.stream.wait_stream(torch.cuda.current_stream())   # shards written, readers done
        self.epoch = self.epoch % 0x7fffffff + 1
        with torch.cuda.stream(self.stream):
            self._push(shards[:1], (0,), 0, 1)
            ev_k = torch.cuda.Event()
            ev_k.record(self.stream)
            self._push(shards[1:], (1, 2, 3), 1, 0)
            ev_v = torch.cuda.Event()
            ev_v.record(self.stream)
        for t in shards:
            t.record_stream(self.stream)
        return [_EventWait(ev_k), _EventWait(ev_v)]

    def check_status(self):
        """Raises if a wait of an exchange ran out (synchronises)."""
        if int(self.status.item()):
            raise RuntimeError("a K/V exchange wait ran out (status %d): outputs are invalid"
                               % int(self.status.item()))


class FrameShardedLayer:
    """The layer with its K/V sharded by frames and its query blocks split
    across ranks (sequence parallel: what a QKV projection applied to each
    rank's own frames leaves on each GPU).

    ``__call__(q_local, kp_local, vp_local, ks_local, vs_local, out=None)``
    takes this rank's query rows ``rows(n_tokens)`` of q and the patch /
    special K/V of its frames ``frame_range`` (every rank the same number of
    frames), and returns this rank's output rows.  K and V are all-gathered
    into head-major buffers.  The default is ``gather="push"`` for
    ``schedule="kfirst"`` over NCCL and ``"bulk"`` otherwise.  ``gather="bulk"`` moves one
    all-gather per tensor into rank-major staging and copies it into place;
    ``gather="heads"`` (and any head group that is not a consecutive range)
    moves one all-gather per head and tensor straight into place (more,
    smaller messages: slower as the rank count grows).  Either
    way the calls of one step are coalesced into one launch on NCCL's stream.
    ``gather="push"`` (``schedule="kfirst"`` only) skips NCCL: the full
    buffers live in symmetric memory and ``vggt_kv_push`` stores each rank's
    shards straight into every rank's buffers over NVLink, with a bounded
    handshake in the same launch (``check_status()`` reports an expired wait).

    ``schedule="kfirst"`` (default): one layer over all heads; the patch keys
    move first, and V and the specials follow on NCCL's stream while the
    estimator runs on the full keys, so only the key transfer is exposed.
    ``schedule="groups"``: one layer per head group in ``groups`` order
    (default: the dense-profiled heads, then the rest); group g+1's transfer
    runs while group g computes, at the price of one attention launch per
    group.
    """

    def __init__(self, heads, world, rank, frames, *, dense_heads=(), schedule="kfirst",
                 groups=None, group=None, gather=None, **layer_kwargs):
        if frames % world:
            raise ValueError("frames (%d) must divide evenly over %d ranks" % (frames, world))
        if schedule not in ("kfirst", "groups"):
            raise ValueError("schedule must be 'kfirst' or 'groups'")
        if gather is None:
            gather = "push" if schedule == "kfirst" and _backend(group) == "nccl" else "bulk"
        if gather not in ("heads", "bulk", "push"):
            raise ValueError("gather must be 'heads', 'bulk' or 'push'")
        if gather == "push" and schedule != "kfirst":
            raise ValueError("gather='push' runs with schedule='kfirst'")
        self.gather_mode = gather
        self.world, self.rank, self.frames, self.group = world, rank, frames, group
        self.schedule = schedule
        dense = sorted(set(int(h) for h in dense_heads))
        if schedule == "kfirst":
            if groups is not None:
                raise ValueError("groups apply to schedule='groups' only")
            groups = [list(range(heads))]
        elif groups is None:
            rest = [h for h in range(heads) if h not in set(dense)]
            groups = [g for g in (dense, rest) if g]
        flat = sorted(h for g in groups for h in g)
        if flat != list(range(heads)):
            raise ValueError("groups must cover every head exactly once")
        self.groups = [list(g) for g in groups]
        self.heads = heads
        self.layers = [SparseGlobalLayer(heads, dense_heads=dense, head_subset=g, **layer_kwargs)
                       for g in self.groups]
        self._full = {}

    @property
    def block(self):
        return self.layers[0].block

    def rows(self, n_tokens):
        b0, b1 = qblock_range(math.ceil(n_tokens / self.block), self.world, self.rank)
        return b0 * self.block, min(n_tokens, b1 * self.block)

    def gathered_bytes(self, kp_local, ks_local):
        """Bytes this rank receives per call (the other ranks' shards)."""
        per = (kp_local.numel() + ks_local.numel()) * kp_local.element_size() * 2
        return per * (self.world - 1)

    def _exchange(self, kp_local, ks_local):
        key = ("push", kp_local.device, kp_local.shape, ks_local.shape, kp_local.dtype)
        ex = self._full.get(key)
        if ex is None:
            ex = _PushExchange(kp_local, ks_local, self.world, self.rank, self.group)
            self._full[key] = ex
        return ex

    def check_status(self):
        """Raises if a wait of a peer-memory exchange ran out (synchronises)."""
        for v in self._full.values():
            if isinstance(v, _PushExchange):
                v.check_status()

    def _buffers(self, kp_local, ks_local):
        if self.gather_mode == "push":
            return self._exchange(kp_local, ks_local).full
        key = (kp_local.device, kp_local.shape, ks_local.shape, kp_local.dtype)
        buf = self._full.get(key)
        if buf is None:
            h, npl, d = kp_local.shape
            nsl = ks_local.shape[1]
            mk = lambda n: torch.empty((h, self.world * n, d), device=kp_local.device,
                                       dtype=kp_local.dtype)
            buf = (mk(npl), mk(npl), mk(nsl), mk(nsl))
            self._full[key] = buf
        return buf

    def _staging(self, pairs, heads):
        """Rank-major receive buffers [world, |heads|, n_local, d], one per
        tensor of ``pairs``, cached by shape."""
        # one set per head range and tensor list: transfers of different
        # groups are in flight at the same time
        key = ("stg", heads[0], len(heads)) + tuple((l.device, l.shape, l.dtype)
                                                    for l, _ in pairs)
        stg = self._full.get(key)
        if stg is None:
            stg = [torch.empty((self.world, len(heads)) + tuple(l.shape[1:]), device=l.device,
                               dtype=l.dtype) for l, _ in pairs]
            self._full[key] = stg
        return stg

    def _gather(self, pairs, heads):
        # bulk transfers need a consecutive head range; other groups move
        # head by head
        if self.gather_mode == "bulk" and list(heads) == list(range(heads[0], heads[-1] + 1)):
            return gather_bulk_async(pairs, heads[0], heads[-1] + 1, self.world,
                                     self._staging(pairs, heads), self.group)
        return gather_heads_async(pairs, heads, self.world, self.group)

    def gather(self, kp_local, vp_local, ks_local, vs_local):
        """Enqueues this layer's K/V all-gathers into its full buffers in the
        order the schedule consumes them; returns one handle per step
        (``wait()`` orders the current stream after that transfer)."""
        if self.gather_mode == "push":
            return self._exchange(kp_local, ks_local).exchange(kp_local, vp_local, ks_local,
                                                               vs_local)
        kp, vp, ks, vs = self._buffers(kp_local, ks_local)
        if self.schedule == "kfirst":
            heads = self.groups[0]
            return [self._gather(((kp_local, kp),), heads),
                    self._gather(((vp_local, vp), (ks_local, ks), (vs_local, vs)), heads)]
        pairs = ((kp_local, kp), (vp_local, vp), (ks_local, ks), (vs_local, vs))
        return [self._gather(pairs, g) for g in self.groups]

    def __call__(self, q_local, kp_local, vp_local, ks_local, vs_local, out=None):
        # every rank holds the same number of frames
        n_tokens = self.world * (kp_local.shape[1] + ks_local.shape[1])
        kp, vp, ks, vs = self._buffers(kp_local, ks_local)
        for layer in self.layers:
            if layer.mode == "topk" and layer.topk is None:
                # the budget follows the FULL layer, as the reference computes it
                from .layer import topk_budget
                nb = math.ceil(kp.shape[1] / layer.block)
                layer.topk = topk_budget(layer.retention, n_tokens, ks.shape[1], nb, layer.block)
        # every transfer is enqueued up front; each compute step waits only
        # for what it reads
        pending = self.gather(kp_local, vp_local, ks_local, vs_local)
        if out is None:
            out = torch.empty_like(q_local)
        if self.schedule == "kfirst":
            layer = self.layers[0]
            pending[0].wait()
            layer.estimate(q_local, kp, ks.shape[1])
            pending[1].wait()
            layer.attend(q_local, kp, vp, ks, vs, out=out)
            return out
        for layer, work in zip(self.layers, pending):
            work.wait()
            layer(q_local, kp, vp, ks, vs, out=out)
        return out

    def kept_flops(self, n_tokens, n_patch, n_special, dim):
        return sum(l.kept_flops(n_tokens, n_patch, n_special, dim) for l in self.layers)
