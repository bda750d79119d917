#!/usr/bin/env python
"""Benchmark of one sparse global-attention layer (the hot path) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config cfg2] [--shard qblocks|heads] [--kernel auto]

A step is one pass of the hot path over one layer of synthetic input:
block-mask estimator on the sparse heads + one block-sparse attention launch
(sparse heads through their masks, dense-profiled heads through the dense path
of the same kernel).  Default workload: config 2 (32 frames, 43,968 tokens,
16 heads x 64, mass 0.9, heads 0-3 dense).  With N > 1 ranks (torchrun, one
process per GPU, NCCL) the layer is split across ranks with total work fixed
("strong"); by default (--shard kv-allgather) each rank starts from its own
query blocks' rows and its own frames' K/V, and every step all-gathers K/V
over NCCL (NVLink) before and while the rank computes its query blocks.

Prints ONE JSON line on rank 0.  ``value`` is ms per layer (max over ranks).
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "sparse-attention-vggt_b200"))
sys.path.insert(0, REPO)

import torch  # noqa: E402

METRIC = "ms per sparse global-attn layer & kept-block TFLOPS at 32/100 frames; frames/s"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


GATHER_WHAT = {
    "bulk": "K/V (patch and special) of the other ranks' frames, one NCCL all-gather per tensor "
            "into rank-major staging plus one copy into head-major place: the patch keys first "
            "(exposed), then V and the specials while the estimator runs on the full keys",
    "heads": "K/V (patch and special) of the other ranks' frames, NCCL all-gathers per head "
             "straight into head-major place: the patch keys first (exposed), then V and the "
             "specials while the estimator runs on the full keys",
    "push": "K/V (patch and special) of the other ranks' frames: each rank's kernel stores its "
            "shards into every rank's head-major buffers over NVLink peer memory (symmetric "
            "memory, bounded handshake in the same launch): the patch keys first (exposed), "
            "then V and the specials while the estimator runs on the full keys",
}


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--config", default="cfg2")
    p.add_argument("--shard", choices=("kv-allgather", "qblocks", "heads"), default="kv-allgather",
                   help="with N > 1 ranks: kv-allgather (default) = each rank holds its query "
                        "blocks' rows and its frames' K/V and all-gathers K/V over NCCL in "
                        "every step; qblocks = query-block shards with the layer's K/V "
                        "replicated on every rank (no collective); heads = each rank holds "
                        "only a cost-balanced set of heads (no collective)")
    p.add_argument("--gather", choices=("auto", "bulk", "heads", "push"), default="auto",
                   help="kv-allgather transfer: auto (default) = push over NCCL process "
                        "groups; bulk = one NCCL all-gather per tensor, then a "
                        "copy into place; heads = NCCL all-gathers per head; push = this "
                        "library's kernel storing each rank's shards into every rank's "
                        "buffers over NVLink peer memory")
    p.add_argument("--kernel", default="auto")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--cpu-sample-blocks", type=int, default=48)
    p.add_argument("--component",
                   choices=("layer", "assembly", "triton-ref", "token-ref", "qk-topk",
                            "aggregator", "qkv"),
                   default="layer",
                   help="layer: estimator + attention (the headline); assembly: mask "
                        "assembly with history and value order + the history update; "
                        "triton-ref: the reference's own Triton block_attention (installed "
                        "in baseline/_ref) against this drop-in on the same inputs and masks; "
                        "token-ref: per-token sparse attention, this library and (when "
                        "installed) the reference's Triton kernels; qk-topk: per-frame QK "
                        "top-k, this library and the reference's Triton kernel; aggregator: "
                        "config 3, the reference's VGGT aggregator end to end with its "
                        "Triton operator and with this drop-in; qkv: the layer from its "
                        "input activations with the QKV projection + pooling fused, against "
                        "the reference's PyTorch composition")
    p.add_argument("--qk-queries", type=int, default=0,
                   help="qk-topk: query rows (default: all 43,808 tokens of the 32 frames)")
    p.add_argument("--qk-topk", default="4,16,64",
                   help="qk-topk: comma-separated top-k values per frame")
    p.add_argument("--no-reference", action="store_true",
                   help="qk-topk: skip the reference's Triton kernel")
    return p.parse_args()


def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", 0.0)),
                "source": "measured"}
    except (OSError, KeyError, ValueError):
        return dict(FALLBACK_PEAKS)


def profiled_traffic(config):
    """DRAM bytes (read + write) per attention launch from the committed ncu
    summary of this workload, or None when no summary exists."""
    import re
    path = os.path.join(REPO, "profiles", "attn_tc05_%s.md" % config)
    try:
        text = open(path).read()
    except OSError:
        return None
    m = re.search(r"traffic per launch \(read \+ write\) \| ([0-9.]+) MB", text)
    return float(m.group(1)) * 1e6 if m else None


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        if torch.cuda.is_available():
            torch.cuda.set_device(local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=300))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def reduce_max(x, world):
    if world == 1:
        return float(x)
    import torch.distributed as dist
    t = torch.tensor([float(x)], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t)


def reduce_sum(x, world):
    if world == 1:
        return float(x)
    import torch.distributed as dist
    t = torch.tensor([float(x)], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t)


class ClockSampler:
    """nvidia-smi clock / throttle sampling while the timed region runs.

    nvidia-smi takes a few hundred ms to emit its first row, longer than a
    short timed loop, so `start()` returns only once samples are flowing and
    every row carries a timestamp: `stop()` keeps the rows taken between
    `mark_begin()` and `mark_end()` (plus the first row after the end, so a
    loop shorter than the sampling period still has one sample)."""
    QUERY = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    PERIOD_MS = 20

    def __init__(self, device_index):
        self.proc = None
        self.path = None
        self.device_index = device_index
        self.t_begin = self.t_end = None

    def _rows(self):
        import datetime
        rows = []
        try:
            with open(self.path) as f:
                for line in f:
                    parts = [x.strip() for x in line.split(",")]
                    if len(parts) < 10:
                        continue
                    try:
                        ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f")
                    except ValueError:
                        continue
                    rows.append((ts.timestamp(), parts[1:]))
        except OSError:
            pass
        return rows

    def start(self, ready_timeout_s=10.0):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            bus = None
            try:
                pr = torch.cuda.get_device_properties(self.device_index)
                bus = "%08X:%02X:%02X.0" % (pr.pci_domain_id, pr.pci_bus_id, pr.pci_device_id)
            except Exception:
                pass
            cmd = ["nvidia-smi", "--query-gpu=" + self.QUERY, "--format=csv,noheader,nounits",
                   "-lms", str(self.PERIOD_MS)]
            if bus:
                cmd += ["--id=" + bus]
            self.proc = subprocess.Popen(cmd, stdout=open(self.path, "w"),
                                         stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
            return
        deadline = time.time() + ready_timeout_s
        while time.time() < deadline and not self._rows() and self.proc.poll() is None:
            time.sleep(0.02)

    def mark_begin(self):
        self.t_begin = time.time()

    def mark_end(self):
        self.t_end = time.time()
        if self.proc is None:
            return
        # wait (bounded) for the first row stamped after the timed region
        deadline = time.time() + 1.0
        while time.time() < deadline and self.proc.poll() is None:
            rows = self._rows()
            if rows and rows[-1][0] >= self.t_end:
                break
            time.sleep(self.PERIOD_MS / 1000.0)

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = self._rows()
        os.unlink(self.path)
        if self.t_begin is not None and self.t_end is not None:
            inside = [r for t, r in rows if self.t_begin <= t <= self.t_end]
            after = [r for t, r in rows if t > self.t_end][:1]
            rows = inside + after
        else:
            rows = [r for _, r in rows]
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


def shard_inputs(x, cfg, rank, world, shard, device):
    """Per-rank slice of the layer.  qblocks / kv-allgather: a contiguous range
    of 64-row query blocks, all heads; heads: a cost-balanced set of heads
    (dense-profiled heads spread out), all tokens."""
    if world == 1:
        return x.q, x.kp, x.vp, x.ks, x.vs, list(cfg.dense_heads), (0, x.shape.n_tokens)
    from vggt_sparse import distributed as vd
    if shard in ("qblocks", "kv-allgather"):
        b0, b1 = vd.qblock_range(x.shape.n_qblocks, world, rank)
        r0, r1 = b0 * cfg.block, min(x.shape.n_tokens, b1 * cfg.block)
        q = x.q[:, r0:r1].contiguous()
        return q, x.kp, x.vp, x.ks, x.vs, list(cfg.dense_heads), (r0, r1)
    mine = vd.head_assignment(cfg.heads, world, cfg.dense_heads)[rank]
    idx = torch.tensor(mine, device=device)
    dense = [i for i, h in enumerate(mine) if h in set(cfg.dense_heads)]
    sel = [t.index_select(0, idx).contiguous() for t in (x.q, x.kp, x.vp, x.ks, x.vs)]
    return (*sel, dense, (0, x.shape.n_tokens))


def _spread_blocks(qbc, n):
    n = min(n, qbc)
    return sorted(set(int(round(i * (qbc - 1) / max(n - 1, 1))) for i in range(n)))


def cpu_baseline(cfg, x_cpu, sample_blocks, check_blocks=None):
    """The reference's CPU PyTorch path (restated in oracle.cpu_path) on a
    bounded sample of query blocks spread over the layer, extrapolated to ms
    per full layer: pooling over the whole layer (timed once) plus the
    sample's per-query-block cost times the layer's query blocks.  With
    ``check_blocks`` a second, smaller sample is timed too and both per-block
    costs are reported, so the extrapolation's dependence on the sample size
    is visible."""
    from oracle import cpu_path
    shape = x_cpu.shape
    qbc = shape.n_qblocks
    scale = cfg.dim ** -0.5
    if cfg.mode == "topk":
        from oracle import topk_budget
        budget = topk_budget(cfg.retention, shape.n_tokens, shape.n_special, shape.n_blocks,
                             cfg.block)
    else:
        budget = cfg.tau
    q, kp, vp, ks, vs, k, v = (t.float() for t in (x_cpu.q, x_cpu.kp, x_cpu.vp, x_cpu.ks,
                                                     x_cpu.vs, x_cpu.k, x_cpu.v))
    t0 = time.perf_counter()
    cpu_path.block_mean(q, cfg.block)
    cpu_path.block_mean(kp, cfg.block)
    t_pool = time.perf_counter() - t0

    def per_block(n):
        qblocks = _spread_blocks(qbc, n)
        t0 = time.perf_counter()
        cpu_path.layer_sample(q, kp, vp, ks, vs, mode=cfg.mode, budget=budget,
                              dense_heads=cfg.dense_heads, qblocks=qblocks, scale=scale,
                              block=cfg.block, k_full=k, v_full=v)
        t = time.perf_counter() - t0
        # the sample re-pools the layer; that part is counted once, in t_pool
        return max(t - t_pool, 0.0) / len(qblocks), len(qblocks), t

    pb, n, t_sample = per_block(sample_blocks)
    ms = (t_pool + pb * qbc) * 1e3
    out = {"value": ms, "unit": "ms/layer", "cores": torch.get_num_threads(), "kind": "port",
           "extrapolated": True, "per_qblock_ms": pb * 1e3, "sample_qblocks": n,
           "sample": "%d of %d query blocks x 16 heads of %s (estimator pooling over the full "
                     "layer), torch fp32 CPU, extrapolated linearly to all query blocks; %.1f s "
                     "measured" % (n, qbc, cfg.name, t_pool + t_sample)}
    if check_blocks:
        pb2, n2, _ = per_block(check_blocks)
        out["per_qblock_ms_check"] = {"sample_qblocks": n2, "per_qblock_ms": pb2 * 1e3,
                                      "ratio_to_main": pb2 / pb if pb > 0 else None}
    return out


def workload_desc(cfg, shape):
    rule = ("top-k %g%% of key blocks" % (cfg.retention * 100) if cfg.mode == "topk"
            else "softmax-mass threshold %g" % cfg.tau)
    dense = ("heads %s dense" % ",".join(map(str, cfg.dense_heads))) if cfg.dense_heads else \
        "all heads sparse"
    return ("%s: one sparse global-attention layer, %d frames x 1374 tokens = %d tokens, "
            "16 heads x 64, 64x64 blocks, %s, %s; estimator + block-sparse attention"
            % (cfg.name, cfg.frames, shape.n_tokens, rule, dense))


def run_reference_arm(args, rank, world):
    from vggt_sparse.configs import CONFIGS
    from vggt_sparse.synthetic import clustered_layer
    cfg = CONFIGS[args.config]
    if rank != 0:
        return
    x = clustered_layer(cfg.frames, centres=cfg.centres, seed=0, device="cpu",
                        dtype=torch.bfloat16)
    torch.set_num_threads(os.cpu_count() or 1)
    # the same query-block sample as the cpu_baseline leg of the GPU arm
    for _ in range(args.warmup):
        cpu_baseline(cfg, x, 2)
    vals = [cpu_baseline(cfg, x, args.cpu_sample_blocks) for _ in range(args.steps)]
    ms = statistics.median(v["value"] for v in vals)
    cb = dict(vals[0])
    cb["value"] = ms
    cb["per_qblock_ms"] = statistics.median(v["per_qblock_ms"] for v in vals)
    cb["per_qblock_ms_spread"] = [min(v["per_qblock_ms"] for v in vals),
                                  max(v["per_qblock_ms"] for v in vals)]
    line = {"metric": METRIC, "value": ms, "unit": "ms/layer", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": False, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic", "impl": "reference",
            "extrapolated": True,
            "note": "each step times the reference's CPU path on %d query blocks spread over "
                    "the layer and extrapolates linearly to the full layer; value is the median "
                    "of the steps' extrapolations, not a measured full-layer step"
                    % cb["sample_qblocks"],
            "config": {"workload": workload_desc(cfg, x.shape), "frames": cfg.frames,
                       "tokens": x.shape.n_tokens, "heads": 16, "head_dim": 64},
            "cpu_baseline": cb,
            "e2e": {"value": ms, "unit": "ms/layer", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def uniform_value_order(nb):
    """Bit-reversal coverage order of the key blocks (the uniform branch of
    saf3r/patch/adaptive_block_value.py:25-38), stable for equal keys."""
    bits = max(1, math.ceil(math.log2(max(nb, 2))))
    rev = [int(format(i, "0%db" % bits)[::-1], 2) for i in range(nb)]
    return sorted(range(nb), key=lambda i: (rev[i], i))


def run_assembly_bench(args):
    """Times vggt_block_mask_assemble (history + value order, every head and
    query block in one launch) and vggt_history_update on the config's
    estimator scores; HBM roofline on their algorithmic bytes."""
    import vggt_sparse
    from vggt_sparse.configs import CONFIGS
    from vggt_sparse.synthetic import clustered_layer
    cfg = CONFIGS[args.config]
    device = torch.device("cuda", torch.cuda.current_device())
    x = clustered_layer(cfg.frames, centres=cfg.centres, seed=0, device=device, keep_full=False)
    sparse = [h for h in range(16) if h not in cfg.dense_heads]
    nb = x.shape.n_blocks
    budget = vggt_sparse.topk_budget(cfg.retention if cfg.mode == "topk" else 0.25,
                                     x.shape.n_tokens, x.shape.n_special, nb, cfg.block)
    res = vggt_sparse.block_mask_estimate(x.q, x.kp, head_ids=torch.tensor(sparse, device=device,
                                                                            dtype=torch.int32),
                                          query_block=cfg.block, key_block=cfg.block, mode="topk",
                                          topk=budget, export_scores=True)
    scores = res.scores.contiguous()
    s, qb, _ = scores.shape
    del x, res
    order = uniform_value_order(nb)
    counts, acnt = [budget] * s, [budget // 2] * s
    keep = max(1, budget // 2)
    ids, _ = vggt_sparse.assemble_masks(scores, order, counts, acnt)
    ev = torch.randn(ids.shape, device=device)
    hist = vggt_sparse.history_update(ev, ids, counts, [keep] * s)
    flush = torch.empty(256 * 1024 * 1024 // 4, device=device)

    def step():
        i2, _ = vggt_sparse.assemble_masks(scores, order, counts, acnt, hist, max_blocks=budget)
        vggt_sparse.history_update(ev, i2, counts, [keep] * s, history_len=keep)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    times = []
    for _ in range(args.steps):
        flush.zero_()
        e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
        e0.record()
        step()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    ms = statistics.median(times)
    rows = s * qb
    nbytes = rows * (nb * 4 + keep * 4 + budget * 5) + rows * (budget * 8 + keep * 4)
    peaks = load_peaks()
    line = {"metric": "ms per mask assembly (history + value order) + history update, all heads",
            "value": ms, "unit": "ms", "component": "assembly", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": False,
            "dtype": "f32", "data": "synthetic",
            "config": {"workload": "%s estimator scores: %d heads x %d query blocks x %d key "
                                   "blocks, count %d, attention %d, history %d"
                                   % (cfg.name, s, qb, nb, budget, budget // 2, keep),
                       "l2": "256 MB flush between steps"},
            "roofline": {"bound": "hbm", "achieved": nbytes / (ms * 1e-3) / 1e9,
                         "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": nbytes / (ms * 1e-3) / 1e9 / peaks["hbm_gbs"],
                         "bytes_per_step": nbytes},
            "gpu_launches": 2 * args.steps}
    print(json.dumps(line), flush=True)


def run_triton_reference_comparison(args):
    """The reference's Triton block_attention (saf3r/triton/adaptive_block_attention.py,
    installed into baseline/_ref) and vggt_sparse.block_attention on the same
    top-k masks (one count per head, as the reference kernel reads it), all 16
    heads sparse, evidence on for both.  Prints one JSON line per shape."""
    ref_dir = os.path.join(REPO, "baseline", "_ref")
    try:
        sys.path.insert(0, ref_dir)
        from saf3r.triton.adaptive_block_attention import block_attention as ref_ba
    except Exception as e:  # not installed on this machine
        print(json.dumps({"component": "triton-ref",
                          "unavailable": "reference not importable from baseline/_ref: %r" % e}))
        return
    import vggt_sparse
    from vggt_sparse.synthetic import clustered_layer
    dev = torch.device("cuda", torch.cuda.current_device())
    flush = torch.empty(256 * 1024 * 1024 // 4, device=dev)

    def timeit(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(args.steps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        return statistics.median(ts)
    for frames, centres, rho in [(4, 64, 0.25), (32, 128, 0.25), (100, 256, 0.15)]:
        x = clustered_layer(frames, centres=centres, seed=0, device=dev)
        layer = vggt_sparse.SparseGlobalLayer(16, mode="topk", retention=rho, kernel="tcgen05")
        layer.topk = vggt_sparse.topk_budget(rho, x.shape.n_tokens, x.shape.n_special,
                                             x.shape.n_blocks, 64)
        layer(x.q, x.kp, x.vp, x.ks, x.vs)
        idx, cnt = layer.last_masks
        flops = layer.kept_flops(x.shape.n_tokens, x.shape.n_patch, x.shape.n_special, 64)
        counts = cnt[:, 0].contiguous()
        heads = torch.arange(16, device=dev, dtype=torch.int32)
        args_ = (x.q, x.kp, x.vp, x.ks, x.vs, idx, counts, heads)
        o_ref, ev_ref = ref_ba(*args_)
        o_us, ev_us = vggt_sparse.block_attention(*args_)
        torch.cuda.synchronize()
        fin = torch.isfinite(ev_ref)
        t_ref = timeit(lambda: ref_ba(*args_))
        t_us = timeit(lambda: vggt_sparse.block_attention(*args_, validate=False))
        t_noev = timeit(lambda: vggt_sparse.block_attention(*args_, validate=False,
                                                            return_evidence=False))
        print(json.dumps({
            "component": "triton-ref", "unit": "ms",
            "workload": "%d frames (%d tokens), 16 sparse heads x 64, top-k %.2f (%d blocks)"
                        % (frames, x.shape.n_tokens, rho, layer.topk),
            "reference_triton_ms": t_ref, "ours_ms": t_us, "ours_no_evidence_ms": t_noev,
            "speedup": t_ref / t_us, "kept_tflop": flops / 1e12,
            "reference_tflops": flops / t_ref / 1e9, "ours_tflops": flops / t_us / 1e9,
            "max_abs_out_diff": (o_ref.float() - o_us.float()).abs().max().item(),
            "max_abs_evidence_diff": (ev_ref[fin] - ev_us[fin]).abs().max().item(),
            "same_empty_slots": bool(torch.equal(fin, torch.isfinite(ev_us))),
            "steps": args.steps, "warmup": args.warmup}), flush=True)


def run_token_attention_bench(args):
    """Per-token sparse attention on a dino_topk-like head: the 43,808 image
    tokens of a 32-frame layer, each attending to 64 random keys of every
    frame (top-k 2048, the reference's first kernel) or 128 (4096, its
    online-softmax kernel).  Reports ms and the gathered K/V bytes per second;
    the reference's Triton kernels run beside it when baseline/_ref has them."""
    import vggt_sparse
    ref = None
    try:
        sys.path.insert(0, os.path.join(REPO, "baseline", "_ref"))
        from saf3r.triton import sparse_topk_attention as ref
    except Exception:
        ref = None
    dev = torch.device("cuda", torch.cuda.current_device())
    flush = torch.empty(256 * 1024 * 1024 // 4, device=dev)
    g = torch.Generator(device=dev).manual_seed(0)
    frames, per, d = 32, 1369, 64
    n = frames * per
    q = torch.randn(n, d, device=dev, generator=g).to(torch.bfloat16)
    k = torch.randn(n, d, device=dev, generator=g).to(torch.bfloat16)
    v = torch.randn(n, d, device=dev, generator=g).to(torch.bfloat16)

    def timeit(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(args.steps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        return statistics.median(ts)
    for per_frame in (64, 128):
        topk = frames * per_frame
        base = torch.arange(frames, device=dev, dtype=torch.int32) * per
        idx = (torch.randint(0, per, (n, frames, per_frame), device=dev, generator=g,
                             dtype=torch.int32) + base[None, :, None]).reshape(n, topk)
        t_us = timeit(lambda: vggt_sparse.token_sparse_attention(q, k, v, idx))
        line = {"component": "token-ref", "unit": "ms",
                "workload": "%d queries x top-k %d (%d per frame x %d frames), dim %d, bf16"
                            % (n, topk, per_frame, frames, d),
                "ours_ms": t_us,
                "gather_gbs": n * topk * 2 * d * 2 / (t_us * 1e-3) / 1e9,
                "steps": args.steps, "warmup": args.warmup}
        if ref is not None:
            fn = (ref.fused_sparse_topk_attention if topk <= 2048
                  else ref.fused_sparse_topk_attention_2)
            o_ref = fn(q, k, v, idx)
            o_us = vggt_sparse.token_sparse_attention(q, k, v, idx)
            line["reference_kernel"] = fn.__name__
            line["reference_triton_ms"] = timeit(lambda: fn(q, k, v, idx))
            line["speedup"] = line["reference_triton_ms"] / t_us
            line["max_abs_out_diff"] = (o_ref.float() - o_us.float()).abs().max().item()
        else:
            line["reference_triton_ms"] = None
        print(json.dumps(line), flush=True)


def run_qk_topk_bench(args):
    """Per-frame QK top-k of the lazy correspondence head: the 43,808 image
    tokens of a 32-frame layer (37 x 37 patches per frame), head dim 64,
    top-4 per frame (the reference's lazy_dino_topk setting), plus top-16 and
    top-64.  Reports ms, the scores per second and the tensor roofline of the
    QK^T FLOPs; the reference's Triton kernel (baseline/_ref) runs beside it
    on the same inputs, once through its public function and once as the bare
    kernel launch that function makes."""
    import contextlib
    import io
    import vggt_sparse
    ref = None
    try:
        sys.path.insert(0, os.path.join(REPO, "baseline", "_ref"))
        from saf3r.triton import fused_qk_topk as ref
        import triton
    except Exception:
        ref = None
    dev = torch.device("cuda", torch.cuda.current_device())
    flush = torch.empty(256 * 1024 * 1024 // 4, device=dev)
    g = torch.Generator(device=dev).manual_seed(0)
    frames, per, d = 32, 1369, 64
    nk = frames * per
    n = args.qk_queries if args.qk_queries > 0 else nk
    q = torch.randn(1, n, d, device=dev, generator=g).to(torch.bfloat16)
    k = torch.randn(1, nk, d, device=dev, generator=g).to(torch.bfloat16)
    if args.no_reference:
        ref = None
    peaks = load_peaks()
    peak = peaks.get("bf16_tflops") if peaks else None

    def timeit(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(args.steps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        return statistics.median(ts)

    flops = 2.0 * n * nk * d
    for topk in (int(t) for t in args.qk_topk.split(",")):
        ours = lambda: vggt_sparse.compute_qk_topk_indices_fused(q, k, topk, num_toks_per_img=per)
        t_ms = timeit(ours)
        tf = flops / (t_ms * 1e-3) / 1e12
        line = {"component": "qk-topk", "unit": "ms",
                "workload": "%d queries x %d keys (%d frames of %d), dim %d, top-%d per frame, bf16"
                            % (n, nk, frames, per, d, topk),
                "ours_ms": t_ms, "scores_per_s": n * nk / (t_ms * 1e-3),
                "roofline": {"bound": "tensor", "achieved": tf, "peak": peak, "unit": "TFLOP/s",
                             "frac": tf / peak if peak else None,
                             "note": "QK^T FLOPs 2*Nq*Nk*D over the call; of measured bf16 burst"},
                "steps": args.steps, "warmup": args.warmup}
        if ref is not None:
            quiet = contextlib.redirect_stdout(io.StringIO())
            with quiet:
                want = ref.compute_qk_topk_indices_fused(q, k, topk, num_toks_per_img=per)
            got = ours()
            line["equal_fraction_vs_reference"] = (got == want).float().mean().item()

            def public():
                with contextlib.redirect_stdout(io.StringIO()):
                    ref.compute_qk_topk_indices_fused(q, k, topk, num_toks_per_img=per)
            line["reference_public_ms"] = timeit(public)
            # the bare kernel launch of that function (its padding and
            # launch parameters, fused_qk_topk.py:166-199)
            te = min(topk, per)
            kv = triton.next_power_of_2(te)
            bn = max(64, kv)
            pad = (bn - per % bn) % bn
            kp = torch.nn.functional.pad(k.view(1, frames, per, d), (0, 0, 0, pad)).reshape(
                1, frames * (per + pad), d)
            out = torch.full((1, n, frames * kv), -1, device=dev, dtype=torch.int32)
            grid = (triton.cdiv(n, 64), 1)

            def bare():
                ref._fused_perframe_qk_topk_kernel[grid](
                    q, kp, out, q.stride(0), q.stride(1), q.stride(2), kp.stride(0),
                    kp.stride(1), kp.stride(2), out.stride(0), out.stride(1), out.stride(2),
                    n, frames * (per + pad), d, per, segment_len=per + pad, BLOCK_M=64,
                    BLOCK_N=bn, BLOCK_DMODEL=triton.next_power_of_2(d), K_VAL=kv, num_warps=8,
                    num_stages=2)
            line["reference_kernel_ms"] = timeit(bare)
            line["speedup_vs_reference_kernel"] = line["reference_kernel_ms"] / t_ms
            line["speedup_vs_reference_public"] = line["reference_public_ms"] / t_ms
        print(json.dumps(line), flush=True)


def reference_stubs():
    """Stand-ins for two packages the reference imports at module load
    (addict in saf3r/patch, omegaconf in its DA3 model) that this image does
    not have; the VGGT path run here uses neither beyond those imports."""
    import types
    try:
        import addict  # noqa: F401
    except ImportError:
        m = types.ModuleType("addict")

        class Dict(dict):
            def __getattr__(self, key):
                try:
                    return self[key]
                except KeyError as e:
                    raise AttributeError(key) from e

            def __setattr__(self, key, value):
                self[key] = value
        m.Dict = Dict
        sys.modules["addict"] = m
    try:
        import omegaconf  # noqa: F401
    except ImportError:
        m = types.ModuleType("omegaconf")

        class OmegaConf:
            @staticmethod
            def register_new_resolver(*a, **k):
                return None

            @staticmethod
            def create(*a, **k):
                raise NotImplementedError("omegaconf is not installed")
            load = create
        m.OmegaConf = OmegaConf
        m.DictConfig = type("DictConfig", (dict,), {})
        m.ListConfig = type("ListConfig", (list,), {})
        sys.modules["omegaconf"] = m


def build_reference_aggregator(device, seed=0, retention=0.25):
    """The reference's VGGT Aggregator (saf3r/models/official_vggt/models/
    aggregator.py: ViT-L/14 patch embed with 4 registers, 24 frame + 24
    global blocks, dim 1024, 16 heads, RoPE-2D), random-init from `seed`, with
    its global attention replaced by the reference's adaptive block attention
    (saf3r/patch/adaptive_block_value.py:444-457) at a fixed top-k budget:
    retention `retention`, no escalation (audit_guard off).  The attention
    operator it calls is saf3r.triton.adaptive_block_attention.block_attention,
    looked up at every call, so assigning that attribute swaps the backend."""
    reference_stubs()
    ref_dir = os.path.join(REPO, "baseline", "_ref")
    if ref_dir not in sys.path:
        sys.path.insert(0, ref_dir)
    from saf3r.models.official_vggt.models.aggregator import Aggregator
    from saf3r.patch.adaptive_block_value import install_adaptive_block_value
    import saf3r.triton.adaptive_block_attention as ref_op
    torch.manual_seed(seed)
    model = torch.nn.Module()
    with torch.device(device):  # initialise on the device (909M parameters)
        model.aggregator = Aggregator()
    model = model.to(device).eval()  # and the buffers made by legacy constructors
    state = install_adaptive_block_value(model, retention=retention,
                                         budget_candidates=(retention,), audit_guard=False,
                                         profile_stages=True)
    return model, state, ref_op


def aggregator_forward(model, images):
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        out, _ = model.aggregator(images)
    return out


def run_aggregator_bench(args):
    """Config 3: the reference's random-init VGGT aggregator end to end on 16
    synthetic 518 x 518 views (a smooth random texture under random
    homographies), global attention sparse at top-k 25 %, forward in bf16
    autocast.  The same model and inputs run twice: with the reference's
    Triton block_attention; with vggt_sparse.block_attention assigned in its
    place; and with vggt_sparse.select_block_mask assigned as well.  The arms
    alternate step by step.  Reports the forward time (dominated by the
    reference module's host-side work, so noisy), the reference's own
    per-stage times of its global-attention module summed over the 24 layers
    (its profile_stages CUDA events), and how far the last block's output
    moves."""
    import vggt_sparse
    from vggt_sparse.synthetic import homography_views
    dev = torch.device("cuda", torch.cuda.current_device())
    frames = 16
    model, state, ref_op = build_reference_aggregator(dev)
    images = homography_views(frames, 518, seed=3, device=dev)
    triton_op = ref_op.block_attention
    calls = {"n": 0}

    def ours(*a, **k):
        calls["n"] += 1
        return vggt_sparse.block_attention(*a, **k)

    import saf3r.patch.adaptive_block_value as abv
    ref_select = abv.select_block_mask

    def forward(arm):
        _, op, select = arm
        ref_op.block_attention = op
        abv.select_block_mask = select
        e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
        e0.record()
        out = aggregator_forward(model, images)
        e1.record()
        torch.cuda.synchronize()
        stages = {}
        for r in state.records:
            for k, v in r["stage_ms"].items():
                stages[k] = stages.get(k, 0.0) + v
        return e0.elapsed_time(e1), stages, out[-1].float()

    # reference: its Triton operator and its PyTorch select_block_mask;
    # ours: the drop-in operator; ours+assembly: also the device mask assembly
    arms = (("reference", triton_op, ref_select), ("ours", ours, ref_select),
            ("ours+assembly", ours, vggt_sparse.select_block_mask))
    fwd = {a[0]: [] for a in arms}
    stage = {a[0]: [] for a in arms}
    last = {}
    try:
        for _ in range(args.warmup):
            for arm in arms:
                forward(arm)
        calls["n"] = 0
        for _ in range(args.steps):  # the arms alternate, step by step
            for arm in arms:
                t, st, last[arm[0]] = forward(arm)
                fwd[arm[0]].append(t)
                stage[arm[0]].append(st)
    finally:
        ref_op.block_attention = triton_op
        abv.select_block_mask = ref_select

    def med_stages(a):
        return {k: statistics.median(st[k] for st in stage[a]) for k in stage[a][0]}
    st_ref, st_us, st_as = med_stages("reference"), med_stages("ours"), med_stages("ours+assembly")
    t_ref, t_us = statistics.median(fwd["reference"]), statistics.median(fwd["ours"])
    s_ref, s_us = st_ref.get("sparse_attention", 0.0), st_us.get("sparse_attention", 0.0)
    diff = (last["ours"] - last["reference"]).abs()
    diff_as = (last["ours+assembly"] - last["reference"]).abs()
    line = {"component": "aggregator", "unit": "ms",
            "workload": "reference VGGT aggregator (random init, ViT-L/14 + 24 frame/24 global "
                        "blocks), 16 views 518x518 (%d tokens), global attention top-k 25%%, "
                        "bf16 autocast" % (frames * 1374),
            "reference_forward_ms": t_ref, "ours_forward_ms": t_us,
            "reference_sparse_attention_ms": s_ref, "ours_sparse_attention_ms": s_us,
            "sparse_attention_speedup": s_ref / s_us if s_us else None,
            "forward_speedup": t_ref / t_us,
            "global_attention_stages_ms": {"reference": sum(st_ref.values()),
                                           "ours": sum(st_us.values()),
                                           "ours+assembly": sum(st_as.values())},
            "mask_assembly_ms": {"reference": st_ref.get("mask_assembly"),
                                 "ours+assembly": st_as.get("mask_assembly")},
            "stage_ms_summed_over_global_layers": {"reference": st_ref, "ours": st_us,
                                                   "ours+assembly": st_as},
            "forward_ms_per_step": fwd,
            "ours_calls_per_forward": calls["n"] / (2 * args.steps),
            "ours+assembly_last_block_mean_rel_diff":
                (diff_as.mean() / last["reference"].abs().mean()).item(),
            "last_block_max_abs_diff": diff.max().item(),
            "last_block_mean_rel_diff": (diff.mean() / last["reference"].abs().mean()).item(),
            "steps": args.steps, "warmup": args.warmup}
    print(json.dumps(line), flush=True)


def run_qkv_bench(args):
    """The layer from its input activations x (config's frames, 1024 channels,
    16 heads): (a) vggt_sparse.project_qkv (tcgen05 GEMM with q/k LayerNorm,
    RoPE-2D, the layout split and the estimator's block means in the
    epilogue) then SparseGlobalLayer.forward_projected (selection from the
    means, attention); (b) the reference's composition: the qkv Linear
    (cuBLAS bf16), LayerNorm and RoPE in PyTorch (fp32, as CUDA autocast runs
    them), the layout gathers, then SparseGlobalLayer (estimator pooling Q and
    K again, selection, attention).  Random-init weights, synthetic x."""
    import vggt_sparse
    from vggt_sparse.configs import CONFIGS
    cfg = CONFIGS[args.config]
    dev = torch.device("cuda", torch.cuda.current_device())
    heads, dim, gh, spf = 16, 1024, 37, 5
    tpf = spf + gh * gh
    n = cfg.frames * tpf
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(n, dim, device=dev, generator=g).to(torch.bfloat16)
    w = (torch.randn(3 * dim, dim, device=dev, generator=g) * 0.03).to(torch.bfloat16)
    b = (torch.randn(3 * dim, device=dev, generator=g) * 0.1).to(torch.bfloat16)
    qn = torch.nn.LayerNorm(64).to(dev)
    kn = torch.nn.LayerNorm(64).to(dev)
    yy, xx = torch.meshgrid(torch.arange(gh, device=dev), torch.arange(gh, device=dev),
                            indexing="ij")
    grid = torch.stack((yy.flatten() + 1, xx.flatten() + 1), -1)
    pos = torch.cat((torch.zeros(spf, 2, dtype=torch.long, device=dev), grid)).repeat(
        cfg.frames, 1)
    pos_count = gh + 1
    cos, sin = vggt_sparse.rope_tables(pos_count, 100.0, dev)
    fr = torch.arange(cfg.frames, device=dev)[:, None] * tpf
    patches = (fr + spf + torch.arange(tpf - spf, device=dev)[None]).reshape(-1)
    specials = (fr + torch.arange(spf, device=dev)[None]).reshape(-1)
    kw = dict(mode=cfg.mode, retention=cfg.retention, tau=cfg.tau, dense_heads=cfg.dense_heads)
    fused, sep = vggt_sparse.SparseGlobalLayer(16, **kw), vggt_sparse.SparseGlobalLayer(16, **kw)
    if cfg.mode == "topk":
        shape = vggt_sparse.LayerShape(frames=cfg.frames)
        fused.topk = sep.topk = vggt_sparse.topk_budget(cfg.retention, shape.n_tokens,
                                                        shape.n_special, shape.n_blocks, 64)

    def rope(t):
        c2 = torch.cat((cos, cos), -1)
        s2 = torch.cat((sin, sin), -1)
        out = []
        for half, axis in ((t[..., :32], 0), (t[..., 32:], 1)):
            p_ = pos[:, axis]
            rot = torch.cat((-half[..., 16:], half[..., :16]), -1)
            out.append(half * c2[p_] + rot * s2[p_])
        return torch.cat(out, -1)

    def unfused():
        qkv = torch.nn.functional.linear(x, w, b).reshape(n, 3, heads, 64).permute(1, 2, 0, 3)
        q, k, v = qkv.unbind(0)
        q, k = rope(qn(q.float())), rope(kn(k.float()))
        q, k, v = q.to(torch.bfloat16).contiguous(), k.to(torch.bfloat16), v
        kp, vp = k[:, patches].contiguous(), v[:, patches].contiguous()
        ks, vs = k[:, specials].contiguous(), v[:, specials].contiguous()
        return sep(q, kp, vp, ks, vs)

    def fusedf():
        out = vggt_sparse.project_qkv(x, w, b, heads=heads, tokens_per_frame=tpf, q_norm=qn,
                                      k_norm=kn, pos=pos, pos_count=pos_count)
        return fused.forward_projected(out)

    def proj_only():
        return vggt_sparse.project_qkv(x, w, b, heads=heads, tokens_per_frame=tpf, q_norm=qn,
                                       k_norm=kn, pos=pos, pos_count=pos_count)

    flush = torch.empty(256 * 1024 * 1024 // 4, device=dev)

    def timeit(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(args.steps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        return statistics.median(ts)
    with torch.no_grad():
        a, b_ = fusedf(), unfused()
        torch.cuda.synchronize()
        same = (fused.last_masks[0] == sep.last_masks[0]).all(-1).float().mean().item()
        diff = (a.float() - b_.float()).abs()
        t_f, t_u, t_p = timeit(fusedf), timeit(unfused), timeit(proj_only)
    gemm_flops = 2.0 * n * dim * 3 * dim
    peaks = load_peaks()
    print(json.dumps({
        "component": "qkv", "unit": "ms", "config": cfg.name,
        "workload": "%s layer from x [%d, %d]: qkv projection (16 heads x 64), q/k LayerNorm, "
                    "RoPE-2D, layout split, estimator, attention" % (cfg.name, n, dim),
        "fused_layer_ms": t_f, "unfused_layer_ms": t_u, "saved_ms": t_u - t_f,
        "fused_projection_ms": t_p,
        "projection_tflops": gemm_flops / t_p / 1e9,
        "projection_frac_of_peak": gemm_flops / t_p / 1e9 / peaks["bf16_tflops"],
        "masks_equal_rows": same, "max_abs_out_diff": diff.max().item(),
        "mean_rel_out_diff": (diff.mean() / b_.float().abs().mean()).item(),
        "steps": args.steps, "warmup": args.warmup}), flush=True)


def main():
    args = parse_args()
    rank, world, local = dist_setup(args)
    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return
    if args.component == "assembly":
        if rank == 0:
            run_assembly_bench(args)
        return
    if args.component == "triton-ref":
        if rank == 0:
            run_triton_reference_comparison(args)
        return
    if args.component == "token-ref":
        if rank == 0:
            run_token_attention_bench(args)
        return
    if args.component == "qk-topk":
        if rank == 0:
            run_qk_topk_bench(args)
        return
    if args.component == "aggregator":
        if rank == 0:
            run_aggregator_bench(args)
        return
    if args.component == "qkv":
        if rank == 0:
            run_qkv_bench(args)
        return
    import vggt_sparse
    from vggt_sparse import ops
    from vggt_sparse.configs import CONFIGS
    from vggt_sparse.synthetic import clustered_layer
    cfg = CONFIGS[args.config]
    device = torch.device("cuda", torch.cuda.current_device())
    x = clustered_layer(cfg.frames, centres=cfg.centres, seed=0, device=device,
                        dtype=torch.bfloat16)
    q, kp, vp, ks, vs, dense, rows = shard_inputs(x, cfg, rank, world, args.shard, device)
    heads = q.shape[0]
    layer_kwargs = dict(mode=cfg.mode, retention=cfg.retention, tau=cfg.tau, block=cfg.block,
                        kernel=args.kernel)
    n_patch_full, n_special_full = x.shape.n_patch, x.shape.n_special
    frame_sharded = args.shard == "kv-allgather" and world > 1
    if frame_sharded:
        # sequence parallel: this rank holds the query rows of its query
        # blocks and the K/V of its frames; every step all-gathers K/V over
        # NCCL head group by head group, overlapped with the groups' compute
        from vggt_sparse import distributed as vd
        runner = vd.FrameShardedLayer(heads, world, rank, cfg.frames, dense_heads=dense,
                                      gather=None if args.gather == "auto" else args.gather,
                                      **layer_kwargs)
        f0, f1 = vd.frame_range(cfg.frames, world, rank)
        ppf, spf = x.shape.patch_h * x.shape.patch_w, x.shape.special_per_frame
        kp, vp = (t[:, f0 * ppf:f1 * ppf].contiguous() for t in (x.kp, x.vp))
        ks, vs = (t[:, f0 * spf:f1 * spf].contiguous() for t in (x.ks, x.vs))
        layers = runner.layers
    else:
        runner = vggt_sparse.SparseGlobalLayer(heads, dense_heads=dense, **layer_kwargs)
        if cfg.mode == "topk":
            # the budget follows the FULL layer size, as the reference computes it
            runner.topk = vggt_sparse.topk_budget(cfg.retention, x.shape.n_tokens,
                                                  x.shape.n_special, x.shape.n_blocks, cfg.block)
        layers = [runner]
    out = torch.empty_like(q)
    flush = torch.empty(256 * 1024 * 1024 // 4, device=device, dtype=torch.float32)

    def launches(layer):
        """Our kernels per call of one layer: estimator (pool Q, pool K, score +
        select), then, when the tcgen05 kernel runs with its workspace,
        query-block pairing (bitmaps, window costs, greedy, schedule),
        attention, and the merge launch of a key-range split (grids under 4
        waves of 2 CTAs per SM, or VGGT_ATTN_SPLIT > 1)."""
        if not layer.sparse_heads and not layer.dense_heads:
            return 0
        n = (3 if layer.sparse_heads else 0) + 1
        n_slots = len(layer.sparse_heads) + len(layer.dense_heads)
        if layer.sparse_heads and layer.pair_qblocks and args.kernel != "mma_sync" and \
                ops.attention_workspace_size(q.shape[1], n_patch_full, n_slots) > 0:
            n += 4
            items = n_slots * ((-(-q.shape[1] // cfg.block) + 1) // 2)
            forced = os.environ.get("VGGT_ATTN_SPLIT", "")
            wave = 2 * torch.cuda.get_device_properties(device).multi_processor_count
            split = int(forced) if forced in ("1", "2", "3", "4") else (
                2 if items < 4 * wave else 1)
            n += 1 if split > 1 else 0
        return n
    launches_per_step = sum(launches(l) for l in layers)

    def step(events=None):
        if events is not None:
            events[0].record()
        if frame_sharded:
            runner(q, kp, vp, ks, vs, out=out)
            if events is not None:
                events[3].record()
            return
        runner(q, kp, vp, ks, vs, out=out, events=None if events is None else events[1:])

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    flops_local = sum(l.kept_flops(q.shape[1], n_patch_full, n_special_full, q.shape[2])
                      for l in layers)

    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    sampler = ClockSampler(device.index) if rank == 0 else None
    barrier(world)
    torch.cuda.synchronize()
    if sampler:
        sampler.start()
    barrier(world)
    torch.cuda.synchronize()
    if sampler:
        sampler.mark_begin()
    for i in range(args.steps):
        flush.zero_()
        step(ev[i])
    torch.cuda.synchronize()
    if sampler:
        sampler.mark_end()
    barrier(world)
    clocks = sampler.stop() if sampler else None
    step_ms = [e[0].elapsed_time(e[3]) for e in ev]
    ms_local = sum(step_ms) / len(step_ms)
    ms = reduce_max(ms_local, world)
    if frame_sharded:
        # estimator and attention of the head groups interleave with the
        # transfers; the split is not separable by events
        att_local = est_local = None
    else:
        est_ms = [e[1].elapsed_time(e[2]) for e in ev]
        att_ms = [e[2].elapsed_time(e[3]) for e in ev]
        att_local = sum(att_ms) / len(att_ms)
        est_local = sum(est_ms) / len(est_ms)
    if frame_sharded:
        runner.check_status()   # a peer-memory exchange whose wait ran out fails the run
    flops_total = reduce_sum(flops_local, world)
    gather_alone = None
    if frame_sharded:
        # the K/V all-gather by itself (all head groups, nothing overlapped)
        # each transfer timed on its own, the barrier outside the events
        g_ms = []
        for i in range(4):
            barrier(world)
            torch.cuda.synchronize()
            g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            g0.record()
            for w in runner.gather(kp, vp, ks, vs):
                w.wait()
            g1.record()
            torch.cuda.synchronize()
            if i:
                g_ms.append(g0.elapsed_time(g1))
        gms = reduce_max(sum(g_ms) / len(g_ms), world)
        gbytes = runner.gathered_bytes(kp, ks)
        gather_alone = {"ms": gms, "bytes_received_per_rank": gbytes,
                        "gbs_per_rank": gbytes / (gms * 1e-3) / 1e9}

    # end-to-end through the public API with pinned host buffers: every step
    # uploads its five inputs and downloads its output.  `value` is the
    # throughput of a stream of layer calls through HostPipeline (uploads,
    # compute and download of neighbouring calls overlap); `serial_ms` is one
    # call with nothing overlapped (copy in, layer, copy out).
    e2e = None
    if not args.no_e2e:
        host = [t.cpu().pin_memory() for t in (q, kp, vp, ks, vs)]
        dev_in = [torch.empty_like(t) for t in (q, kp, vp, ks, vs)]
        host_out = [torch.empty(q.shape, dtype=q.dtype).pin_memory() for _ in range(2)]
        h2d = sum(t.numel() * t.element_size() for t in host)
        d2h = host_out[0].numel() * host_out[0].element_size()
        e2e_steps = args.steps

        def serial_step():
            for d_, h_ in zip(dev_in, host):
                d_.copy_(h_, non_blocking=True)
            o = runner(*dev_in)
            host_out[0].copy_(o, non_blocking=True)

        for _ in range(max(1, args.warmup // 2)):
            serial_step()
        torch.cuda.synchronize()
        barrier(world)
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(e2e_steps):
            serial_step()
        s1.record()
        torch.cuda.synchronize()
        barrier(world)
        serial_ms = reduce_max(s0.elapsed_time(s1) / e2e_steps, world)

        pipe = vggt_sparse.HostPipeline(runner)
        for i in range(max(2, args.warmup // 2)):
            pipe(*host, out=host_out[i % 2])
        pipe.synchronize()
        torch.cuda.synchronize()
        barrier(world)
        p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        p0.record()
        for i in range(e2e_steps):
            pipe(*host, out=host_out[i % 2], after=p0 if i == 0 else None)
        pipe.wait_output()
        p1.record()
        torch.cuda.synchronize()
        barrier(world)
        e2e_ms = reduce_max(p0.elapsed_time(p1) / e2e_steps, world)
        e2e = {"value": e2e_ms, "unit": "ms/layer", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "steps": e2e_steps, "serial_ms": serial_ms,
               "path": "host pinned q/k_patch/v_patch/k_special/v_special -> "
                       "vggt_sparse.HostPipeline(SparseGlobalLayer) -> host out; "
                       "consecutive calls overlap their copies with compute"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        x_cpu = clustered_layer(cfg.frames, centres=cfg.centres, seed=0, device="cpu",
                                dtype=torch.bfloat16)
        torch.set_num_threads(os.cpu_count() or 1)
        cpu = cpu_baseline(cfg, x_cpu, args.cpu_sample_blocks,
                           check_blocks=max(2, args.cpu_sample_blocks // 2))

    if rank != 0:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return
    peaks = load_peaks()
    # the attention launch alone (single layer); the whole step when the
    # frame-sharded layer interleaves transfers, estimator and attention
    att_tflops = flops_local / ((att_local if att_local is not None else ms_local) * 1e-3) / 1e12
    est_bytes = 0
    for l in layers:
        if l.sparse_heads and l.last_masks is not None:
            idx, cnt = l.last_masks
            est_bytes += (len(l.sparse_heads) * (q.shape[1] + n_patch_full) * q.shape[2] * 2 +
                          idx.numel() * 4 + cnt.numel() * 4)
    line = {
        "metric": METRIC, "value": ms, "unit": "ms/layer", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": False,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": workload_desc(cfg, x.shape), "frames": cfg.frames,
                   "tokens": x.shape.n_tokens, "heads": 16, "head_dim": 64,
                   "selection": cfg.mode, "dense_heads": list(cfg.dense_heads),
                   "parallelism": ("%s-sharded x%d%s" % (
                       args.shard, world, (", %s transfer" % runner.gather_mode)
                       if args.shard == "kv-allgather" else "")) if world > 1
                   else "single GPU",
                   "l2": "inputs 270 MB > 126 MB L2; 256 MB flush write between timed steps "
                         "(outside the per-step events)",
                   "kernel": args.kernel},
        "kept_block_tflops": flops_total / (ms * 1e-3) / 1e12,
        "kept_block_gflop_per_layer": flops_total / 1e9,
        "frames_per_s": cfg.frames / (ms * 1e-3),
        "estimator_ms": est_local, "attention_ms": att_local,
        "allgather": ({"what": GATHER_WHAT[runner.gather_mode], "alone": gather_alone}
                      if frame_sharded else None),
        "roofline": {"bound": "tensor", "kernel": "block-sparse attention (rank 0)",
                     "achieved": att_tflops, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": att_tflops / peaks["bf16_tflops"],
                     "traffic": profiled_traffic(args.config),
                     "traffic_unit": "bytes per launch (dram read + write)",
                     "traffic_source": "static: the committed ncu capture "
                                       "profiles/attn_tc05_%s.md of this workload, not "
                                       "measured in this run" % args.config,
                     "flops_per_launch": flops_local,
                     "peak_source": peaks["source"] + " bf16 burst"},
        "estimator_roofline": ({"bound": "hbm", "achieved": est_bytes / (est_local * 1e-3) / 1e9,
                                "peak": peaks["hbm_gbs"], "unit": "GB/s",
                                "frac": est_bytes / (est_local * 1e-3) / 1e9 / peaks["hbm_gbs"],
                                "bytes_per_step": est_bytes,
                                "peak_source": peaks["source"]} if est_local else None),
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
