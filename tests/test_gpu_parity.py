"""GPU parity: the CUDA path (through the C ABI) against the CPU oracle and the
golden vectors from the reference.

Tolerances: attention outputs in bf16/fp16 follow the reference's own test
(rtol=.02, atol=.006, tests/test_adaptive_block_value.py:180) and the stated
bar max-abs <= 2e-2, mean-relative <= 1e-2 against fp32; evidence rtol=atol=1e-4
(:184); block ids bit-exact given identical fp32 pooled scores; pooled scores
rtol=1e-4 / atol=1e-5 against the fp32 oracle.
"""
import math

import numpy as np
import pytest
import torch

import oracle
import vggt_sparse
from conftest import load_golden
from vggt_sparse import ops
from vggt_sparse.synthetic import clustered_layer

pytestmark = pytest.mark.gpu

KERNELS = ["mma_sync", "tcgen05"]
EVIDENCE_KERNELS = {"mma_sync", "tcgen05"}


def _supported(kernel, d, bq, bk):
    return kernel == "mma_sync" or (d == 64 and bq == 64 and bk == 64)


def check_out(actual, expected, rtol=0.02, atol=0.006):
    a = actual.float().cpu().numpy()
    e = np.asarray(expected, dtype=np.float32)
    np.testing.assert_allclose(a, e, rtol=rtol, atol=atol)
    assert np.max(np.abs(a - e)) <= 2e-2
    assert np.mean(np.abs(a - e)) / max(np.mean(np.abs(e)), 1e-12) <= 1e-2


@pytest.mark.parametrize("cfg,tau", [("cfg2", 0.9), ("cfg5", 0.85)])
def test_mass_select_on_layer_rows_matches_reference_counts(cuda, golden, cfg, tau):
    """The kernel's mass selection on pooled-score rows of the 32- and
    256-frame layers (tests/golden/mass_rows.npz): ids bit-exact against the
    oracle and counts equal to the reference's own fp32 softmax +
    concentration rule recorded in the fixture."""
    g = golden("mass_rows.npz")
    scores = g["%s_scores" % cfg]
    ids, counts = vggt_sparse.block_select(torch.tensor(scores, device=cuda), mode="mass",
                                           tau=tau)
    exp, exp_counts = oracle.select_mass(scores, tau)
    np.testing.assert_array_equal(counts.cpu().numpy(), exp_counts)
    np.testing.assert_array_equal(ids.cpu().numpy(), exp)
    np.testing.assert_array_equal(counts.cpu().numpy(), g["%s_m%d" % (cfg, round(tau * 100))])


@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("case", ["d64_bq64_bk64", "d32_bq32_bk128", "d64_bq32_bk32",
                                  "d32_bq64_bk64"])
def test_block_attention_matches_reference_golden(cuda, kernel, dtype, case):
    g = load_golden("attention_%s.npz" % case)
    d, bq, bk = (int(x[1:]) if i == 0 else int(x[2:]) for i, x in enumerate(case.split("_")))
    if not _supported(kernel, d, bq, bk):
        pytest.skip("shape served by the mma.sync kernel")
    t = {k: torch.tensor(g[k]).to(cuda, dtype) for k in ("q", "kp", "vp", "ks", "vs")}
    masks = torch.tensor(g["masks"], device=cuda)
    counts = torch.tensor(g["counts"], device=cuda)
    heads = torch.tensor(g["heads"], device=cuda)
    with_ev = kernel in EVIDENCE_KERNELS
    out, ev = vggt_sparse.block_attention(t["q"], t["kp"], t["vp"], t["ks"], t["vs"], masks, counts,
                                          heads, query_block=bq, key_block=bk,
                                          scale=float(g["scale"]), kernel=kernel,
                                          return_evidence=with_ev)
    for head in g["heads"]:
        check_out(out[head], g["out"][head])
    if not with_ev:
        return
    finite = np.isfinite(g["evidence"])
    evn = ev.cpu().numpy()
    np.testing.assert_array_equal(np.isfinite(evn), finite)
    np.testing.assert_allclose(evn[finite], g["evidence"][finite], rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("head_dim", [32, 64])
@pytest.mark.parametrize("query_block", [32, 64])
@pytest.mark.parametrize("key_block", [32, 64, 128])
def test_reference_parameter_grid_against_oracle(cuda, dtype, head_dim, query_block, key_block):
    """The full grid of tests/test_adaptive_block_value.py:154-184 (N=137 tail
    query block, tail key block, 7 specials, heads [0,2], counts [2,3])."""
    torch.manual_seed(8)
    n = 137
    q = torch.randn(3, n, head_dim).to(dtype)
    npatch = 2 * key_block + 43 if key_block >= 64 else 2 * key_block + 19
    kp = torch.randn(3, npatch, head_dim).to(dtype)
    vp = torch.randn_like(kp)
    ks = torch.randn(3, 7, head_dim).to(dtype)
    vs = torch.randn_like(ks)
    nq = math.ceil(n / query_block)
    patterns = [[0, 2, -1], [1, 2, -1], [0, 1, -1]]
    masks = torch.tensor([[patterns[i % 3] for i in range(nq)], [[0, 1, 2]] * nq],
                         dtype=torch.int32)
    heads = torch.tensor([0, 2], dtype=torch.int32)
    counts = torch.tensor([2, 3], dtype=torch.int32)
    exp_out, exp_ev = oracle.block_sparse_attention(
        q.float().numpy(), kp.float().numpy(), vp.float().numpy(), ks.float().numpy(),
        vs.float().numpy(), masks.numpy(), counts.numpy(), heads.numpy(),
        query_block=query_block, key_block=key_block, scale=0.2)
    for kernel in KERNELS:
        if not _supported(kernel, head_dim, query_block, key_block):
            continue
        with_ev = kernel in EVIDENCE_KERNELS
        out, ev = vggt_sparse.block_attention(
            q.to(cuda), kp.to(cuda), vp.to(cuda), ks.to(cuda), vs.to(cuda), masks.to(cuda),
            counts.to(cuda), heads.to(cuda), query_block=query_block, key_block=key_block,
            scale=0.2, kernel=kernel, return_evidence=with_ev)
        for head in (0, 2):
            check_out(out[head], exp_out[head])
        if not with_ev:
            continue
        finite = np.isfinite(exp_ev)
        np.testing.assert_allclose(ev.cpu().numpy()[finite], exp_ev[finite], rtol=1e-4, atol=1e-4)


def test_reference_cpu_layer_path(cuda):
    """Same masks and q/k/v as the reference's CPU branch of
    AdaptiveBlockValueAttention.forward (adaptive_block_value.py:371-385)."""
    g = load_golden("layer_cpu.npz")
    dt = torch.float16
    q = torch.tensor(g["q"]).to(cuda, dt)
    k = torch.tensor(g["k"]).to(cuda, dt)
    v = torch.tensor(g["v"]).to(cuda, dt)
    patches = torch.tensor(g["patches"], device=cuda)
    specials = torch.tensor(g["specials"], device=cuda)
    kp, vp = k[:, patches].contiguous(), v[:, patches].contiguous()
    ks, vs = k[:, specials].contiguous(), v[:, specials].contiguous()
    masks = torch.tensor(g["masks"], device=cuda).contiguous()
    h = q.shape[0]
    counts = torch.full((h,), masks.shape[-1], device=cuda, dtype=torch.int32)
    heads = torch.arange(h, device=cuda, dtype=torch.int32)
    block = int(g["block"])
    out, _ = vggt_sparse.block_attention(q, kp, vp, ks, vs, masks, counts, heads,
                                         query_block=block, key_block=block,
                                         scale=float(g["scale"]))
    check_out(out, g["out"])


def _layer(cuda, frames=4, centres=64, seed=0, heads=16):
    return clustered_layer(frames, centres=centres, heads=heads, seed=seed, device="cpu",
                           dtype=torch.bfloat16)


@pytest.mark.parametrize("mode,budget", [("topk", 22), ("topk", 1), ("topk", 86),
                                         ("mass", 0.9), ("mass", 0.5), ("mass", 1.0)])
def test_estimator_matches_oracle_cfg1(cuda, mode, budget):
    x = _layer(cuda)
    q, kp = x.q.to(cuda), x.kp.to(cuda)
    heads = [1, 5, 9, 15]
    res = vggt_sparse.block_mask_estimate(q, kp, head_ids=heads, mode=mode,
                                          topk=budget if mode == "topk" else None,
                                          tau=budget if mode == "mass" else None,
                                          export_scores=True)
    scale = 64 ** -0.5
    pq, _ = oracle.block_mean(x.q.float().numpy()[heads], 64)
    pk, _ = oracle.block_mean(x.kp.float().numpy()[heads], 64)
    exp_scores = oracle.pooled_scores(pq, pk, scale)
    got_scores = res.scores.cpu().numpy()
    np.testing.assert_allclose(got_scores, exp_scores, rtol=1e-4, atol=1e-5)
    # bit-exact selection given the kernel's own fp32 scores
    if mode == "topk":
        exp_ids = oracle.select_topk(got_scores, budget)
        exp_counts = np.full(exp_ids.shape[:-1], exp_ids.shape[-1])
    else:
        exp_ids, exp_counts = oracle.select_mass(got_scores, budget)
    np.testing.assert_array_equal(res.counts.cpu().numpy(), exp_counts)
    np.testing.assert_array_equal(res.indices.cpu().numpy(), exp_ids)


@pytest.mark.parametrize("mode,budget", [("topk", 7), ("mass", 0.85)])
def test_select_kernel_bit_exact_with_ties(cuda, mode, budget):
    rng = np.random.default_rng(5)
    scores = (rng.integers(0, 9, size=(3, 50, 233)) / 4.0).astype(np.float32)
    scores[0, 0] = 0.0
    scores[0, 1, ::2] = -0.0            # signed zeros tie with +0.0
    ids, counts = vggt_sparse.block_select(torch.tensor(scores, device=cuda), mode=mode,
                                           topk=budget if mode == "topk" else None,
                                           tau=budget if mode == "mass" else None)
    if mode == "topk":
        exp = oracle.select_topk(scores, budget)
        exp_counts = np.full(exp.shape[:-1], budget)
    else:
        exp, exp_counts = oracle.select_mass(scores, budget)
    np.testing.assert_array_equal(counts.cpu().numpy(), exp_counts)
    np.testing.assert_array_equal(ids.cpu().numpy(), exp)


@pytest.mark.parametrize("rows,width", [(40, 5476), (6, 12000)])
def test_select_kernel_bit_exact_random_wide_rows(cuda, rows, width):
    """cfg5-wide rows (8 rows per CTA) and rows past that (2 rows per CTA)."""
    rng = np.random.default_rng(7)
    scores = (rng.standard_normal((rows, width)) * 4).astype(np.float32)
    for mode, b in (("topk", 315), ("mass", 0.85), ("mass", 0.99)):
        ids, counts = vggt_sparse.block_select(torch.tensor(scores, device=cuda), mode=mode,
                                               topk=b if mode == "topk" else None,
                                               tau=b if mode == "mass" else None)
        if mode == "topk":
            exp = oracle.select_topk(scores, b)
            exp_counts = np.full(rows, b)
        else:
            exp, exp_counts = oracle.select_mass(scores, b)
        np.testing.assert_array_equal(counts.cpu().numpy(), exp_counts)
        np.testing.assert_array_equal(ids.cpu().numpy(), exp)


@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("mode", ["topk", "mass"])
def test_full_layer_cfg1_against_oracle(cuda, kernel, mode):
    """Estimator + one attention launch (sparse heads from masks, heads 0 and
    3 dense) at config 1, checked on every query block of 4 heads."""
    x = _layer(cuda)
    layer = vggt_sparse.SparseGlobalLayer(16, mode=mode, retention=0.25, tau=0.9,
                                          dense_heads=(0, 3), kernel=kernel)
    dev = {k: getattr(x, k).to(cuda) for k in ("q", "kp", "vp", "ks", "vs")}
    out = layer(dev["q"], dev["kp"], dev["vp"], dev["ks"], dev["vs"])
    idx, cnt = (t.cpu().numpy() for t in layer.last_masks)
    sparse = layer.sparse_heads
    exp, _ = oracle.block_sparse_attention(
        x.q.float().numpy(), x.kp.float().numpy(), x.vp.float().numpy(), x.ks.float().numpy(),
        x.vs.float().numpy(), idx, cnt, sparse)
    for head in (1, 7, 15):
        check_out(out[head], exp[head])
    dense_exp = oracle.dense_attention(x.q.float().numpy()[[0, 3]],
                                       x.k.float().numpy()[[0, 3]],
                                       x.v.float().numpy()[[0, 3]])
    check_out(out[[0, 3]], dense_exp)


def test_empty_counts_attend_only_specials(cuda):
    torch.manual_seed(1)
    q = torch.randn(2, 100, 64).to(torch.bfloat16)
    kp = torch.randn(2, 130, 64).to(torch.bfloat16)
    vp = torch.randn_like(kp)
    ks = torch.randn(2, 5, 64).to(torch.bfloat16)
    vs = torch.randn_like(ks)
    idx = torch.full((1, 2, 3), -1, dtype=torch.int32)
    cnt = torch.zeros(1, dtype=torch.int32)
    heads = torch.tensor([1], dtype=torch.int32)
    out, ev = vggt_sparse.block_attention(*(t.to(cuda) for t in (q, kp, vp, ks, vs, idx, cnt,
                                                                  heads)))
    exp = oracle.dense_attention(q.float().numpy()[[1]], ks.float().numpy()[[1]],
                                 vs.float().numpy()[[1]])
    check_out(out[1:2], exp)
    assert torch.isinf(ev).all()


def test_no_specials(cuda):
    torch.manual_seed(2)
    q = torch.randn(1, 70, 64).to(torch.bfloat16)
    kp = torch.randn(1, 70, 64).to(torch.bfloat16)
    vp = torch.randn_like(kp)
    e = q.new_empty((1, 0, 64))
    idx = torch.tensor([[[1, 0], [0, 1]]], dtype=torch.int32)
    cnt = torch.tensor([2], dtype=torch.int32)
    heads = torch.tensor([0], dtype=torch.int32)
    out, _ = vggt_sparse.block_attention(q.to(cuda), kp.to(cuda), vp.to(cuda), e.to(cuda),
                                         e.to(cuda), idx.to(cuda), cnt.to(cuda), heads.to(cuda))
    exp = oracle.dense_attention(q.float().numpy(), kp.float().numpy(), vp.float().numpy())
    check_out(out, exp)


def test_invalid_ids_counts_heads_raise(cuda):
    q = torch.randn(2, 64, 64, device=cuda).to(torch.bfloat16)
    kp = torch.randn(2, 128, 64, device=cuda).to(torch.bfloat16)
    ks = torch.randn(2, 5, 64, device=cuda).to(torch.bfloat16)
    heads = torch.tensor([0], device=cuda, dtype=torch.int32)
    bad_id = torch.tensor([[[0, 7]]], device=cuda, dtype=torch.int32)
    two = torch.tensor([2], device=cuda, dtype=torch.int32)
    with pytest.raises(ValueError, match="block id"):
        vggt_sparse.block_attention(q, kp, kp, ks, ks, bad_id, two, heads, validate=True)
    with pytest.raises(ValueError, match="count"):
        vggt_sparse.block_attention(q, kp, kp, ks, ks, bad_id, torch.tensor(
            [5], device=cuda, dtype=torch.int32), heads, validate=True)
    with pytest.raises(ValueError, match="head id"):
        vggt_sparse.block_attention(q, kp, kp, ks, ks, bad_id[:, :, :1], two.clamp(max=1),
                                    torch.tensor([4], device=cuda, dtype=torch.int32),
                                    validate=True)
    # the context is still usable afterwards
    torch.cuda.synchronize()
    assert torch.isfinite(q.float()).all()


def test_default_validation_is_deferred_and_never_syncs(cuda):
    """The default call enqueues and returns like the reference operator: no
    host synchronisation (torch's sync debug mode turns any into an error);
    a bad id is reported by check_status (or a later call) instead."""
    q = torch.randn(2, 64, 64, device=cuda).to(torch.bfloat16)
    kp = torch.randn(2, 128, 64, device=cuda).to(torch.bfloat16)
    ks = torch.randn(2, 5, 64, device=cuda).to(torch.bfloat16)
    heads = torch.tensor([0], device=cuda, dtype=torch.int32)
    good = torch.tensor([[[0, 1]]], device=cuda, dtype=torch.int32)
    bad = torch.tensor([[[0, 7]]], device=cuda, dtype=torch.int32)
    two = torch.tensor([2], device=cuda, dtype=torch.int32)
    vggt_sparse.check_status()  # nothing pending from earlier tests
    torch.cuda.synchronize()
    torch.cuda.set_sync_debug_mode("error")
    try:
        for _ in range(20):
            vggt_sparse.block_attention(q, kp, kp, ks, ks, good, two, heads)
        vggt_sparse.block_attention(q, kp, kp, ks, ks, bad, two, heads)
    finally:
        torch.cuda.set_sync_debug_mode("default")
    with pytest.raises(ValueError, match="block id"):
        vggt_sparse.check_status()
    # reported once; later good calls are clean
    vggt_sparse.block_attention(q, kp, kp, ks, ks, good, two, heads)
    vggt_sparse.check_status()
    # a later call raises for an earlier bad one once its status copy has landed
    vggt_sparse.block_attention(q, kp, kp, ks, ks, bad, two, heads)
    torch.cuda.synchronize()
    with pytest.raises(ValueError, match="earlier call"):
        vggt_sparse.block_attention(q, kp, kp, ks, ks, good, two, heads)
    vggt_sparse.check_status()


def test_torch_ops_registration(cuda):
    x = _layer(cuda)
    q, kp, vp, ks, vs = (getattr(x, k).to(cuda) for k in ("q", "kp", "vp", "ks", "vs"))
    heads = torch.tensor([2, 4], device=cuda, dtype=torch.int32)
    idx, cnt, scores = torch.ops.vggt_sparse.block_mask_estimate(q, kp, heads, 64, 64, "topk", 22,
                                                                 0.0, 0.125, True)
    assert idx.shape == (2, 86, 22) and scores.shape == (2, 86, 86)
    out, ev = torch.ops.vggt_sparse.block_sparse_attn_fwd(q, kp, vp, ks, vs, idx, cnt, heads, None,
                                                          0.125, 64, 64, True)
    exp, exp_ev = oracle.block_sparse_attention(
        x.q.float().numpy(), x.kp.float().numpy(), x.vp.float().numpy(), x.ks.float().numpy(),
        x.vs.float().numpy(), idx.cpu().numpy(), cnt.cpu().numpy(), [2, 4], scale=0.125)
    check_out(out[[2, 4]], exp[[2, 4]])
    finite = np.isfinite(exp_ev)
    np.testing.assert_allclose(ev.cpu().numpy()[finite], exp_ev[finite], rtol=1e-4, atol=1e-4)


def test_cfg2_scale_properties(cuda):
    """Config 2 (32 frames, mass 0.9, heads 0-3 dense) at full size:
    size-independent properties of the masks, and sampled query blocks of the
    output against the oracle."""
    x = clustered_layer(32, centres=128, seed=0, device=cuda)
    layer = vggt_sparse.SparseGlobalLayer(16, mode="mass", tau=0.9, dense_heads=(0, 1, 2, 3))
    out = layer(x.q, x.kp, x.vp, x.ks, x.vs)
    idx, cnt = layer.last_masks
    nb = x.shape.n_blocks
    assert int(cnt.min()) >= 1 and int(cnt.max()) <= nb
    slot = torch.arange(idx.shape[-1], device=cuda)[None, None] < cnt[..., None]
    assert bool(((idx >= 0) == slot).all())
    d = torch.where(slot[..., 1:] & slot[..., :-1], idx[..., 1:] - idx[..., :-1], 1)
    assert bool((d > 0).all())              # ascending and unique
    # re-selecting on exported scores reproduces the masks (determinism)
    res = vggt_sparse.block_mask_estimate(x.q, x.kp, head_ids=layer.sparse_heads, mode="mass",
                                          tau=0.9, export_scores=True)
    assert torch.equal(res.indices, idx) and torch.equal(res.counts, cnt)
    p = torch.softmax(res.scores.double(), -1)
    kept = torch.zeros_like(p).scatter_add_(-1, idx.clamp(min=0).long(), slot.double())
    assert float(kept.max()) <= 1.0
    mass = (p * kept).sum(-1)
    assert float(mass.min()) >= 0.9 - 1e-5
    # every row's ids bit-exact against the oracle's selection on the kernel's
    # fp32 scores, and those scores against the oracle's pooled scores
    scores = res.scores.cpu().numpy()
    exp_idx, exp_cnt = oracle.select_mass(scores, 0.9)
    np.testing.assert_array_equal(cnt.cpu().numpy(), exp_cnt)
    np.testing.assert_array_equal(idx.cpu().numpy(), exp_idx[..., :idx.shape[-1]])
    sel = np.asarray(layer.sparse_heads)
    pq, _ = oracle.block_mean(x.q[sel].float().cpu().numpy(), 64)
    pk, _ = oracle.block_mean(x.kp[sel].float().cpu().numpy(), 64)
    np.testing.assert_allclose(scores, oracle.pooled_scores(pq, pk, 64 ** -0.5), rtol=1e-4,
                               atol=1e-5)
    # sampled query blocks against the oracle
    qbs = [0, 1, 300, x.shape.n_qblocks - 1]
    rows = np.concatenate([np.arange(b * 64, min((b + 1) * 64, x.shape.n_tokens)) for b in qbs])
    sparse = layer.sparse_heads
    exp, _ = oracle.block_sparse_attention(
        x.q.float().cpu().numpy(), x.kp.float().cpu().numpy(), x.vp.float().cpu().numpy(),
        x.ks.float().cpu().numpy(), x.vs.float().cpu().numpy(), idx.cpu().numpy(),
        cnt.cpu().numpy(), sparse, qblocks=qbs)
    got = out.float().cpu().numpy()
    for head in (4, 10, 15):
        check_out(torch.tensor(got[head, rows]), exp[head, rows])
    dense_exp = oracle.dense_attention(x.q.float().cpu().numpy()[:1], x.k.float().cpu().numpy()[:1],
                                       x.v.float().cpu().numpy()[:1], rows=rows[:128])
    check_out(torch.tensor(got[:1, rows[:128]]), dense_exp)


def _sampled_rows_against_oracle(x, out, idx, cnt, slot_heads, dense_heads, qbs):
    """Query blocks ``qbs`` of the given sparse (slot, head) pairs and dense
    heads against the fp64 oracle, one head at a time (full-size layers do not
    fit the oracle whole)."""
    rows = np.concatenate([np.arange(b * 64, min((b + 1) * 64, x.shape.n_tokens)) for b in qbs])
    ks, vs = x.ks.float().cpu().numpy(), x.vs.float().cpu().numpy()
    for slot, head in slot_heads:
        q1 = x.q[head:head + 1].float().cpu().numpy()
        kp1 = x.kp[head:head + 1].float().cpu().numpy()
        vp1 = x.vp[head:head + 1].float().cpu().numpy()
        exp, _ = oracle.block_sparse_attention(
            q1, kp1, vp1, ks[head:head + 1], vs[head:head + 1],
            idx[slot:slot + 1].cpu().numpy(), cnt[slot:slot + 1].cpu().numpy(), [0], qblocks=qbs)
        check_out(out[head, rows], exp[0, rows])
    for head in dense_heads:
        k1 = torch.cat((x.ks[head], x.kp[head])).float().cpu().numpy()[None]
        v1 = torch.cat((x.vs[head], x.vp[head])).float().cpu().numpy()[None]
        exp = oracle.dense_attention(x.q[head:head + 1].float().cpu().numpy(), k1, v1, rows=rows)
        check_out(out[head, rows], exp[0])


def test_cfg4_full_masks_and_sampled_attention(cuda):
    """Config 4 (100 frames, 137,400 tokens, top-k 15 % = 315 of 2,140 key
    blocks, all heads sparse) at full size: every row's ids bit-exact against
    the oracle's top-k on the kernel's fp32 scores, and the first, a middle and
    the last query block of three heads against the fp64 oracle."""
    x = clustered_layer(100, centres=256, seed=0, device=cuda)
    layer = vggt_sparse.SparseGlobalLayer(16, mode="topk", retention=0.15)
    layer.topk = vggt_sparse.topk_budget(0.15, x.shape.n_tokens, x.shape.n_special,
                                         x.shape.n_blocks, 64)
    assert layer.topk == 315
    out = layer(x.q, x.kp, x.vp, x.ks, x.vs)
    idx, cnt = layer.last_masks
    res = vggt_sparse.block_mask_estimate(x.q, x.kp, head_ids=layer.sparse_heads, mode="topk",
                                          topk=315, export_scores=True)
    assert torch.equal(res.indices, idx) and torch.equal(res.counts, cnt)
    assert bool((cnt == 315).all())
    exp = oracle.select_topk(res.scores.cpu().numpy(), 315)
    np.testing.assert_array_equal(idx.cpu().numpy(), exp)
    qbc = x.shape.n_qblocks
    _sampled_rows_against_oracle(x, out, idx, cnt, [(0, 0), (7, 7), (15, 15)], [],
                                 [0, qbc // 2, qbc - 1])


def test_cfg5_sampled_masks_and_attention(cuda):
    """Config 5 (256 frames, 351,744 tokens, mass 0.85 over 5,476 key blocks,
    heads 0-3 dense) at full size on one GPU: sampled rows' ids bit-exact
    against the oracle's mass rule on the kernel's fp32 scores, and the first,
    a middle and the last query block of a sparse and a dense head against the
    fp64 oracle."""
    x = clustered_layer(256, centres=512, seed=0, device=cuda)
    layer = vggt_sparse.SparseGlobalLayer(16, mode="mass", tau=0.85, dense_heads=(0, 1, 2, 3))
    out = layer(x.q, x.kp, x.vp, x.ks, x.vs)
    idx, cnt = layer.last_masks
    qbc = x.shape.n_qblocks
    qbs = [0, qbc // 2, qbc - 1]
    res = vggt_sparse.block_mask_estimate(x.q, x.kp, head_ids=layer.sparse_heads, mode="mass",
                                          tau=0.85, export_scores=True)
    assert torch.equal(res.indices, idx) and torch.equal(res.counts, cnt)
    pick = [0, 1, 2, 1000, qbc // 2, qbc - 2, qbc - 1]
    scores = res.scores[:, pick].cpu().numpy()
    exp_idx, exp_cnt = oracle.select_mass(scores, 0.85)
    np.testing.assert_array_equal(cnt[:, pick].cpu().numpy(), exp_cnt)
    np.testing.assert_array_equal(idx[:, pick].cpu().numpy(), exp_idx[..., :idx.shape[-1]])
    del res
    # slot 0 is head 4 (the first sparse head), slot 11 head 15
    _sampled_rows_against_oracle(x, out, idx, cnt, [(0, 4), (11, 15)], [0], qbs)
