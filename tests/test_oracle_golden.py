"""Pin the CPU oracle against golden vectors produced by the reference's own
functions (tests/golden/make_golden.py).  CPU only."""
import math

import numpy as np
import pytest

import oracle
from oracle import estimator as est
from conftest import load_golden


@pytest.mark.parametrize("block", [32, 64, 128])
def test_block_mean_matches_reference(block):
    g = load_golden("block_mean.npz")
    mean, pop = oracle.block_mean(g["x"], block)
    np.testing.assert_array_equal(pop, g["pop_%d" % block])
    np.testing.assert_allclose(mean, g["mean_%d" % block], rtol=1e-6, atol=1e-7)


def test_token_layout_matches_reference():
    g = load_golden("token_layout.npz")
    for frames, ppf in ((3, 10), (4, 1369)):
        p, s = oracle.token_layout(frames, ppf, 5)
        np.testing.assert_array_equal(p, g["patch_%d_%d" % (frames, ppf)])
        np.testing.assert_array_equal(s, g["special_%d_%d" % (frames, ppf)])


def test_pooled_scores_match_reference_relevance_logits():
    g = load_golden("relevance.npz")
    s = oracle.pooled_scores(g["q"], g["pooled"], float(g["scale"]))
    np.testing.assert_allclose(s, g["logits"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("k", [1, 5, 13, 40])
def test_topk_matches_reference_on_tie_free_scores(k):
    g = load_golden("select_topk.npz")
    ids = oracle.select_topk(g["scores"], k)
    np.testing.assert_array_equal(ids, g["ids_%d" % k])


@pytest.mark.parametrize("k", [1, 5, 13, 40])
def test_topk_with_ties_keeps_the_same_score_multiset_and_lower_ids(k):
    """With ties the reference's torch.topk may pick any tied id; the oracle
    picks the lowest.  Both must keep the same multiset of scores, and among
    boundary ties the oracle's choice must be the lowest ids."""
    g = load_golden("select_topk.npz")
    tied = g["tied"]
    ours = oracle.select_topk(tied, k)
    ref = g["tied_ids_%d" % k]
    for h in range(tied.shape[0]):
        for r in range(tied.shape[1]):
            row = tied[h, r]
            assert sorted(row[ours[h, r]]) == sorted(row[ref[h, r]])
            assert len(set(ours[h, r].tolist())) == min(k, row.size)
            kth = np.sort(row)[::-1][min(k, row.size) - 1]
            boundary = np.flatnonzero(row == kth)
            taken = [i for i in ours[h, r] if row[i] == kth]
            assert taken == sorted(boundary.tolist())[:len(taken)]


def test_concentration_known_answer():
    """tests/test_region_history_attention.py:53 known answer [0, .75]."""
    g = load_golden("concentration.npz")
    p = g["known_probs"]
    ids, counts = oracle.select_mass(np.log(p), 0.8)
    conc = 1.0 - counts / p.shape[1]
    np.testing.assert_allclose(conc, g["known_conc"])
    np.testing.assert_allclose(conc, [0.0, 0.75])


@pytest.mark.parametrize("tau", [0.5, 0.8, 0.85, 0.9])
def test_mass_rule_matches_reference_concentration(tau):
    """Counts agree with the reference's fp32 rule except where the float64
    cumulative mass is within fp32 rounding of tau at the boundary."""
    g = load_golden("concentration.npz")
    logits = g["logits"]
    _, counts = oracle.select_mass(logits, tau)
    ref_m = g["m_%g" % tau]
    probs = g["probs"].astype(np.float64)
    cum = np.cumsum(np.sort(probs, 1)[:, ::-1], 1)
    mismatches = 0
    for r in range(logits.shape[0]):
        if counts[r] != ref_m[r]:
            lo = min(counts[r], ref_m[r]) - 1
            assert abs(cum[r, lo] - tau) < 1e-5, (r, counts[r], ref_m[r], cum[r, lo])
            mismatches += 1
    assert mismatches <= 1


def test_mass_selection_keeps_highest_blocks_and_reaches_tau():
    rng = np.random.default_rng(0)
    s = (rng.standard_normal((50, 97)) * 2).astype(np.float32)
    ids, counts = oracle.select_mass(s, 0.9)
    for r in range(s.shape[0]):
        m = counts[r]
        chosen = ids[r, :m]
        assert np.all(ids[r, m:] == -1)
        assert np.all(np.diff(chosen) > 0)
        p = np.exp(s[r].astype(np.float64) - s[r].max())
        p /= p.sum()
        assert p[chosen].sum() >= 0.9 - 1e-6
        # dropping the lowest kept block must fall below tau
        if m > 1:
            low = chosen[np.argmin(s[r, chosen])]
            assert p[chosen].sum() - p[low] < 0.9 + 1e-6
        # every unchosen block scores no higher than every chosen one
        rest = np.setdiff1d(np.arange(s.shape[1]), chosen)
        if rest.size:
            assert s[r, rest].max() <= s[r, chosen].min()


def test_mass_weights_are_exact_powers_at_integers():
    """2^n for integer log2 offsets is exact, and the maximum weighs 2^40."""
    row = np.array([0.0, -math.log(2.0), -2 * math.log(2.0)], dtype=np.float32)
    w = est.mass_weights(row, np.float32(0.0))
    assert w[0] == 2 ** 40
    assert abs(int(w[1]) - 2 ** 39) <= 2 ** 39 * 1e-6
    assert abs(int(w[2]) - 2 ** 38) <= 2 ** 38 * 1e-6


def test_mass_weight_polynomial_accuracy():
    x = np.linspace(-30, 0, 10001).astype(np.float32)
    w = est.mass_weights(x, np.float32(0.0)).astype(np.float64) / 2 ** 40
    ref = np.exp(x.astype(np.float64))
    # relative error from the fp32 range reduction grows with |x|; the 2^-40
    # quantum bounds the absolute error of tiny weights
    assert np.all(np.abs(w - ref) <= 4e-6 * ref + 2.0 ** -40)


def test_topk_budget_rule():
    # adaptive_block_value.py:187 at the benchmark configs
    assert est.topk_budget(0.25, 5496, 20, 86, 64) == 22
    assert est.topk_budget(0.25, 21984, 80, 344, 64) == 85
    assert est.topk_budget(0.15, 137400, 500, 2140, 64) == 315


@pytest.mark.parametrize("case", ["d64_bq64_bk64", "d32_bq32_bk128", "d64_bq32_bk32",
                                  "d32_bq64_bk64"])
def test_attention_oracle_matches_reference_formula(case):
    g = load_golden("attention_%s.npz" % case)
    bq, bk = (int(x[2:]) for x in case.split("_")[1:])
    out, ev = oracle.block_sparse_attention(g["q"], g["kp"], g["vp"], g["ks"], g["vs"], g["masks"],
                                            g["counts"], g["heads"], query_block=bq,
                                            key_block=bk, scale=float(g["scale"]))
    for head in g["heads"]:
        np.testing.assert_allclose(out[head], g["out"][head], rtol=1e-5, atol=1e-5)
    finite = np.isfinite(g["evidence"])
    np.testing.assert_array_equal(finite, np.isfinite(ev))
    np.testing.assert_allclose(ev[finite], g["evidence"][finite], rtol=1e-5, atol=1e-5)


def test_attention_oracle_matches_reference_cpu_layer_path():
    """The reference's own CPU kernel branch (adaptive_block_value.py:371-385),
    captured from AdaptiveBlockValueAttention.forward."""
    g = load_golden("layer_cpu.npz")
    q, k, v = g["q"], g["k"], g["v"]
    kp, vp = k[:, g["patches"]], v[:, g["patches"]]
    ks, vs = k[:, g["specials"]], v[:, g["specials"]]
    masks = g["masks"]
    heads = list(range(q.shape[0]))
    counts = np.full(len(heads), masks.shape[-1], dtype=np.int32)
    block = int(g["block"])
    out, _ = oracle.block_sparse_attention(q, kp, vp, ks, vs, masks, counts, heads,
                                           query_block=block, key_block=block,
                                           scale=float(g["scale"]))
    np.testing.assert_allclose(out, g["out"], rtol=1e-5, atol=1e-5)


def test_reference_layer_masks_are_topk_of_its_routing():
    """The captured masks are the top-k (ascending) of the reference routing
    scores: the oracle's selection reproduces them."""
    g = load_golden("layer_cpu.npz")
    for head in range(g["masks"].shape[0]):
        ours = oracle.select_topk(g["routing"][head], g["masks"].shape[-1])
        np.testing.assert_array_equal(ours, g["masks"][head])


def _boundary_mismatches(scores, counts, ref_m, tau):
    """Rows whose kept count differs from the reference's fp32 rule, and the
    largest distance from tau of the float64 cumulative mass at the boundary
    of each such row (the rule is m = #(cumsum < tau) + 1)."""
    x = scores.astype(np.float64)
    p = np.exp(x - x.max(1, keepdims=True))
    p /= p.sum(1, keepdims=True)
    cum = np.cumsum(np.sort(p, 1)[:, ::-1], 1)
    rows, worst = [], 0.0
    for r in range(scores.shape[0]):
        if counts[r] != ref_m[r]:
            lo, hi = sorted((int(counts[r]), int(ref_m[r])))
            # every cumulative mass between the two counts sits at tau
            gap = np.abs(cum[r, lo - 1:hi - 1] - tau).max()
            rows.append(r)
            worst = max(worst, gap)
    return rows, worst


@pytest.mark.parametrize("cfg,tau", [("cfg2", 0.9), ("cfg2", 0.85), ("cfg5", 0.85),
                                     ("cfg5", 0.9)])
def test_mass_rule_on_layer_sized_rows(cfg, tau):
    """Pooled-score rows of the 32- and 256-frame layers (685 and 5,476 key
    blocks; tests/golden/make_mass_golden.py): the oracle's quantised mass rule
    keeps the same count as the reference's fp32 softmax + concentration
    except on rows whose cumulative mass at the boundary lies within fp32
    rounding of tau (a few ulps of a sum of thousands of fp32 terms)."""
    g = load_golden("mass_rows.npz")
    scores = g["%s_scores" % cfg]
    ref_m = g["%s_m%d" % (cfg, round(tau * 100))]
    _, counts = oracle.select_mass(scores, tau)
    rows, worst = _boundary_mismatches(scores, counts, ref_m, tau)
    assert worst < 2e-6, (rows, worst)
    assert len(rows) <= max(1, scores.shape[0] // 20), rows
