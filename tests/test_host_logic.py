"""Host-side logic: layout, head profiles, budgets, configs, synthetic data."""
import json
import os
import math

import numpy as np
import pytest
import torch

import oracle
import vggt_sparse
from vggt_sparse import profile as prof
from vggt_sparse.configs import CONFIGS
from vggt_sparse.layout import LayerShape, token_layout
from vggt_sparse.synthetic import clustered_layer


def test_token_layout_matches_oracle():
    p, s = token_layout(4, 1369, 5)
    op, os_ = oracle.token_layout(4, 1369, 5)
    np.testing.assert_array_equal(p.numpy(), op)
    np.testing.assert_array_equal(s.numpy(), os_)


@pytest.mark.parametrize("name,n,ns,qb,nb", [
    ("cfg1", 5496, 20, 86, 86), ("cfg2", 43968, 160, 687, 685), ("cfg3", 21984, 80, 344, 343),
    ("cfg4", 137400, 500, 2147, 2140), ("cfg5", 351744, 1280, 5496, 5476)])
def test_config_shapes(name, n, ns, qb, nb):
    shape = LayerShape(frames=CONFIGS[name].frames)
    assert (shape.n_tokens, shape.n_special, shape.n_qblocks, shape.n_blocks) == (n, ns, qb, nb)


def test_topk_budget_matches_oracle_rule():
    for rho, frames in ((0.25, 4), (0.25, 16), (0.15, 100), (0.1, 128)):
        s = LayerShape(frames=frames)
        assert vggt_sparse.topk_budget(rho, s.n_tokens, s.n_special, s.n_blocks, 64) == \
            oracle.topk_budget(rho, s.n_tokens, s.n_special, s.n_blocks, 64)


def test_head_profile_defaults_to_full(tmp_path):
    profile = {"0": [{"mode": "stride", "head_ids": [1, 2]},
                     {"mode": "dino_topk", "head_ids": [5]}],
               "1": [{"mode": "full", "head_ids": [3]}]}
    path = tmp_path / "p.json"
    path.write_text(json.dumps(profile))
    dense0 = prof.dense_heads_from_profile(str(path), 0, 8)
    assert dense0 == [0, 3, 4, 6, 7]
    assert prof.dense_heads_from_profile(profile, 1, 4) == [0, 1, 2, 3]
    assert prof.dense_heads_from_profile(profile, 7, 3) == [0, 1, 2]


def test_head_profile_rejects_double_assignment():
    bad = {"0": [{"mode": "stride", "head_ids": [1]}, {"mode": "stride", "head_ids": [1]}]}
    with pytest.raises(ValueError, match="multiple"):
        prof.dense_heads_from_profile(bad, 0, 4)


def test_split_heads_and_decisions():
    assert prof.split_heads(6, [4, 0]) == ([1, 2, 3, 5], [0, 4])
    dec = [dict(dense_fallback=b) for b in (False, True, False)]
    assert prof.dense_heads_from_decisions(dec) == [1]
    with pytest.raises(ValueError):
        prof.split_heads(4, [4])


def test_synthetic_generator_is_seeded_and_scaled():
    a = clustered_layer(2, centres=16, heads=2, dim=32, patch_h=8, patch_w=8, seed=3,
                        dtype=torch.float32)
    b = clustered_layer(2, centres=16, heads=2, dim=32, patch_h=8, patch_w=8, seed=3,
                        dtype=torch.float32)
    assert torch.equal(a.q, b.q) and torch.equal(a.kp, b.kp)
    n = a.shape.n_tokens
    assert a.q.shape == (2, n, 32) and a.kp.shape == (2, n - 10, 32) and a.ks.shape == (2, 10, 32)
    logits = torch.einsum("hnd,hmd->hnm", a.q, a.k) / math.sqrt(32)
    assert 2.0 < float(logits.std()) < 4.5
    # specials are the first 5 tokens of each frame
    torch.testing.assert_close(a.ks[:, :5], a.k[:, :5])


def test_layer_flop_count_formula():
    layer = vggt_sparse.SparseGlobalLayer(2, mode="topk", topk=1, dense_heads=(1,))
    idx = torch.tensor([[[0], [1]]], dtype=torch.int32)
    cnt = torch.tensor([[1, 1]], dtype=torch.int32)
    layer.last_masks = (idx, cnt)
    # n=100 -> q rows 64 + 36; npatch=90 -> blocks 64 + 26 cols; 10 specials
    flops = layer.kept_flops(100, 90, 10, 8)
    expect = 4 * 8 * (64 * (64 + 10) + 36 * (26 + 10)) + 4 * 8 * 100 * 100
    assert flops == expect


def test_head_profile_parser_on_the_reference_profile():
    """The reference's shipped VGGT profile (an unmodified copy,
    tests/golden/head_profile_eth3d.json): per layer, the parser assigns every
    head the mode the reference's own wrapper assigns
    (tests/golden/make_profile_golden.py), and leaves the profile unchanged."""
    import copy
    from conftest import GOLDEN
    path = os.path.join(GOLDEN, "head_profile_eth3d.json")
    g = np.load(os.path.join(GOLDEN, "head_profile.npz"))
    with open(path) as f:
        profile = json.load(f)
    before = copy.deepcopy(profile)
    assert len(g["layers"]) == 24
    for layer, want in zip(g["layers"], g["modes"]):
        assert prof.head_modes_from_profile(profile, int(layer), 16) == list(want)
        assert prof.head_modes_from_profile(path, int(layer), 16) == list(want)
        dense = prof.dense_heads_from_profile(profile, int(layer), 16)
        assert dense == [h for h, m in enumerate(want) if m == "full"]
    assert profile == before
