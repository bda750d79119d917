"""Device mask assembly (vggt_block_mask_assemble) and history update
(vggt_history_update) against the reference's own outputs (golden vectors)
and the numpy restatement (ties included)."""
import numpy as np
import pytest
import torch

import vggt_sparse
from conftest import load_golden
from oracle import assembly as oa

pytestmark = pytest.mark.gpu


def test_select_block_mask_matches_reference_golden(cuda):
    g = load_golden("mask_assembly.npz")
    scores = torch.tensor(g["scores"], device=cuda)
    history = torch.tensor(g["history"], device=cuda)
    for i, (count, a, use_h) in enumerate(g["cases"]):
        ids, origin = vggt_sparse.select_block_mask(scores, torch.tensor(g["value_order"]),
                                                    int(count), int(a),
                                                    history if use_h else None)
        np.testing.assert_array_equal(ids.cpu().numpy(), g["ids_%d" % i], err_msg="case %d" % i)
        np.testing.assert_array_equal(origin.cpu().numpy(), g["origin_%d" % i],
                                      err_msg="case %d" % i)


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_batched_assembly_matches_oracle_with_ties(cuda, seed):
    """Integer-valued scores (many ties), several slots with their own count,
    attention count and history (with empty entries)."""
    rng = np.random.default_rng(seed)
    s, qb, nb, hlen = 4, 37, 211, 24
    scores = rng.integers(-6, 7, size=(s, qb, nb)).astype(np.float32)
    value_order = rng.permutation(nb).astype(np.int32)
    counts = np.array([40, 25, 60, 11], np.int32)
    acnt = np.array([16, 25, 0, 5], np.int32)
    history = np.stack([np.stack([rng.permutation(nb)[:hlen] for _ in range(qb)])
                        for _ in range(s)]).astype(np.int32)
    history[rng.random(history.shape) < 0.25] = -1
    ids, origin = vggt_sparse.assemble_masks(torch.tensor(scores, device=cuda), value_order,
                                             counts, acnt, torch.tensor(history, device=cuda),
                                             max_blocks=64)
    ids, origin = ids.cpu().numpy(), origin.cpu().numpy()
    for k in range(s):
        want_ids, want_org = oa.select_block_mask(scores[k], value_order, int(counts[k]),
                                                  int(acnt[k]), history[k])
        c = counts[k]
        np.testing.assert_array_equal(ids[k, :, :c], want_ids, err_msg="slot %d" % k)
        np.testing.assert_array_equal(origin[k, :, :c], want_org, err_msg="slot %d" % k)
        assert (ids[k, :, c:] == -1).all()


def test_wide_rows_match_oracle(cuda):
    """cfg5-wide rows (5,476 key blocks)."""
    rng = np.random.default_rng(4)
    qb, nb = 6, 5476
    scores = (rng.standard_normal((1, qb, nb)) * 3).astype(np.float32)
    value_order = rng.permutation(nb).astype(np.int32)
    history = np.stack([rng.permutation(nb)[:300] for _ in range(qb)])[None].astype(np.int32)
    ids, origin = vggt_sparse.assemble_masks(torch.tensor(scores, device=cuda), value_order,
                                             [900], [400], torch.tensor(history, device=cuda))
    want_ids, want_org = oa.select_block_mask(scores[0], value_order, 900, 400, history[0])
    np.testing.assert_array_equal(ids[0].cpu().numpy(), want_ids)
    np.testing.assert_array_equal(origin[0].cpu().numpy(), want_org)


def test_history_update_matches_reference_and_oracle(cuda):
    g = load_golden("mask_assembly.npz")
    count, keep = int(g["cases"][3][0]), int(g["keep"])
    ev = torch.tensor(g["evidence"], device=cuda)[None].contiguous()
    ids = torch.tensor(g["ids_3"], dtype=torch.int32, device=cuda)[None].contiguous()
    out = vggt_sparse.history_update(ev, ids, [count], [keep])
    np.testing.assert_array_equal(out[0].cpu().numpy(), np.sort(g["new_history"], axis=1))
    # ties and several slots against the oracle
    rng = np.random.default_rng(9)
    s, qb, mb = 3, 20, 48
    evn = rng.integers(0, 5, size=(s, qb, mb)).astype(np.float32)
    idn = np.sort(np.stack([[rng.permutation(500)[:mb] for _ in range(qb)] for _ in range(s)]),
                  axis=-1).astype(np.int32)
    counts, keeps = [48, 30, 12], [10, 30, 3]
    out = vggt_sparse.history_update(torch.tensor(evn, device=cuda), torch.tensor(idn, device=cuda),
                                     counts, keeps, history_len=32).cpu().numpy()
    for k in range(s):
        want = oa.history_update(evn[k], idn[k], counts[k], keeps[k])
        np.testing.assert_array_equal(out[k, :, :keeps[k]], want)
        assert (out[k, :, keeps[k]:] == -1).all()


def test_value_order_out_of_range_sets_status(cuda):
    scores = torch.zeros(1, 2, 10, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    vggt_sparse.assemble_masks(scores, [0, 1, 2, 3, 4, 5, 6, 7, 8, 99], [10], [0], status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & 1
