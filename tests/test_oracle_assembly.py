"""The mask-assembly oracle (select_block_mask with value order and history,
and the same-pass history update) against golden vectors produced by the
reference's own functions (tests/golden/make_golden.py: mask_assembly)."""
import numpy as np

from conftest import load_golden
from oracle import assembly


def test_select_block_mask_matches_reference_every_case():
    g = load_golden("mask_assembly.npz")
    for i, (count, a, use_h) in enumerate(g["cases"]):
        ids, origin = assembly.select_block_mask(g["scores"], g["value_order"], int(count), int(a),
                                                 g["history"] if use_h else None)
        np.testing.assert_array_equal(ids, g["ids_%d" % i], err_msg="case %d" % i)
        np.testing.assert_array_equal(origin, g["origin_%d" % i], err_msg="case %d" % i)


def test_history_update_matches_reference_as_sets():
    g = load_golden("mask_assembly.npz")
    count = int(g["cases"][3][0])
    got = assembly.history_update(g["evidence"], g["ids_3"], count, int(g["keep"]))
    np.testing.assert_array_equal(got, np.sort(g["new_history"], axis=1))


def test_origin_codes_partition_the_slots():
    """Reused blocks are a subset of the attention blocks; attention blocks
    number exactly min(count, A); value-fill blocks make up the rest."""
    g = load_golden("mask_assembly.npz")
    for i, (count, a, use_h) in enumerate(g["cases"]):
        o = g["origin_%d" % i]
        assert ((o == 1) | (o == 2)).sum(1).tolist() == [min(count, a)] * o.shape[0]
        if not use_h or a < 2:
            assert not (o == 1).any()


def test_ties_break_to_the_lower_index():
    scores = np.zeros((1, 10), np.float32)
    ids, origin = assembly.select_block_mask(scores, np.arange(10)[::-1], 4, 2)
    np.testing.assert_array_equal(ids[0], [0, 1, 8, 9])     # top-2 ties -> 0, 1; fill 9, 8
    np.testing.assert_array_equal(origin[0], [2, 2, 0, 0])
