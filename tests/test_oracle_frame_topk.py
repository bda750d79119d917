"""The per-frame QK top-k oracle against the reference's own outputs.

qk_topk_cpu.npz holds the reference's PyTorch path (torch.topk, unordered:
compared as sets); qk_topk_gpu.npz its Triton kernel on a B200 (ordered,
ties to the lower index: compared entry by entry, exactly on integer inputs,
and up to fp32 rounding of near-tied scores otherwise)."""
import os

import numpy as np
import pytest

from oracle import qk_topk_per_frame, score_keys32
from oracle.frame_topk import frame_scores

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def bf16(bits):
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def cases(path):
    data = np.load(path)
    names = sorted({k[:-4] for k in data.files if k.endswith("_idx")})
    for name in names:
        q = bf16(data[name + "_q_bf16"])
        k = bf16(data[name + "_k_bf16"])
        b, nq, frames, tokens, dim, topk = (int(x) for x in data[name + "_meta"])
        yield name, q, k, tokens, topk, data[name + "_idx"]


def near_tie_only(q, k, got, want, tokens, rel=1e-5):
    """Every differing entry picks a key whose score is within fp32 rounding
    of the score of the key it replaces."""
    s = frame_scores(q, k).astype(np.float64)
    diff = np.argwhere(got != want)
    for bi, r, j in diff:
        a = s[bi, r, got[bi, r, j]]
        c = s[bi, r, want[bi, r, j]]
        scale = max(1.0, np.abs(s[bi, r]).max())
        if abs(a - c) > rel * scale:
            return False
    return True


def test_sortable_key_order():
    vals = np.array([-np.inf, -2.0, -0.0, 0.0, 1e-30, 3.0, np.inf], dtype=np.float32)
    keys = score_keys32(vals)
    assert np.all(np.diff(keys.astype(np.int64)) > 0)  # -0 ranks below +0


def test_ties_go_to_the_lower_index():
    q = np.ones((1, 1, 64), dtype=np.float32)
    k = np.zeros((1, 12, 64), dtype=np.float32)
    k[0, [1, 4, 5, 9], 0] = 2.0  # four equal top scores across two frames of 6
    got = qk_topk_per_frame(q, k, 3, 6)
    assert got.tolist() == [[[1, 4, 5, 9, 6, 7]]]


def test_topk_is_clamped_to_the_frame():
    rng = np.random.default_rng(1)
    q = rng.standard_normal((1, 3, 64)).astype(np.float32)
    k = rng.standard_normal((1, 8, 64)).astype(np.float32)
    got = qk_topk_per_frame(q, k, 10, 4)
    assert got.shape == (1, 3, 8)
    assert sorted(got[0, 0, :4]) == [0, 1, 2, 3] and sorted(got[0, 0, 4:]) == [4, 5, 6, 7]


@pytest.mark.parametrize("name", ["small", "pad", "wide", "dim32", "dim128", "k64", "clamp"])
def test_oracle_matches_reference_cpu_path(name):
    for case, q, k, tokens, topk, want in cases(os.path.join(GOLDEN, "qk_topk_cpu.npz")):
        if case != name:
            continue
        got = qk_topk_per_frame(q, k, topk, tokens)
        assert got.shape == want.shape
        te = min(topk, tokens)
        frames = k.shape[1] // tokens
        g = np.sort(got.reshape(*got.shape[:2], frames, te), axis=-1)
        w = np.sort(want.reshape(*want.shape[:2], frames, te), axis=-1)
        assert np.array_equal(g, w)
        return
    pytest.fail("case %s missing" % name)


GPU_GOLDEN = os.path.join(GOLDEN, "qk_topk_gpu.npz")


@pytest.mark.skipif(not os.path.exists(GPU_GOLDEN), reason="no Triton golden recorded")
def test_oracle_matches_reference_triton_kernel():
    seen = 0
    for name, q, k, tokens, topk, want in cases(GPU_GOLDEN):
        got = qk_topk_per_frame(q, k, topk, tokens)
        assert got.shape == want.shape, name
        if name == "ties":  # small integers: every sum is exact, order included
            assert np.array_equal(got, want), name
        else:
            assert near_tie_only(q, k, got, want, tokens), name
        seen += 1
    assert seen == 8
