"""Per-frame QK top-k on the GPU (vggt_frame_qk_topk) against the oracle and
the reference's recorded Triton outputs.

Small-integer inputs make every fp32 sum exact, so there the indices must
match the oracle exactly, order and tie-breaking included.  On Gaussian
inputs the tensor cores and the oracle round differently, so an entry may
differ only where the two keys' scores are within fp32 rounding."""
import os

import numpy as np
import pytest
import torch

import vggt_sparse
from oracle import qk_topk_per_frame
from test_oracle_frame_topk import GPU_GOLDEN, bf16, cases, near_tie_only

pytestmark = pytest.mark.gpu


def integer_inputs(b, nq, nk, dim, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randint(-2, 3, (b, nq, dim), generator=g).float()
    k = torch.randint(-2, 3, (b, nk, dim), generator=g).float()
    q[:, :, 0] = 1.0
    return q.to(torch.bfloat16), k.to(torch.bfloat16)


def run(q, k, topk, tokens, cuda, **kw):
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = vggt_sparse.compute_qk_topk_indices_fused(q.to(cuda), k.to(cuda), topk,
                                                     num_toks_per_img=tokens, status=status, **kw)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return out.cpu().numpy()


# batch, n_queries, frames, tokens, dim, topk
SHAPES = [
    (1, 130, 3, 50, 64, 4),      # register list, one partial tile per frame
    (2, 128, 2, 128, 64, 8),     # exact tiles, batch 2
    (1, 70, 2, 300, 128, 5),     # head dim 128, three tiles per frame
    (1, 64, 2, 200, 64, 16),     # shared-memory list
    (1, 200, 2, 1369, 64, 4),    # the VGGT frame (37 x 37 patches)
    (1, 20, 3, 6, 64, 10),       # top-k clamped to the frame
    (1, 40, 1, 1000, 64, 128),   # the largest top-k
    (1, 48, 3, 90, 32, 6),       # head dim 32 (zero-padded to 64)
    (1, 33, 4, 129, 96, 9),      # head dim 96 (zero-padded to 128), 9 -> shared list
    (1, 130, 2, 400, 128, 100),  # head dim 128 with a 100-entry heap: a single K stage
]


@pytest.mark.parametrize("b,nq,frames,tokens,dim,topk", SHAPES)
def test_exact_on_integer_inputs(cuda, b, nq, frames, tokens, dim, topk):
    q, k = integer_inputs(b, nq, frames * tokens, dim, seed=nq + tokens + topk)
    want = qk_topk_per_frame(q.float().numpy(), k.float().numpy(), topk, tokens)
    got = run(q, k, topk, tokens, cuda)
    assert got.shape == want.shape
    assert np.array_equal(got, want)


@pytest.mark.parametrize("b,nq,frames,tokens,dim,topk", SHAPES)
def test_gaussian_inputs_match_up_to_rounding(cuda, b, nq, frames, tokens, dim, topk):
    g = torch.Generator().manual_seed(7 * nq + tokens)
    q = torch.randn(b, nq, dim, generator=g).to(torch.bfloat16)
    k = torch.randn(b, frames * tokens, dim, generator=g).to(torch.bfloat16)
    qn, kn = q.float().numpy(), k.float().numpy()
    want = qk_topk_per_frame(qn, kn, topk, tokens)
    got = run(q, k, topk, tokens, cuda)
    assert got.shape == want.shape
    assert near_tie_only(qn, kn, got, want, tokens)
    assert (got == want).mean() > 0.99


def test_frame_groups_do_not_change_the_result(cuda):
    q, k = integer_inputs(1, 300, 5 * 200, 64, seed=3)
    outs = [run(q, k, 4, 200, cuda, groups=g) for g in (0, 1, 2, 5)]
    for o in outs[1:]:
        assert np.array_equal(o, outs[0])


def test_other_input_dtypes_are_taken_as_bf16(cuda):
    q, k = integer_inputs(1, 50, 2 * 70, 64, seed=5)
    a = run(q, k, 4, 70, cuda)
    b = run(q.float(), k.half(), 4, 70, cuda)
    assert np.array_equal(a, b)


@pytest.mark.skipif(not os.path.exists(GPU_GOLDEN), reason="no Triton golden recorded")
def test_matches_reference_triton_outputs(cuda):
    for name, q, k, tokens, topk, want in cases(GPU_GOLDEN):
        got = run(torch.from_numpy(q).to(torch.bfloat16), torch.from_numpy(k).to(torch.bfloat16),
                  topk, tokens, cuda)
        assert got.shape == want.shape, name
        if name == "ties":
            assert np.array_equal(got, want), name
        else:
            assert near_tie_only(q, k, got, want, tokens), name


def test_vggt_layer_size_sampled_rows(cuda):
    """32 frames of 1369 patch tokens, top-4 per frame (the lazy correspondence
    head's call): every row computed, 256 rows checked against the oracle."""
    frames, tokens, dim = 32, 1369, 64
    g = torch.Generator().manual_seed(11)
    q = torch.randn(1, frames * tokens, dim, generator=g).to(torch.bfloat16)
    k = torch.randn(1, frames * tokens, dim, generator=g).to(torch.bfloat16)
    got = run(q, k, 4, tokens, cuda)
    assert got.shape == (1, frames * tokens, frames * 4)
    rows = np.random.default_rng(0).choice(frames * tokens, 256, replace=False)
    qn = q.float().numpy()[:, rows]
    kn = k.float().numpy()
    want = qk_topk_per_frame(qn, kn, 4, tokens)
    assert near_tie_only(qn, kn, got[:, rows], want, tokens)
    # every frame's entries lie in that frame and are distinct
    f = got.reshape(1, -1, frames, 4) // tokens
    assert np.all(f == np.arange(frames)[None, None, :, None])
    s = np.sort(got.reshape(-1, 4), axis=1)
    assert np.all(np.diff(s, axis=1) > 0)
