"""The estimator entry point that allocates nothing (vggt_block_mask_estimate_noalloc).

Callers that cannot allocate device memory (no cudaMalloc allowed where they
run, or memory planned once at start-up) use this variant: the pooled Q/K rows
go to a fixed 8 MiB array inside the library instead of caller scratch.  The
test calls both entry points through the C ABI on the same inputs and expects
identical masks, counts and pooled scores, on two calls in a row with
different shapes and rules (the second call runs over the first call's
leftovers in the shared array).  This file is collected last on purpose.
"""
import ctypes
import math

import pytest
import torch

from vggt_sparse import _lib
from vggt_sparse.synthetic import clustered_layer

pytestmark = pytest.mark.gpu

TOPK, MASS = _lib.SELECT_TOPK, _lib.SELECT_MASS


def _case(dev, frames, heads, seed):
    x = clustered_layer(frames, centres=64, heads=heads, seed=seed, device="cpu",
                        dtype=torch.bfloat16)
    return x.q.to(dev), x.kp.to(dev)


def _outputs(q, kp, slots, max_blocks):
    qbc = math.ceil(q.shape[1] / 64)
    nb = math.ceil(kp.shape[1] / 64)
    idx = torch.full((slots, qbc, max_blocks), -7, device=q.device, dtype=torch.int32)
    cnt = torch.full((slots, qbc), -7, device=q.device, dtype=torch.int32)
    scores = torch.full((slots, qbc, nb), float("nan"), device=q.device, dtype=torch.float32)
    return idx, cnt, scores


def _run(lib, noalloc, q, kp, head_ids, mode, topk, tau, max_blocks):
    h, n, d = q.shape
    slots = head_ids.numel()
    idx, cnt, scores = _outputs(q, kp, slots, max_blocks)
    status = torch.zeros(1, device=q.device, dtype=torch.int32)
    stream = torch.cuda.current_stream().cuda_stream
    common = (q.data_ptr(), kp.data_ptr(), _lib.DTYPE_BF16, h, n, kp.shape[1], d,
              head_ids.data_ptr(), slots, 64, 64, mode, topk, tau, d ** -0.5)
    if noalloc:
        rc = lib.vggt_block_mask_estimate_noalloc(
            *common, idx.data_ptr(), max_blocks, cnt.data_ptr(), scores.data_ptr(),
            status.data_ptr(), stream)
    else:
        qbc, nb = idx.shape[1], scores.shape[2]
        pooled = torch.empty(slots * (qbc + nb) * d, device=q.device, dtype=torch.float32)
        rc = lib.vggt_block_mask_estimate(
            *common, pooled.data_ptr(), pooled[slots * qbc * d:].data_ptr(), idx.data_ptr(),
            max_blocks, cnt.data_ptr(), scores.data_ptr(), status.data_ptr(), stream)
    assert rc == 0, lib.vggt_sparse_last_error().decode()
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return idx, cnt, scores


def test_noalloc_estimator_matches_the_scratch_entry_point_twice(cuda):
    lib = _lib.load()
    # call 1: 4 frames, 16 heads, top-22 (config 1)
    q, kp = _case(cuda, 4, 16, seed=0)
    heads = torch.arange(16, device=cuda, dtype=torch.int32)
    ref = _run(lib, False, q, kp, heads, TOPK, 22, 0.0, 22)
    got = _run(lib, True, q, kp, heads, TOPK, 22, 0.0, 22)
    assert torch.equal(got[0], ref[0]) and torch.equal(got[1], ref[1])
    torch.testing.assert_close(got[2], ref[2], rtol=1e-4, atol=1e-5)
    # call 2: another shape and the mass rule, over call 1's leftovers
    q2, kp2 = _case(cuda, 3, 8, seed=5)
    heads2 = torch.tensor([1, 4, 6], device=cuda, dtype=torch.int32)
    nb2 = math.ceil(kp2.shape[1] / 64)
    ref2 = _run(lib, False, q2, kp2, heads2, MASS, 0, 0.9, nb2)
    got2 = _run(lib, True, q2, kp2, heads2, MASS, 0, 0.9, nb2)
    assert torch.equal(got2[0], ref2[0]) and torch.equal(got2[1], ref2[1])
    torch.testing.assert_close(got2[2], ref2[2], rtol=1e-4, atol=1e-5)


def test_noalloc_estimator_rejects_sizes_beyond_its_scratch(cuda):
    lib = _lib.load()
    # 16 slots x (5496 + 5476 pooled rows) x 64 x 4 B = 45 MB > 8 MiB: refused before any launch
    rc = lib.vggt_block_mask_estimate_noalloc(
        16, 16, _lib.DTYPE_BF16, 16, 351744, 350464, 64, 16, 16, 64, 64, TOPK, 10, 0.0, 0.125, 16,
        10, 16, None, None, None)
    assert rc < 0
    assert "scratch" in lib.vggt_sparse_last_error().decode()
