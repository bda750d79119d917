"""The drop-in at the reference's own call site: the reference's VGGT
aggregator (random init) with its adaptive block attention, run once with
the reference's Triton block_attention and once with vggt_sparse's assigned
in its place (the module-attribute patch of the integration notes).  Needs
the reference package installed in baseline/_ref."""
import os

import pytest
import torch

import vggt_sparse
from conftest import REPO
from vggt_sparse.synthetic import homography_views

pytestmark = pytest.mark.gpu

REF = os.path.join(REPO, "baseline", "_ref", "saf3r")


@pytest.mark.skipif(not os.path.isdir(REF), reason="reference not installed in baseline/_ref")
def test_reference_aggregator_runs_on_the_drop_in(cuda):
    import bench
    model, state, ref_op = bench.build_reference_aggregator(cuda)
    images = homography_views(4, 518, seed=5, device=cuda)
    triton_op = ref_op.block_attention
    calls = [0]

    def ours(*a, **k):
        calls[0] += 1
        return vggt_sparse.block_attention(*a, **k)

    try:
        want = bench.aggregator_forward(model, images)[-1].float()
        ref_blocks = [[d["blocks"] for d in r["decisions"]] for r in state.records]
        ref_op.block_attention = ours
        got = bench.aggregator_forward(model, images)[-1].float()
        our_blocks = [[d["blocks"] for d in r["decisions"]] for r in state.records]
    finally:
        ref_op.block_attention = triton_op
    assert calls[0] == 24  # every global layer went through the drop-in
    assert our_blocks == ref_blocks
    assert torch.isfinite(got).all()
    diff = (got - want).abs()
    assert (diff.mean() / want.abs().mean()).item() < 1e-2
