"""Failure detection on the GPU: every pipeline wait in the tcgen05 attention
kernel is bounded.  The self-test switch makes each CTA's MMA issuer wait on
a barrier that nothing completes; with a 2 ms limit every CTA gives up, the
launch reports VGGT_STATUS_TIMEOUT (raised as ValueError by the validating
drop-in), and the context stays usable: the next launch is correct.  Nothing
faults, traps or hangs; the wait that runs out is an ordinary bounded wait."""
import numpy as np
import pytest
import torch

import oracle
import vggt_sparse
from vggt_sparse import _lib
from vggt_sparse.synthetic import clustered_layer

pytestmark = pytest.mark.gpu


def _case(cuda):
    x = clustered_layer(2, centres=32, heads=2, seed=3, device=cuda)
    heads = torch.tensor([0, 1], device=cuda, dtype=torch.int32)
    res = vggt_sparse.block_mask_estimate(x.q, x.kp, head_ids=heads, mode="topk", topk=8)
    return x, heads, res.indices, res.counts


@pytest.mark.parametrize("paired", [False, True])
def test_wait_timeout_sets_status_and_context_stays_usable(cuda, paired):
    x, heads, idx, cnt = _case(cuda)
    args = (x.q, x.kp, x.vp, x.ks, x.vs, idx, cnt, heads)
    out = torch.zeros_like(x.q)
    prev_limit = _lib.set_wait_limit_ns(2_000_000)
    prev_test = _lib.set_wait_selftest(True)
    try:
        status = torch.zeros(1, device=cuda, dtype=torch.int32)
        vggt_sparse.ops.launch_block_attention(*args, out=out, status=status, kernel="tcgen05",
                                               pair_qblocks=paired)
        torch.cuda.synchronize()
        assert int(status.item()) & _lib.STATUS_TIMEOUT
        with pytest.raises(ValueError, match="timed out"):
            vggt_sparse.block_attention(*args, kernel="tcgen05", validate=True)
    finally:
        _lib.set_wait_selftest(prev_test)
        _lib.set_wait_limit_ns(prev_limit)
    # the context survived: the same call now completes and matches the oracle
    got, _ = vggt_sparse.block_attention(*args, kernel="tcgen05", validate=True)
    exp, _ = oracle.block_sparse_attention(
        x.q.float().cpu().numpy(), x.kp.float().cpu().numpy(), x.vp.float().cpu().numpy(),
        x.ks.float().cpu().numpy(), x.vs.float().cpu().numpy(), idx.cpu().numpy(),
        cnt.cpu().numpy(), [0, 1])
    a = got.float().cpu().numpy()
    assert np.abs(a - exp).max() <= 2e-2
