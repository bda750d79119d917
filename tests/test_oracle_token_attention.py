"""The per-token attention oracle against the reference's own Triton kernels'
outputs (tests/golden/make_token_golden.py ran fused_sparse_topk_attention
and fused_sparse_topk_attention_2 on a GPU; their bf16 outputs are the golden
values).  Tolerance: the bf16 rounding of the reference's outputs."""
import numpy as np
import torch

from conftest import load_golden
from oracle import token_attention


def test_oracle_matches_reference_kernels():
    g = load_golden("token_attention.npz")
    for name in ("small", "wide"):
        q, k, v = (torch.from_numpy(g["%s_%s_bf16" % (name, t)].view(np.int16))
                   .view(torch.bfloat16).float().numpy() for t in ("q", "k", "v"))
        got = token_attention.token_sparse_attention(q, k, v, g[name + "_idx"])
        want = g[name + "_out"]
        np.testing.assert_allclose(got, want, rtol=1e-2, atol=4e-3, err_msg=name)
