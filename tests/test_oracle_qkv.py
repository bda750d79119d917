"""The QKV-projection oracle (oracle/qkv.py) against the reference's own
attention module run with CUDA bf16 autocast's casts
(tests/golden/make_qkv_golden.py)."""
import numpy as np
import torch

import oracle
from conftest import load_golden


def bf16(a):
    """float32 values of int16 bf16 bit patterns"""
    return torch.from_numpy(np.asarray(a)).view(torch.bfloat16).float().numpy()


def golden_inputs(g):
    return dict(x=bf16(g["x"]), w=bf16(g["w"]), b=bf16(g["b"]), heads=g["w"].shape[1] // 64,
                tokens_per_frame=int(g["tokens_per_frame"]),
                special_per_frame=int(g["special_per_frame"]), qn=(g["qn_w"], g["qn_b"]),
                kn=(g["kn_w"], g["kn_b"]), eps=float(g["ln_eps"]), pos=g["pos"])


def test_qkv_oracle_matches_reference_module():
    g = load_golden("qkv.npz")
    got = oracle.project_qkv(**golden_inputs(g))
    names = ("q", "k_patch", "v_patch", "k_special", "v_special")
    for name, a in zip(names, got[:5]):
        want = bf16(g[name])
        assert a.shape == want.shape, name
        # bf16 outputs: equal but for an occasional 1-ulp rounding difference
        # (the reference's bf16 matmul accumulates in its own order)
        diff = np.abs(a - want)
        ulp = np.maximum(np.abs(want), 1e-3) * 2.0 ** -7
        assert (diff <= 2 * ulp + 1e-6).all(), (name, float(diff.max()))
        assert (diff > 0).mean() < 1e-3, (name, float((diff > 0).mean()))
    np.testing.assert_allclose(got[5], g["pooled_q"], rtol=2e-3, atol=2e-3)
    np.testing.assert_allclose(got[6], g["pooled_k"], rtol=2e-3, atol=2e-3)
    # the means are block_mean of the bf16 outputs
    np.testing.assert_allclose(got[5], oracle.block_mean(got[0], 64)[0], rtol=1e-6)
