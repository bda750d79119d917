"""Golden vectors of the reference's per-token sparse attention.

The reference implements it only as Triton kernels
(saf3r/triton/sparse_topk_attention.py: fused_sparse_topk_attention for
top-k <= 2048 and fused_sparse_topk_attention_2 above), so this script runs
on a GPU with the reference package importable:

    python tests/golden/make_token_golden.py <dir holding the saf3r package> <out.npz>

It writes seeded bf16 inputs (as uint16 bit patterns) and the reference's
outputs (fp32 holding its bf16 values); the committed
tests/golden/token_attention.npz came from it.  Tests only read the .npz.
"""
import sys

import numpy as np
import torch


def main(ref_dir, out_path):
    sys.path.insert(0, ref_dir)
    from saf3r.triton.sparse_topk_attention import (fused_sparse_topk_attention,
                                                    fused_sparse_topk_attention_2)
    dev = torch.device("cuda:0")
    g = torch.Generator().manual_seed(2024)
    out = {}
    for name, n, nk, topk, fn in (("small", 64, 500, 48, fused_sparse_topk_attention),
                                  ("wide", 32, 4000, 2600, fused_sparse_topk_attention_2)):
        q = torch.randn(n, 64, generator=g).to(torch.bfloat16)
        k = torch.randn(nk, 64, generator=g).to(torch.bfloat16)
        v = torch.randn(nk, 64, generator=g).to(torch.bfloat16)
        idx = torch.randint(0, nk, (n, topk), generator=g, dtype=torch.int32)
        res = fn(q.to(dev), k.to(dev), v.to(dev), idx.to(dev))
        torch.cuda.synchronize()
        for key, t in (("q", q), ("k", k), ("v", v)):   # bf16 bit patterns
            out["%s_%s_bf16" % (name, key)] = t.view(torch.int16).numpy().view(np.uint16)
        out["%s_idx" % name] = idx.numpy()
        out["%s_out" % name] = res.float().cpu().numpy()
    np.savez_compressed(out_path, **out)
    print("wrote", out_path)


if __name__ == "__main__":
    main(sys.argv[1], sys.argv[2])
