"""Golden vectors of the reference's per-frame QK top-k.

saf3r/triton/fused_qk_topk.py:compute_qk_topk_indices_fused answers CPU
tensors with its PyTorch path (_reference_perframe: torch.topk, unordered)
and CUDA tensors with the Triton kernel (ordered, ties to the lower index).
This script records both on seeded bf16 inputs:

    python tests/golden/make_qk_topk_golden.py cpu <dir holding saf3r> <out.npz>
    python tests/golden/make_qk_topk_golden.py gpu <dir holding saf3r> <out.npz>

Inputs are stored as uint16 bf16 bit patterns, outputs as int32.  The
committed tests/golden/qk_topk_cpu.npz and qk_topk_gpu.npz came from it; the
tests only read the .npz files.
"""
import contextlib
import io
import sys

import numpy as np
import torch

# name, batch, n_queries, frames, tokens, dim, topk, integer-valued inputs
CASES = (
    ("small", 1, 40, 3, 50, 64, 4, False),
    ("pad", 2, 70, 2, 100, 64, 8, False),
    ("wide", 1, 33, 2, 300, 64, 16, False),
    ("dim32", 1, 20, 2, 64, 32, 5, False),
    ("dim128", 1, 24, 3, 80, 128, 4, False),
    ("k64", 1, 16, 2, 200, 64, 64, False),
    ("clamp", 1, 12, 3, 6, 64, 10, False),
    ("ties", 1, 48, 3, 90, 64, 6, True),
)


def make_inputs(case, seed):
    name, b, nq, frames, tokens, dim, topk, integer = case
    g = torch.Generator().manual_seed(seed)
    if integer:
        q = torch.randint(-2, 3, (b, nq, dim), generator=g).float()
        k = torch.randint(-2, 3, (b, frames * tokens, dim), generator=g).float()
        q[:, :, 0] = 1.0  # no all-zero rows
    else:
        q = torch.randn(b, nq, dim, generator=g)
        k = torch.randn(b, frames * tokens, dim, generator=g)
    return q.to(torch.bfloat16), k.to(torch.bfloat16)


def main(mode, ref_dir, out_path):
    sys.path.insert(0, ref_dir)
    from saf3r.triton.fused_qk_topk import compute_qk_topk_indices_fused
    dev = torch.device("cuda:0") if mode == "gpu" else torch.device("cpu")
    out = {}
    for i, case in enumerate(CASES):
        name, b, nq, frames, tokens, dim, topk, integer = case
        if mode == "cpu" and integer:
            continue  # torch.topk leaves the choice among tied keys open
        q, k = make_inputs(case, 100 + i)
        with contextlib.redirect_stdout(io.StringIO()):  # the reference prints a timing line
            idx = compute_qk_topk_indices_fused(q.to(dev), k.to(dev), topk, num_toks_per_img=tokens)
        if dev.type == "cuda":
            torch.cuda.synchronize()
        out["%s_q_bf16" % name] = q.view(torch.int16).numpy().view(np.uint16)
        out["%s_k_bf16" % name] = k.view(torch.int16).numpy().view(np.uint16)
        out["%s_meta" % name] = np.array([b, nq, frames, tokens, dim, topk], dtype=np.int64)
        out["%s_idx" % name] = idx.cpu().numpy().astype(np.int32)
    np.savez_compressed(out_path, **out)
    print("wrote", out_path, "cases:", sorted({k.rsplit("_", 1)[0] for k in out if k.endswith("_idx")}))


if __name__ == "__main__":
    main(sys.argv[1], sys.argv[2], sys.argv[3])
