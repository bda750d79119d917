"""Golden vectors for the softmax-mass selection rule on realistic rows.

Run in a container where the reference checkout exists:

    python tests/golden/make_mass_golden.py /path/to/Sparse-Attention-VGGT

Pooled block scores are built the way the estimator builds them (64-row block
means of the seeded clustered Q and patch K of vggt_sparse.synthetic, fp32
scores Q_mean . K_mean * d^-1/2) at the shapes of the 32-frame layer (685 key
blocks, tau 0.9) and the 256-frame layer (5,476 key blocks, tau 0.85).  The
reference's own rule then runs on them: torch.softmax in fp32 followed by
saf3r/patch/region_history_attention.py:39-42 ``concentration``, from whose
output the kept count m = (1 - concentration) * n_blocks is recovered.

Writes mass_rows.npz:
  cfg2_scores [R, 685] fp32,  cfg2_m [R] int  (tau 0.9)
  cfg5_scores [R, 5476] fp32, cfg5_m [R] int  (tau 0.85)
  and the same scores' reference counts at the other tau (cfg2_m85, cfg5_m90)
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.join(REPO, "sparse-attention-vggt_b200"))
sys.path.insert(0, REPO)


def score_rows(frames, centres, heads, rows_per_head, seed):
    """fp32 pooled-score rows of `rows_per_head` query blocks spread over the
    layer, for each of `heads` heads."""
    import oracle
    from vggt_sparse.synthetic import clustered_layer
    x = clustered_layer(frames, centres=centres, heads=heads, seed=seed, device="cpu",
                        dtype=torch.bfloat16, keep_full=False)
    q = x.q.float().numpy()
    kp = x.kp.float().numpy()
    qbc = x.shape.n_qblocks
    pick = np.unique(np.linspace(0, qbc - 1, rows_per_head).round().astype(np.int64))
    out = []
    for h in range(heads):
        pq, _ = oracle.block_mean(q[h:h + 1, :], 64)
        pk, _ = oracle.block_mean(kp[h:h + 1], 64)
        s = oracle.pooled_scores(pq[:, pick], pk, 64 ** -0.5)
        out.append(s[0])
    return np.concatenate(out, 0).astype(np.float32)


def reference_counts(concentration, scores, tau):
    p = torch.softmax(torch.from_numpy(scores), dim=-1)
    conc = concentration(p, tau)
    nb = scores.shape[1]
    return np.rint((1.0 - conc.double().numpy()) * nb).astype(np.int64)


def main(ref_path):
    from make_golden import _import_reference
    _, _, concentration, _, _ = _import_reference(ref_path)
    out = {}
    for name, frames, centres, heads, rows, seed in (("cfg2", 32, 128, 4, 40, 11),
                                                     ("cfg5", 256, 512, 2, 24, 12)):
        s = score_rows(frames, centres, heads, rows, seed)
        out["%s_scores" % name] = s
        out["%s_m90" % name] = reference_counts(concentration, s, 0.9)
        out["%s_m85" % name] = reference_counts(concentration, s, 0.85)
        print(name, s.shape, "mean kept (0.9):", out["%s_m90" % name].mean())
    np.savez_compressed(os.path.join(HERE, "mass_rows.npz"), **out)


if __name__ == "__main__":
    main(sys.argv[1])
