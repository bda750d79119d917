"""Golden head modes of the reference's shipped head profile.

Run in a container where the reference checkout exists:

    python tests/golden/make_profile_golden.py /path/to/Sparse-Attention-VGGT

head_profile_eth3d.json is an unmodified copy of the reference's
configs/sparse_attn/vggt/eth3d-train-fltr-calib_cmpmse.json (the per-layer
head profile its VGGT patch loads, saf3r/patch/patch_vggt.py:179-221).  For
every layer this script builds the reference's own
BaseHeadwiseSparseAttentionWrapper with that layer's group list
(saf3r/patch/wrapper.py:29-40: heads default to "full", each head may be
claimed by one group only) and records the mode it assigns to each of the 16
heads.  Writes head_profile.npz: layers [L] int, modes [L, 16] str.
"""
import copy
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)


def main(ref_path):
    from make_golden import _import_reference
    _import_reference(ref_path)
    from saf3r.patch.wrapper import BaseHeadwiseSparseAttentionWrapper
    with open(os.path.join(HERE, "head_profile_eth3d.json")) as f:
        profile = json.load(f)
    layers = sorted(int(k) for k in profile)
    modes = []
    for layer in layers:
        # the wrapper pops head_ids from the groups it is given
        w = BaseHeadwiseSparseAttentionWrapper(torch.nn.Identity(), 5, 16,
                                               config=copy.deepcopy(profile[str(layer)]))
        modes.append([c["mode"] for c in w.head_cfg])
    np.savez_compressed(os.path.join(HERE, "head_profile.npz"), layers=np.array(layers),
                        modes=np.array(modes))
    print(len(layers), "layers;", sum(m == "full" for row in modes for m in row), "full heads")


if __name__ == "__main__":
    main(sys.argv[1])
