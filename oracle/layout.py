"""Token layout restatement (oracle; test infrastructure only)."""
import numpy as np


def token_layout(frames, patches_per_frame, special_per_frame=5):
    """Frame-major split of token ids into (patch ids, special ids).

    Restates saf3r/patch/value_evolving_attention.py:17-20: token t is special
    when ``t mod (P + S) < S``; every frame starts with its S special tokens
    (1 camera + 4 register tokens in VGGT, models/aggregator.py:128-132).
    """
    per = patches_per_frame + special_per_frame
    ids = np.arange(frames * per, dtype=np.int64)
    special = (ids % per) < special_per_frame
    return ids[~special], ids[special]
