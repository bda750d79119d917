"""Head-profile dispatch: which heads take the dense path of the kernel.

The reference stores a per-layer head profile as JSON
``{layer: [{"mode": ..., "head_ids": [...], ...}, ...]}``
(configs/sparse_attn/vggt/*.json); heads not listed default to ``"full"``,
i.e. dense attention (saf3r/patch/wrapper.py:29-40).  The adaptive policy
marks dense heads per layer with ``decisions[h]['dense_fallback']``
(saf3r/patch/adaptive_block_value.py:340-341).  Both reduce to a boolean
mask over heads; heads with any other mode are served by the block-sparse
path here.
"""
import json

DENSE_MODES = ("full", "dense")


def head_modes_from_profile(profile, layer, num_heads):
    """The mode of each head of ``layer`` ("full" when no group lists it) from
    a profile dict or JSON path, as saf3r/patch/wrapper.py:29-40 assigns
    them; a head listed by two groups raises ValueError.  The profile is not
    modified."""
    if isinstance(profile, str):
        with open(profile) as f:
            profile = json.load(f)
    modes = ["full"] * num_heads
    for group in profile.get(str(layer), profile.get(layer, [])):
        for head in group["head_ids"]:
            if not 0 <= head < num_heads:
                raise ValueError("head id %d out of range" % head)
            if modes[head] != "full":
                raise ValueError("Head %d assigned to multiple patterns!" % head)
            modes[head] = group["mode"]
    return modes


def dense_heads_from_profile(profile, layer, num_heads):
    """Dense head ids of ``layer`` from a profile dict or JSON path."""
    modes = head_modes_from_profile(profile, layer, num_heads)
    return [h for h, m in enumerate(modes) if m in DENSE_MODES]


def dense_heads_from_decisions(decisions):
    """Dense head ids from the adaptive policy's per-head decisions."""
    return [h for h, c in enumerate(decisions) if c["dense_fallback"]]


def split_heads(num_heads, dense_heads):
    """(sparse head ids, dense head ids), each ascending."""
    dense = sorted(set(int(h) for h in dense_heads))
    for h in dense:
        if not 0 <= h < num_heads:
            raise ValueError("dense head %d out of range" % h)
    sparse = [h for h in range(num_heads) if h not in dense]
    return sparse, dense
