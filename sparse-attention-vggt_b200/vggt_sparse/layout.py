"""Frame-major token layout of VGGT global attention.

Every frame contributes 1 camera + 4 register tokens followed by its
patch_h x patch_w patch tokens (saf3r/models/official_vggt/models/aggregator.py:128-132);
the global blocks see all frames concatenated.  ``token_layout`` restates
saf3r/patch/value_evolving_attention.py:17-20.
"""
import math
from dataclasses import dataclass

import torch

SPECIAL_PER_FRAME = 5


def token_layout(frames, patches_per_frame, special_per_frame=SPECIAL_PER_FRAME, device=None):
    """(patch ids, special ids) as int64 tensors, frame-major."""
    per = patches_per_frame + special_per_frame
    ids = torch.arange(frames * per, device=device)
    special = ids.remainder(per) < special_per_frame
    return ids[~special], ids[special]


@dataclass(frozen=True)
class LayerShape:
    """Sizes of one global-attention layer."""
    frames: int
    patch_h: int = 37
    patch_w: int = 37
    heads: int = 16
    dim: int = 64
    special_per_frame: int = SPECIAL_PER_FRAME
    block: int = 64

    @property
    def tokens_per_frame(self):
        return self.special_per_frame + self.patch_h * self.patch_w

    @property
    def n_tokens(self):
        return self.frames * self.tokens_per_frame

    @property
    def n_special(self):
        return self.frames * self.special_per_frame

    @property
    def n_patch(self):
        return self.n_tokens - self.n_special

    @property
    def n_qblocks(self):
        return math.ceil(self.n_tokens / self.block)

    @property
    def n_blocks(self):
        return math.ceil(self.n_patch / self.block)


def split_keys(k, v, frames, patches_per_frame, special_per_frame=SPECIAL_PER_FRAME):
    """Contiguous (patch_k, patch_v, special_k, special_v) from [H, N, d] keys/values
    (saf3r/patch/adaptive_block_value.py:308-309)."""
    patches, specials = token_layout(frames, patches_per_frame, special_per_frame, k.device)
    return (k[:, patches].contiguous(), v[:, patches].contiguous(),
            k[:, specials].contiguous(), v[:, specials].contiguous())
