"""Seeded synthetic global-attention inputs (clustered Q/K, Gaussian V).

Stand-in for the reference's 7Scenes/ETH3D inputs, which (like the VGGT
checkpoint) are not available offline.  Per head, C shared centres
c_j ~ N(0, I_d).  Each patch token takes the centre of a coarse spatial cell
of its frame (cells of ``cell`` x ``cell`` patches, the cell->centre table
shared by all frames, each frame shifted by a random offset so views overlap
but differ); specials take random centres.  q and k of a token are
s * (c + noise * N(0, I)) with independent noise, v ~ N(0, 1); s is set so the
std of q.k / sqrt(d) over random token pairs is ``logit_std``.
"""
import math
from dataclasses import dataclass

import torch

from .layout import SPECIAL_PER_FRAME, LayerShape, split_keys


@dataclass
class LayerInputs:
    shape: LayerShape
    q: torch.Tensor   # [H, N, d]
    k: torch.Tensor   # [H, N, d]
    v: torch.Tensor   # [H, N, d]
    kp: torch.Tensor  # [H, NP, d]
    vp: torch.Tensor
    ks: torch.Tensor  # [H, NS, d]
    vs: torch.Tensor


def clustered_layer(frames, *, centres=64, heads=16, dim=64, patch_h=37, patch_w=37,
                    special=SPECIAL_PER_FRAME, seed=0, device="cpu", dtype=torch.bfloat16,
                    logit_std=3.0, noise=0.3, cell=6, keep_full=True):
    """Generate one layer's q/k/v and the patch/special split."""
    g = torch.Generator(device=device).manual_seed(int(seed))
    shape = LayerShape(frames=frames, patch_h=patch_h, patch_w=patch_w, heads=heads, dim=dim,
                       special_per_frame=special)
    n = shape.n_tokens
    grid = max(patch_h, patch_w) // cell + 2
    table = torch.randint(0, centres, (grid, grid), generator=g, device=device)
    shifts = torch.randint(0, cell, (frames, 2), generator=g, device=device)
    yy = torch.arange(patch_h, device=device)[None, :, None]
    xx = torch.arange(patch_w, device=device)[None, None, :]
    cy = (yy + shifts[:, 0, None, None]) // cell
    cx = (xx + shifts[:, 1, None, None]) // cell
    patch_labels = table[cy % grid, cx % grid].reshape(frames, patch_h * patch_w)
    special_labels = torch.randint(0, centres, (frames, special), generator=g, device=device)
    labels = torch.cat((special_labels, patch_labels), 1).reshape(-1)
    cen = torch.randn((heads, centres, dim), generator=g, device=device)
    base = cen[:, labels]
    q = base + noise * torch.randn((heads, n, dim), generator=g, device=device)
    k = base + noise * torch.randn((heads, n, dim), generator=g, device=device)
    del base
    v = torch.randn((heads, n, dim), generator=g, device=device)
    m = 8192
    hi = torch.randint(0, heads, (m,), generator=g, device=device)
    ii = torch.randint(0, n, (m,), generator=g, device=device)
    jj = torch.randint(0, n, (m,), generator=g, device=device)
    dots = (q[hi, ii] * k[hi, jj]).sum(-1) / math.sqrt(dim)
    s = math.sqrt(logit_std / float(dots.std()))
    q = (q * s).to(dtype)
    k = (k * s).to(dtype)
    v = v.to(dtype)
    kp, vp, ks, vs = split_keys(k, v, frames, patch_h * patch_w, special)
    if not keep_full:
        k = v = None
    return LayerInputs(shape, q.contiguous(), k, v, kp, vp, ks, vs)


def homography_views(frames, size=518, *, seed=0, device="cpu", texture=48, max_shift=0.08,
                     max_persp=0.15):
    """`frames` RGB views [1, S, 3, size, size] in [0, 1] of one smooth random
    texture (low-pass noise: a `texture`^2 random grid upsampled bicubically),
    each warped by its own random homography near the identity (translation
    up to `max_shift` of the image, perspective terms up to `max_persp`), so
    neighbouring views overlap the way a camera sweep's do."""
    import torch.nn.functional as F
    g = torch.Generator(device="cpu").manual_seed(int(seed))
    base = torch.rand(1, 3, texture, texture, generator=g)
    base = F.interpolate(base, size=(2 * size, 2 * size), mode="bicubic", align_corners=False)
    base = base.clamp(0, 1).to(device)
    ys, xs = torch.meshgrid(torch.linspace(-0.5, 0.5, size), torch.linspace(-0.5, 0.5, size),
                            indexing="ij")
    pts = torch.stack((xs, ys, torch.ones_like(xs)), -1).reshape(-1, 3)
    views = []
    for _ in range(frames):
        hmat = torch.eye(3)
        hmat[:2, :2] += (torch.rand(2, 2, generator=g) - 0.5) * 2 * max_persp
        hmat[:2, 2] = (torch.rand(2, generator=g) - 0.5) * 2 * max_shift
        hmat[2, :2] = (torch.rand(2, generator=g) - 0.5) * 2 * max_persp
        w = pts @ hmat.T
        grid = (w[:, :2] / w[:, 2:3]).reshape(1, size, size, 2).to(device)
        views.append(F.grid_sample(base, grid, mode="bilinear", padding_mode="reflection",
                                   align_corners=False))
    return torch.stack(views, 1)
