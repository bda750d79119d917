"""QKV projection + q/k LayerNorm + RoPE-2D + layout split + block means
(oracle; test infrastructure only).

Restates saf3r/patch/adaptive_block_value.py:297-315 at bf16 inference
precision: the `qkv` Linear computed exactly (float64) and rounded to bf16 (an
fp32-accumulating GEMM's output rounds to the same bf16 except within an ulp
of a rounding boundary), LayerNorm (torch.nn.LayerNorm: biased variance) in
fp32, RoPE-2D of saf3r/models/official_vggt/layers/rope.py (frequencies
base^(-2i/32), the first 32 dims rotated by the y position, the last 32 by the
x position, x cos + rotate(x) sin with rotate(a, b) = (-b, a)) in fp32, q and k
rounded to bf16; the token layout of saf3r/patch/value_evolving_attention.py
token_layout (specials first in each frame); block means of
adaptive_block_value.py:16-23.
"""
import numpy as np
import torch

from .estimator import block_mean


def _bf16(a):
    return torch.from_numpy(np.asarray(a, dtype=np.float32)).to(torch.bfloat16).float().numpy()


def _layer_norm(v, w, b, eps):
    t = torch.from_numpy(v.astype(np.float32))
    return torch.nn.functional.layer_norm(t, (v.shape[-1],), torch.from_numpy(w),
                                          torch.from_numpy(b), eps).numpy()


def _rope(v, pos, base):
    t = torch.from_numpy(v.astype(np.float32))
    exponents = torch.arange(0, 32, 2).float() / 32
    inv_freq = 1.0 / (base ** exponents)
    positions = torch.arange(int(pos.max()) + 1, dtype=torch.float32)
    ang = torch.einsum("i,j->ij", positions, inv_freq)
    ang = torch.cat((ang, ang), -1)
    cos, sin = ang.cos(), ang.sin()
    out = []
    for half, axis in ((t[..., :32], 0), (t[..., 32:], 1)):
        p = torch.from_numpy(pos[:, axis].astype(np.int64))
        c, s = cos[p], sin[p]
        rot = torch.cat((-half[..., 16:], half[..., :16]), -1)
        out.append(half * c + rot * s)
    return torch.cat(out, -1).numpy()


def project_qkv(x, w, b, heads, tokens_per_frame, special_per_frame, qn=None, kn=None,
                eps=1e-5, pos=None, base=100.0):
    """x [N, C], w [3C, C], b [3C] or None (bf16 values as float arrays);
    qn / kn (weight, bias) fp32 [64] or None; pos [N, 2] int (y, x) or None.
    Returns (q [H, N, 64], k_patch, v_patch, k_special, v_special, pooled_q
    [H, QB, 64], pooled_k [H, NB, 64]) as float32 arrays."""
    x = np.asarray(x, dtype=np.float64)
    n, c = x.shape
    y = x @ np.asarray(w, dtype=np.float64).T
    if b is not None:
        y = y + np.asarray(b, dtype=np.float64)
    y = _bf16(y).reshape(n, 3, heads, 64).transpose(1, 2, 0, 3)  # [3, H, N, 64]
    q, k, v = y[0], y[1], y[2]
    if qn is not None:
        q = _layer_norm(q, np.asarray(qn[0], np.float32), np.asarray(qn[1], np.float32), eps)
    if kn is not None:
        k = _layer_norm(k, np.asarray(kn[0], np.float32), np.asarray(kn[1], np.float32), eps)
    if pos is not None:
        pos = np.asarray(pos)
        q, k = _rope(q, pos, base), _rope(k, pos, base)
    q, k = _bf16(q), _bf16(k)
    frames = n // tokens_per_frame
    ppf = tokens_per_frame - special_per_frame
    fr = np.arange(frames)[:, None] * tokens_per_frame
    patches = (fr + special_per_frame + np.arange(ppf)[None]).reshape(-1)
    specials = (fr + np.arange(special_per_frame)[None]).reshape(-1)
    kp, vp, ks, vs = k[:, patches], v[:, patches], k[:, specials], v[:, specials]
    pooled_q, _ = block_mean(q, 64)
    pooled_k, _ = block_mean(kp, 64)
    return (q.astype(np.float32), kp.astype(np.float32), vp.astype(np.float32),
            ks.astype(np.float32), vs.astype(np.float32), pooled_q, pooled_k)
