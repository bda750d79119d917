"""QKV projection with the estimator's block pooling fused into its epilogue.

``project_qkv`` replaces the steps of saf3r/patch/adaptive_block_value.py:297-315
that precede the estimator: the attention module's ``qkv`` Linear, ``q_norm``
/ ``k_norm``, RoPE-2D, the patch / special split of the token layout, and the
block means of q (64-token query blocks) and of the patch keys (64-row
blocks).  One launch of ``vggt_qkv_project_pool`` (tcgen05 GEMM, LayerNorm,
RoPE and pooling in the epilogue) plus a small fold of the patch-key block
sums; the estimator then selects from the means (``SparseGlobalLayer.
estimate_pooled``) without reading Q and K again.
"""
import math
from dataclasses import dataclass

import torch

from . import _lib
from .ops import _ptr, _require_contig, _require_cuda, _stream, dtype_code


_TABLES = {}


def _cached_tables(pos_count, base, device):
    key = (int(pos_count), float(base), torch.device(device))
    t = _TABLES.get(key)
    if t is None:
        t = _TABLES[key] = rope_tables(pos_count, base, device)
    return t


def rope_tables(pos_count, base=100.0, device="cuda"):
    """cos / sin [pos_count, 16] fp32 of position * base^(-2i/32), i < 16: the
    frequency components saf3r/models/official_vggt/layers/rope.py computes
    for a 32-dim half (exponents arange(0, 32, 2) / 32, inv_freq = 1 / base **
    exponents, angles = positions x inv_freq), with the same torch ops."""
    exponents = torch.arange(0, 32, 2, device=device).float() / 32
    inv_freq = 1.0 / (base ** exponents)
    positions = torch.arange(pos_count, device=device, dtype=inv_freq.dtype)
    angles = torch.einsum("i,j->ij", positions, inv_freq)
    return angles.cos().contiguous(), angles.sin().contiguous()


def _norm_params(norm, device):
    """(weight, bias) fp32 [64] of a LayerNorm module or pair, or (None, None)."""
    if norm is None or isinstance(norm, torch.nn.Identity):
        return None, None, None
    if isinstance(norm, torch.nn.LayerNorm):
        if tuple(norm.normalized_shape) != (64,) or norm.weight is None:
            raise ValueError("q_norm / k_norm must be LayerNorm(64) with an affine weight")
        w, b, eps = norm.weight, norm.bias, float(norm.eps)
    else:
        w, b = norm[:2]
        eps = float(norm[2]) if len(norm) > 2 else 1e-5
    w = w.detach().to(device=device, dtype=torch.float32).contiguous()
    b = (b.detach().to(device=device, dtype=torch.float32).contiguous() if b is not None
         else torch.zeros(64, device=device, dtype=torch.float32))
    return w, b, eps


@dataclass
class QkvOut:
    q: torch.Tensor          # [H, N, 64]
    patch_k: torch.Tensor    # [H, NP, 64]
    patch_v: torch.Tensor
    special_k: torch.Tensor  # [H, NS, 64]
    special_v: torch.Tensor
    pooled_q: torch.Tensor   # [H, ceil(N / 64), 64] fp32 block means (or None)
    pooled_k: torch.Tensor   # [H, ceil(NP / 64), 64] fp32 (or None)


def project_qkv(x, w_qkv, b_qkv=None, *, heads, tokens_per_frame, special_per_frame=5,
                q_norm=None, k_norm=None, pos=None, rope_base=100.0, pool=True, status=None,
                pos_count=None):
    """x [N, C] (or [1, N, C]) bf16/fp16 CUDA, C = 64 * heads; w_qkv [3C, C] and
    b_qkv [3C] (the nn.Linear's weight and bias, converted to x's dtype as
    autocast does); q_norm / k_norm: LayerNorm(64) modules or (weight, bias[,
    eps]) pairs, or None; pos: [N, 2] int (y, x) token positions for RoPE-2D
    (as VGGT's aggregator builds them), or None; ``pos_count`` (largest
    position + 1) saves the host read of pos.max() that computing it costs
    (the kernel clamps positions to [0, pos_count - 1]).
    Returns a QkvOut."""
    if x.dim() == 3:
        if x.shape[0] != 1:
            raise ValueError("batch one only")
        x = x[0]
    if x.dim() != 2:
        raise ValueError("x must be [N, C]")
    _require_cuda(x, w_qkv, b_qkv, pos, status)
    n, c = x.shape
    if c != 64 * heads:
        raise ValueError("x has %d channels, heads * 64 = %d" % (c, 64 * heads))
    code = dtype_code(x.dtype)
    w = w_qkv.to(x.dtype).contiguous()
    if w.shape != (3 * c, c):
        raise ValueError("w_qkv must be [3C, C]")
    b = b_qkv.to(x.dtype).contiguous() if b_qkv is not None else None
    if b is not None and b.shape != (3 * c,):
        raise ValueError("b_qkv must be [3C]")
    x = x.contiguous()
    if n % tokens_per_frame:
        raise ValueError("N must be a whole number of frames")
    frames = n // tokens_per_frame
    npatch = frames * (tokens_per_frame - special_per_frame)
    nspecial = frames * special_per_frame
    dev = x.device
    qw, qb, qeps = _norm_params(q_norm, dev)
    kw, kb, keps = _norm_params(k_norm, dev)
    if qeps is not None and keps is not None and qeps != keps:
        raise ValueError("q_norm and k_norm must share eps")
    eps = qeps if qeps is not None else (keps if keps is not None else 1e-5)
    cos = sin = None
    if pos is None:
        pos_count = 0
    else:
        pos = pos.reshape(-1, 2).to(device=dev, dtype=torch.int32).contiguous()
        if pos.shape[0] != n:
            raise ValueError("pos must be [N, 2]")
        if pos_count is None:
            pos_count = int(pos.max()) + 1 if n else 1  # one host read
        cos, sin = _cached_tables(pos_count, rope_base, dev)
    empty = lambda rows: torch.empty((heads, rows, 64), device=dev, dtype=x.dtype)
    q, kp, vp, ks, vs = empty(n), empty(npatch), empty(npatch), empty(nspecial), empty(nspecial)
    pq = pk = ws = None
    if pool:
        pq = torch.empty((heads, math.ceil(n / 64), 64), device=dev, dtype=torch.float32)
        pk = torch.empty((heads, math.ceil(npatch / 64), 64), device=dev, dtype=torch.float32)
        lib = _lib.load()
        ws = torch.empty(int(lib.vggt_qkv_workspace_size(n, heads)), device=dev,
                         dtype=torch.uint8)
    _require_contig(q=q)
    lib = _lib.load()
    rc = lib.vggt_qkv_project_pool(
        _ptr(x), _ptr(w), _ptr(b), code, n, heads, tokens_per_frame, special_per_frame,
        _ptr(qw), _ptr(qb), _ptr(kw), _ptr(kb), float(eps), _ptr(pos), _ptr(cos), _ptr(sin),
        pos_count, _ptr(q), _ptr(kp), _ptr(vp), _ptr(ks), _ptr(vs), _ptr(pq), _ptr(pk),
        _ptr(ws), ws.numel() if ws is not None else 0, _ptr(status), _stream(dev))
    _lib.check(rc)
    return QkvOut(q, kp, vp, ks, vs, pq, pk)
