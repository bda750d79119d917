"""GPU parity of the fused QKV projection (vggt_qkv_project_pool): against the
reference module's outputs (tests/golden/qkv.npz), against the oracle at the
VGGT shape (1024 channels, 16 heads, 37 x 37 patches), pooled means equal to
block means of the kernel's own outputs, and the layer fed by them selects
the masks the separate estimator selects.

Tolerances: q / k / v are bf16 and may differ from the reference where the
GEMM's fp32 accumulation order moves a projected value across a bf16 rounding
boundary; LayerNorm and RoPE spread that step over the row (check_bf16 states
the bound).  Block means rtol 1e-5 against block means of the kernel's own
q / k."""
import numpy as np
import pytest
import torch

import oracle
import vggt_sparse
from conftest import load_golden

pytestmark = pytest.mark.gpu

NAMES = ("q", "patch_k", "patch_v", "special_k", "special_v")
GOLD = ("q", "k_patch", "v_patch", "k_special", "v_special")


def bf16(a):
    return torch.from_numpy(np.asarray(a)).view(torch.bfloat16)


def check_bf16(got, want, frac=0.02):
    """bf16 outputs: a one-step rounding difference of the projection (GEMM
    accumulation order) moves LayerNorm / RoPE outputs by up to a few 1e-3, so
    each element must be within 2 bf16 steps of the larger magnitude plus 8e-3,
    few elements may differ at all, and the mean difference is tiny."""
    got = got.float().cpu().numpy()
    want = np.asarray(want, dtype=np.float32)
    assert got.shape == want.shape
    diff = np.abs(got - want)
    mag = np.maximum(np.maximum(np.abs(got), np.abs(want)), 2.0 ** -20)
    step = 2.0 ** (np.floor(np.log2(mag)) - 7)
    stats = (float(diff.max()), float((diff > 0).mean()),
             float(diff.mean() / max(np.abs(want).mean(), 1e-12)))
    assert (diff <= 2 * step + 8e-3).all(), stats
    assert stats[1] <= frac, stats
    assert stats[2] <= 1e-3, stats


def run_golden(cuda, g):
    heads = g["w"].shape[1] // 64
    ln = lambda w, b: (torch.tensor(w, device=cuda), torch.tensor(b, device=cuda),
                       float(g["ln_eps"]))
    return vggt_sparse.project_qkv(
        bf16(g["x"]).to(cuda), bf16(g["w"]).to(cuda), bf16(g["b"]).to(cuda), heads=heads,
        tokens_per_frame=int(g["tokens_per_frame"]),
        special_per_frame=int(g["special_per_frame"]), q_norm=ln(g["qn_w"], g["qn_b"]),
        k_norm=ln(g["kn_w"], g["kn_b"]), pos=torch.tensor(g["pos"], device=cuda))


def test_qkv_projection_matches_reference_module(cuda):
    g = load_golden("qkv.npz")
    out = run_golden(cuda, g)
    torch.cuda.synchronize()
    for name, gname in zip(NAMES, GOLD):
        check_bf16(getattr(out, name), bf16(g[gname]).float().numpy())
    # the means are the block means of the kernel's own bf16 outputs
    np.testing.assert_allclose(out.pooled_q.cpu().numpy(),
                               oracle.block_mean(out.q.float().cpu().numpy(), 64)[0], rtol=1e-5,
                               atol=1e-6)
    np.testing.assert_allclose(out.pooled_k.cpu().numpy(),
                               oracle.block_mean(out.patch_k.float().cpu().numpy(), 64)[0],
                               rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(out.pooled_q.cpu().numpy(), g["pooled_q"], rtol=2e-3, atol=2e-3)
    np.testing.assert_allclose(out.pooled_k.cpu().numpy(), g["pooled_k"], rtol=2e-3, atol=2e-3)


def _vggt_case(cuda, frames, seed):
    heads, dim, gh = 16, 1024, 37
    tpf = 5 + gh * gh
    n = frames * tpf
    gen = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(n, dim, generator=gen).to(torch.bfloat16)
    w = (torch.randn(3 * dim, dim, generator=gen) * 0.03).to(torch.bfloat16)
    b = (torch.randn(3 * dim, generator=gen) * 0.1).to(torch.bfloat16)
    qn = (1 + 0.1 * torch.randn(64, generator=gen), 0.1 * torch.randn(64, generator=gen))
    kn = (1 + 0.1 * torch.randn(64, generator=gen), 0.1 * torch.randn(64, generator=gen))
    yy, xx = torch.meshgrid(torch.arange(gh), torch.arange(gh), indexing="ij")
    grid = torch.stack((yy.flatten() + 1, xx.flatten() + 1), -1)
    pos = torch.cat((torch.zeros(5, 2, dtype=torch.long), grid)).repeat(frames, 1).int()
    return dict(x=x, w=w, b=b, qn=qn, kn=kn, pos=pos, heads=heads, tpf=tpf)


def test_qkv_projection_matches_oracle_at_vggt_shape(cuda):
    c = _vggt_case(cuda, 2, 7)
    out = vggt_sparse.project_qkv(
        c["x"].to(cuda), c["w"].to(cuda), c["b"].to(cuda), heads=c["heads"],
        tokens_per_frame=c["tpf"], q_norm=tuple(t.to(cuda) for t in c["qn"]),
        k_norm=tuple(t.to(cuda) for t in c["kn"]), pos=c["pos"].to(cuda))
    want = oracle.project_qkv(c["x"].float().numpy(), c["w"].float().numpy(),
                              c["b"].float().numpy(), c["heads"], c["tpf"], 5,
                              tuple(t.numpy() for t in c["qn"]),
                              tuple(t.numpy() for t in c["kn"]), 1e-5, c["pos"].numpy())
    for name, w in zip(NAMES, want[:5]):
        check_bf16(getattr(out, name), w)
    np.testing.assert_allclose(out.pooled_q.cpu().numpy(),
                               oracle.block_mean(out.q.float().cpu().numpy(), 64)[0], rtol=1e-5,
                               atol=1e-6)
    np.testing.assert_allclose(out.pooled_k.cpu().numpy(),
                               oracle.block_mean(out.patch_k.float().cpu().numpy(), 64)[0],
                               rtol=1e-5, atol=1e-6)


def test_layer_from_projection_selects_like_the_estimator(cuda):
    """estimate_pooled on the fused means: the means equal the separate
    estimator's pooling of the projection's q / k to fp32 rounding, the masks
    agree with it (but for near-ties of fp32 scores), and the layer's output
    matches the fp64 oracle on the masks it chose."""
    c = _vggt_case(cuda, 2, 9)
    out = vggt_sparse.project_qkv(
        c["x"].to(cuda), c["w"].to(cuda), c["b"].to(cuda), heads=c["heads"],
        tokens_per_frame=c["tpf"], q_norm=tuple(t.to(cuda) for t in c["qn"]),
        k_norm=tuple(t.to(cuda) for t in c["kn"]), pos=c["pos"].to(cuda))
    fused = vggt_sparse.SparseGlobalLayer(16, mode="topk", topk=20, dense_heads=(0, 3))
    got = fused.forward_projected(out)
    sep = vggt_sparse.SparseGlobalLayer(16, mode="topk", topk=20, dense_heads=(0, 3))
    sep(out.q, out.patch_k, out.patch_v, out.special_k, out.special_v)
    torch.cuda.synchronize()
    same = (fused.last_masks[0] == sep.last_masks[0]).all(-1)
    assert float(same.float().mean()) >= 0.99
    idx, cnt = (t.cpu().numpy() for t in fused.last_masks)
    qbs = [0, 40, idx.shape[1] - 1]
    f = lambda t: t.float().cpu().numpy()
    exp, _ = oracle.block_sparse_attention(f(out.q), f(out.patch_k), f(out.patch_v),
                                           f(out.special_k), f(out.special_v), idx, cnt,
                                           fused.sparse_heads, qblocks=qbs)
    rows = np.concatenate([np.arange(b * 64, min((b + 1) * 64, out.q.shape[1])) for b in qbs])
    g = got.float().cpu().numpy()
    for h in fused.sparse_heads[:3]:
        d = np.abs(g[h, rows] - exp[h, rows])
        assert d.max() <= 2e-2 and d.mean() / np.abs(exp[h, rows]).mean() <= 1e-2


@pytest.mark.parametrize("heads,bias,extras", [(48, "aligned", True), (48, "offset", True),
                                               (4, None, False)])
def test_qkv_projection_variants_against_oracle(cuda, heads, bias, extras):
    """Paths the VGGT shape does not take: a model too wide for the bias to
    be staged in shared memory (48 heads: read from global memory, 16-byte
    vectors when aligned, element by element when the bias starts 4 bytes
    off), and a plain projection with no bias, LayerNorm or RoPE."""
    dim, gh, frames = 64 * heads, 6, 2
    tpf = 5 + gh * gh
    n = frames * tpf
    gen = torch.Generator(device="cpu").manual_seed(11 + heads)
    x = torch.randn(n, dim, generator=gen).to(torch.bfloat16)
    w = (torch.randn(3 * dim, dim, generator=gen) * dim ** -0.5).to(torch.bfloat16)
    b = None
    if bias is not None:
        full = (torch.randn(3 * dim + 2, generator=gen) * 0.1).to(torch.bfloat16)
        b = full[2:] if bias == "offset" else full[:3 * dim]
    ln = (1 + 0.1 * torch.randn(64, generator=gen), 0.1 * torch.randn(64, generator=gen))
    yy, xx = torch.meshgrid(torch.arange(gh), torch.arange(gh), indexing="ij")
    grid = torch.stack((yy.flatten() + 1, xx.flatten() + 1), -1)
    pos = torch.cat((torch.zeros(5, 2, dtype=torch.long), grid)).repeat(frames, 1).int()
    bd = None
    if b is not None:
        store = full.to(cuda)
        bd = store[2:] if bias == "offset" else store[:3 * dim]
        assert (bd.data_ptr() % 16 != 0) == (bias == "offset")
    lnd = tuple(t.to(cuda) for t in ln) if extras else None
    out = vggt_sparse.project_qkv(x.to(cuda), w.to(cuda), bd, heads=heads, tokens_per_frame=tpf,
                                  q_norm=lnd, k_norm=lnd, pos=pos.to(cuda) if extras else None)
    lnn = tuple(t.numpy() for t in ln) if extras else None
    want = oracle.project_qkv(x.float().numpy(), w.float().numpy(),
                              b.float().numpy() if b is not None else None, heads, tpf, 5,
                              lnn, lnn, 1e-5, pos.numpy() if extras else None)
    for name, wv in zip(NAMES, want[:5]):
        check_bf16(getattr(out, name), wv)
    np.testing.assert_allclose(out.pooled_q.cpu().numpy(),
                               oracle.block_mean(out.q.float().cpu().numpy(), 64)[0], rtol=1e-5,
                               atol=1e-6)
    np.testing.assert_allclose(out.pooled_k.cpu().numpy(),
                               oracle.block_mean(out.patch_k.float().cpu().numpy(), 64)[0],
                               rtol=1e-5, atol=1e-6)
