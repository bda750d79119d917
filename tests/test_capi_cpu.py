"""C-ABI library: loads, exports every declared symbol, validates arguments.
No kernel is launched (argument errors return before any CUDA call)."""
import ctypes
import os
import re

import pytest

from conftest import REPO

HEADER = os.path.join(REPO, "include", "vggt_sparse.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\w[\w\s\*]*?\b(vggt_\w+)\s*\(", text, re.M)))


@pytest.fixture(scope="module")
def lib():
    from vggt_sparse import _lib
    if not os.path.exists(_lib.LIB_PATH):
        from vggt_sparse.build import build
        build()
    return _lib.load()


def test_header_declares_the_documented_entry_points():
    assert declared_symbols() == sorted([
        "vggt_block_attention", "vggt_block_attention_ex", "vggt_block_attention_workspace_size",
        "vggt_block_mask_assemble", "vggt_block_mask_estimate", "vggt_block_mask_estimate_noalloc",
        "vggt_block_select", "vggt_block_select_pooled", "vggt_frame_qk_topk",
        "vggt_history_update", "vggt_kv_push", "vggt_kv_push_flag_bytes",
        "vggt_qkv_project_pool", "vggt_qkv_workspace_size",
        "vggt_sparse_last_error",
        "vggt_sparse_set_wait_limit_ns", "vggt_sparse_set_wait_selftest", "vggt_sparse_version", "vggt_token_sparse_attention"])


def test_wait_limit_setter_round_trips(lib):
    from vggt_sparse import _lib
    assert _lib.set_wait_limit_ns(12345) == 0
    assert _lib.set_wait_limit_ns(0) == 12345
    assert _lib.set_wait_limit_ns(0) == 0
    assert _lib.set_wait_selftest(True) == 0
    assert _lib.set_wait_selftest(False) == 1


@pytest.mark.parametrize("lang,std", [("c", "-std=c99"), ("c++", "-std=c++17")])
def test_header_compiles_alone(lang, std, tmp_path):
    """include/vggt_sparse.h is self-contained plain C (a cgo / ctypes-style
    caller includes it with nothing before it)."""
    import shutil
    import subprocess
    cc = shutil.which("gcc" if lang == "c" else "g++")
    if cc is None:
        pytest.skip("no host compiler")
    hdr = os.path.join(REPO, "include", "vggt_sparse.h")
    res = subprocess.run([cc, "-fsyntax-only", "-x", lang, std, "-Wall", "-Wextra", "-pedantic",
                          "-Werror", hdr], capture_output=True, text=True)
    assert res.returncode == 0, res.stderr


def test_library_exports_every_declared_symbol(lib):
    from vggt_sparse import _lib
    for name in declared_symbols():
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, name


def test_attention_workspace_size(lib):
    """Pair table [slots, ceil(QB/2), 2] int32 + work order [slots * ceil(QB/2)]
    + bitmaps + window costs + singles + pair sizes, each rounded up to 256
    bytes; 0 when the shape is not paired."""
    up = lambda x: (x + 255) // 256 * 256
    n, npatch, slots = 43968, 43808, 12
    qb, nb = -(-n // 64), -(-npatch // 64)
    nwords = -(-nb // 32)
    npairs = -(-qb // 2)
    want = (up(slots * npairs * 2 * 4) + up(slots * npairs * 4) + up(slots * qb * nwords * 4) +
            up(slots * qb * 128 * 2) + up(slots * qb * 4) + up(slots * npairs * 4))
    assert lib.vggt_block_attention_workspace_size(n, npatch, slots, 64, 64) == want
    assert lib.vggt_block_attention_workspace_size(64, npatch, slots, 64, 64) == 0  # one block
    assert lib.vggt_block_attention_workspace_size(n, npatch, 0, 64, 64) == 0


def test_version(lib):
    assert lib.vggt_sparse_version() == (1 << 16)


def _attn(lib, **kw):
    args = dict(q=16, pk=16, pv=16, sk=16, sv=16, dtype=0, heads=2, n=128, npatch=64, nspecial=5,
                dim=64, indices=16, counts=16, per_row=0, head_ids=16, dense=None, slots=1,
                maxk=1, bq=64, bk=64, scale=0.125, out=16, ev=None, status=None, kernel=0,
                stream=None)
    args.update(kw)
    return lib.vggt_block_attention(*args.values())


@pytest.mark.parametrize("bad,msg", [
    (dict(dtype=5), "BF16 or FP16"),
    (dict(dim=128), "head dim"),
    (dict(bq=16), "query_block"),
    (dict(bk=256), "key_block"),
    (dict(heads=0), "size"),
    (dict(npatch=0, nspecial=0), "no keys"),
    (dict(scale=float("inf")), "finite"),
    (dict(kernel=9), "kernel"),
    (dict(q=None), "non-NULL"),
    (dict(q=8), "aligned"),
    (dict(slots=70000), "65535"),
])
def test_attention_argument_errors(lib, bad, msg):
    rc = _attn(lib, **bad)
    assert rc < 0
    assert msg in lib.vggt_sparse_last_error().decode()


def test_attention_empty_is_a_no_op(lib):
    assert _attn(lib, slots=0) == 0
    assert _attn(lib, n=0) == 0


def _est(lib, **kw):
    args = dict(q=16, kp=16, dtype=0, heads=2, n=128, npatch=64, dim=64, head_ids=16, slots=1,
                bq=64, bk=64, mode=0, topk=1, tau=0.0, scale=0.125, pq=16, pk=16, idx=16,
                maxk=1, counts=16, scores=None, status=None, stream=None)
    args.update(kw)
    return lib.vggt_block_mask_estimate(*args.values())


@pytest.mark.parametrize("bad,msg", [
    (dict(dtype=2), "BF16 or FP16"),
    (dict(mode=0, topk=0), "topk"),
    (dict(mode=0, topk=4, maxk=0), "max_blocks"),
    (dict(mode=1, tau=0.0, maxk=1), "tau"),
    (dict(mode=1, tau=1.5, maxk=1), "tau"),
    (dict(mode=1, tau=0.9, maxk=0), "max_blocks"),
    (dict(mode=7), "mode"),
    (dict(npatch=0), "n_patch"),
    (dict(npatch=64 * 60000), "exceed"),
    (dict(pq=None), "non-NULL"),
])
def test_estimator_argument_errors(lib, bad, msg):
    rc = _est(lib, **bad)
    assert rc < 0
    assert msg in lib.vggt_sparse_last_error().decode()


def test_assemble_and_history_argument_errors(lib):
    asm = lambda **kw: lib.vggt_block_mask_assemble(*dict(dict(
        scores=16, s=1, qb=4, nb=100, vo=16, counts=16, a=16, hist=None, hlen=0, ids=16, org=None,
        maxk=8, status=None, stream=None), **kw).values())
    assert asm(s=-1) < 0
    assert asm(nb=0) < 0 and "n_blocks" in lib.vggt_sparse_last_error().decode()
    assert asm(nb=100000) < 0 and "exceeds" in lib.vggt_sparse_last_error().decode()
    assert asm(scores=None) < 0 and "non-NULL" in lib.vggt_sparse_last_error().decode()
    assert asm(hlen=5) < 0 and "history" in lib.vggt_sparse_last_error().decode()
    assert asm(maxk=0) < 0
    assert asm(s=0) == 0
    hist = lambda **kw: lib.vggt_history_update(*dict(dict(
        ev=16, ids=16, s=1, qb=4, maxk=8, counts=16, keeps=16, out=16, hlen=4, stream=None),
        **kw).values())
    assert hist(ev=None) < 0
    assert hist(hlen=0) == 0


def test_token_attention_argument_errors(lib):
    call = lambda **kw: lib.vggt_token_sparse_attention(*dict(dict(
        q=16, k=16, v=16, idx=16, stride=4, n=8, nk=100, topk=4, dim=64, dtype=0,
        scale=0.125, out=16, status=None, stream=None), **kw).values())
    for bad, msg in ((dict(dtype=3), "BF16 or FP16"), (dict(dim=48), "head dim"),
                     (dict(topk=-1), "negative"), (dict(scale=float("nan")), "finite"),
                     (dict(q=None), "non-NULL"), (dict(v=8), "aligned")):
        assert call(**bad) < 0
        assert msg in lib.vggt_sparse_last_error().decode()
    assert call(n=0) == 0


def test_kv_push_argument_errors(lib):
    assert lib.vggt_kv_push_flag_bytes(8) == 256 and lib.vggt_kv_push_flag_bytes(17) == 0
    two = lambda *v: (ctypes.c_void_p * 2)(*v)
    i64 = lambda *v: (ctypes.c_int64 * len(v))(*v)
    call = lambda **kw: lib.vggt_kv_push(*dict(dict(
        shards=two(256, 512), rows=i64(10, 10), offs=i64(0, 4096), n=2, heads=4, dim=64, es=2,
        bases=two(1 << 20, 1 << 21), world=2, rank=0, flags=8192, phase=0, epoch=1, hs=1, grid=0,
        status=None, stream=None), **kw).values())
    for bad, msg in ((dict(n=0), "n_tensors"), (dict(world=17), "world"), (dict(rank=2), "rank"),
                     (dict(phase=2), "phase"), (dict(dim=4), "16 bytes"), (dict(epoch=0), "epoch"),
                     (dict(flags=6), "flags_offset"), (dict(offs=i64(0, 8)), "dst_offsets"),
                     (dict(shards=two(256, 520)), "aligned"), (dict(rows=i64(10, 0)), "rows_local"),
                     (dict(bases=two(1 << 20, 0)), "rank_bases"), (dict(bases=None), "non-NULL")):
        assert call(**bad) < 0, bad
        assert msg in lib.vggt_sparse_last_error().decode(), (bad, lib.vggt_sparse_last_error())


def test_token_attention_checks_out_and_status():
    """A caller's out must have q's shape and dtype and be contiguous, and status
    must be int32: the kernel writes N * D elements of q's dtype from out's first
    byte.  These checks run before any device work, so CPU tensors reach them."""
    import torch
    import vggt_sparse
    q = torch.zeros(8, 64, dtype=torch.bfloat16)
    kv = torch.zeros(20, 64, dtype=torch.bfloat16)
    idx = torch.zeros(8, 4, dtype=torch.int32)
    for bad in (torch.empty(4, 64, dtype=torch.bfloat16),              # too small
                torch.empty(8, 64, dtype=torch.float32),               # other dtype
                torch.empty(64, 8, dtype=torch.bfloat16).t()):         # not contiguous
        with pytest.raises(ValueError, match="out must be"):
            vggt_sparse.token_sparse_attention(q, kv, kv, idx, out=bad)
    for bad in (torch.zeros(1, dtype=torch.int64), torch.zeros(0, dtype=torch.int32)):
        with pytest.raises(ValueError, match="status must be"):
            vggt_sparse.token_sparse_attention(q, kv, kv, idx, status=bad)
    with pytest.raises(ValueError, match="CUDA"):  # well-formed CPU call: no CPU path
        vggt_sparse.token_sparse_attention(q, kv, kv, idx, out=torch.empty_like(q))


def test_token_attention_query_limit(lib):
    lim = 0x7fffffff * 4  # the grid has one CTA per 4 queries, at most 2^31 - 1 CTAs
    call = lambda n: lib.vggt_token_sparse_attention(16, 16, 16, 16, 4, n, 100, 4, 64, 0,
                                                     0.125, 16, None, None)
    assert call(lim + 1) < 0
    assert "too many queries" in lib.vggt_sparse_last_error().decode()


def test_frame_topk_argument_errors(lib):
    call = lambda **kw: lib.vggt_frame_qk_topk(*dict(dict(
        q=16, k=16, out=16, batch=1, nq=8, frames=2, tokens=100, dim=64, topk=4, groups=0,
        status=None, stream=None), **kw).values())
    for bad, msg in ((dict(dim=48), "unsupported"), (dict(topk=129, tokens=200), "unsupported"),
                     (dict(tokens=0), "tokens"), (dict(groups=-1), ">= 0"),
                     (dict(q=None), "non-NULL"), (dict(out=8), "aligned")):
        assert call(**bad) < 0, bad
        assert msg in lib.vggt_sparse_last_error().decode()
    assert call(nq=0) == 0 and call(frames=0) == 0
    assert call(topk=500, tokens=100, q=None) < 0  # clamped to 100, then the pointer check
    assert "non-NULL" in lib.vggt_sparse_last_error().decode()


def test_frame_topk_python_checks():
    import torch
    import vggt_sparse
    q = torch.zeros(1, 4, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        vggt_sparse.compute_qk_topk_indices_fused(q, q, 2, num_toks_per_img=2)
    with pytest.raises(AssertionError):
        vggt_sparse.compute_qk_topk_indices_fused(q, q, 2, num_toks_per_img=3)
    with pytest.raises(AssertionError):
        vggt_sparse.compute_qk_topk_indices_fused(q, q, 2)


def test_select_argument_errors(lib):
    assert lib.vggt_block_select(16, 4, 0, 0, 1, 0.0, 16, 1, 16, None) < 0
    assert lib.vggt_block_select(16, 4, 10, 1, 0, 0.9, 16, 5, 16, None) < 0
    assert lib.vggt_block_select(16, 0, 10, 0, 3, 0.0, 16, 3, 16, None) == 0


def test_python_layer_rejects_cpu_tensors_and_fp32():
    import torch
    import vggt_sparse
    q = torch.zeros(2, 8, 64, dtype=torch.float32)
    with pytest.raises(ValueError, match="BF16 or FP16"):
        vggt_sparse.block_attention(q, q, q, q, q, torch.zeros(1, 1, 1, dtype=torch.int32),
                                    torch.zeros(1, dtype=torch.int32),
                                    torch.zeros(1, dtype=torch.int32))
    qb = q.to(torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        vggt_sparse.block_attention(qb, qb, qb, qb, qb, torch.zeros(1, 1, 1, dtype=torch.int32),
                                    torch.zeros(1, dtype=torch.int32),
                                    torch.zeros(1, dtype=torch.int32), validate=False)


def test_missing_library_fails_loudly(tmp_path):
    from vggt_sparse import _lib
    with pytest.raises(_lib.ExtensionMissing):
        _lib.load(str(tmp_path / "missing.so"))
