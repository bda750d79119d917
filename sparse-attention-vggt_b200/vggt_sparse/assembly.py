"""Device mask assembly with history and value order, and the same-pass
history update (vggt_block_mask_assemble / vggt_history_update).

``select_block_mask`` keeps the signature and return value of
saf3r/patch/adaptive_block_value.py:42-91 for one head; ``assemble_masks``
runs every (head, query block) row in one launch; ``history_update`` is the
update of :389-396.  No host synchronisation; CUDA tensors only.
"""
import torch

from . import _lib
from .ops import _ptr, _require_contig, _require_cuda, _stream


def _i32(x, device):
    return torch.as_tensor(x, dtype=torch.int32, device=device).reshape(-1).contiguous()


def assemble_masks(scores, value_order, counts, attention_counts, history=None, *,
                   max_blocks=None, with_origin=True, status=None):
    """scores [S, QB, NB] fp32; value_order [NB]; counts / attention_counts:
    one per slot (sequence or tensor); history [S, QB, H] int32 (-1 empty) or
    None.  Returns (ids [S, QB, max_blocks] int32 ascending, -1 padded;
    origin uint8 of the same shape (1 reused, 2 attention, 0 value) or None)."""
    if scores.dim() != 3 or scores.dtype != torch.float32:
        raise ValueError("scores must be float32 [slots, query blocks, key blocks]")
    _require_cuda(scores, history, status)
    dev = scores.device
    s, qb, nb = scores.shape
    vo = _i32(value_order, dev)
    cnt = _i32(counts, dev)
    acnt = _i32(attention_counts, dev)
    if vo.numel() != nb:
        raise ValueError("value_order must list the %d key blocks" % nb)
    if cnt.numel() != s or acnt.numel() != s:
        raise ValueError("counts and attention_counts need one entry per slot")
    if max_blocks is None:
        max_blocks = max(1, int(torch.as_tensor(counts).max())) if s else 1
    hlen = 0
    if history is not None:
        if history.dim() != 3 or history.shape[:2] != (s, qb) or history.dtype != torch.int32:
            raise ValueError("history must be int32 [slots, query blocks, H]")
        hlen = history.shape[2]
    _require_contig(scores=scores, history=history)
    ids = torch.empty((s, qb, max_blocks), dtype=torch.int32, device=dev)
    origin = torch.empty((s, qb, max_blocks), dtype=torch.uint8, device=dev) if with_origin else None
    lib = _lib.load()
    rc = lib.vggt_block_mask_assemble(_ptr(scores), s, qb, nb, _ptr(vo), _ptr(cnt), _ptr(acnt),
                                      _ptr(history) if hlen else None, hlen, _ptr(ids),
                                      _ptr(origin), max_blocks, _ptr(status), _stream(dev))
    _lib.check(rc)
    return ids, origin


def select_block_mask(scores, value_order, count, attention_count, history=None):
    """One head, as saf3r/patch/adaptive_block_value.py:42-91: scores
    [rows, key blocks]; returns (ids [rows, count] int64 ascending, origin
    [rows, count] uint8)."""
    if scores.dim() != 2:
        raise ValueError("scores must be [rows, key blocks]")
    h = None
    if history is not None and history.shape[-1]:
        h = history.to(torch.int32).contiguous()[None]
    ids, origin = assemble_masks(scores.float().contiguous()[None], value_order, [count],
                                 [attention_count], h, max_blocks=max(1, count))
    return ids[0, :, :count].long(), origin[0, :, :count]


def history_update(evidence, ids, counts, keeps, history_len=None):
    """evidence / ids [S, QB, max_blocks] (same-pass evidence and the masks);
    counts / keeps one per slot.  Returns new_history [S, QB, history_len]
    int32: each row's keep ids of largest evidence, ascending, -1 padded."""
    _require_cuda(evidence, ids)
    if evidence.shape != ids.shape or evidence.dim() != 3:
        raise ValueError("evidence and ids must be [slots, query blocks, max_blocks]")
    if evidence.dtype != torch.float32 or ids.dtype != torch.int32:
        raise ValueError("evidence must be float32 and ids int32")
    _require_contig(evidence=evidence, ids=ids)
    s, qb, mb = ids.shape
    dev = ids.device
    cnt = _i32(counts, dev)
    kp = _i32(keeps, dev)
    if history_len is None:
        history_len = max(1, int(torch.as_tensor(keeps).max())) if s else 1
    out = torch.empty((s, qb, history_len), dtype=torch.int32, device=dev)
    lib = _lib.load()
    rc = lib.vggt_history_update(_ptr(evidence), _ptr(ids), s, qb, mb, _ptr(cnt), _ptr(kp),
                                 _ptr(out), history_len, _stream(dev))
    _lib.check(rc)
    return out
