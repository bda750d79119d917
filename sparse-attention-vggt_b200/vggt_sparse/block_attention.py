"""Drop-in replacement for saf3r.triton.adaptive_block_attention.block_attention.

Same signature, argument meaning and return value as the reference
(saf3r/triton/adaptive_block_attention.py:63-83): inputs contiguous
[H, N, d] bf16/fp16 CUDA tensors, ``indices`` int32 [sparseH, ceil(N/BQ), maxK]
of unique patch-block ids of which the first ``counts[s]`` are read,
``head_ids`` int32 [sparseH]; returns ``(out, evidence)`` where only the rows of
the selected heads of ``out`` are written and ``evidence`` is fp32 with -inf in
unused slots.  A ValueError is raised for non-BF16/FP16 inputs, as in the
reference; unlike the reference, malformed shapes, counts, heads and ids are
also rejected (ValueError) instead of reading out of bounds.

Like the reference, a call only enqueues work on the current CUDA stream and
returns without waiting for the GPU.  Errors the kernel finds on the device
(bad ids, counts, head ids) are ORed into a per-device status word that is
copied to pinned host memory behind each call; a later call (or
``check_status``) raises the ValueError once that copy has landed, so the
default path never blocks the host.  ``validate=True`` keeps the old
synchronous check (one host sync per call, the error raised by the faulty
call itself); ``validate=False`` skips status reporting entirely.
"""
import math
import threading

import torch

from . import _lib, ops

_RING = 32  # status copies in flight per device before a call waits for the oldest


class _StatusMonitor:
    """The device status word of one GPU and the pinned copies of it that
    calls enqueue; completed copies are inspected without blocking."""

    def __init__(self, device):
        self.word = torch.zeros(1, device=device, dtype=torch.int32)
        self.host = torch.zeros(_RING, dtype=torch.int32).pin_memory()
        self.events = [None] * _RING
        self.next = 0

    def _drain(self, wait):
        bits = 0
        for j, ev in enumerate(self.events):
            if ev is None:
                continue
            if wait:
                ev.synchronize()
            elif not ev.query():
                continue
            bits |= int(self.host[j])
            self.events[j] = None
        return bits

    def _raise(self, bits):
        # the error is reported once: reset the word and forget copies in flight
        self.events = [None] * _RING
        self.word.zero_()
        raise ValueError("block_attention (an earlier call on %s): %s"
                         % (self.word.device, _status_message(bits)))

    def poll(self, wait=False):
        bits = self._drain(wait)
        if bits:
            self._raise(bits)

    def enqueue_copy(self):
        j = self.next
        self.next = (j + 1) % _RING
        ev = self.events[j]
        if ev is not None:  # ring full: the oldest copy must land before reuse
            ev.synchronize()
            bits = int(self.host[j])
            self.events[j] = None
            if bits:
                self._raise(bits)
        self.host[j:j + 1].copy_(self.word, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        self.events[j] = ev


_monitors = {}
_monitors_lock = threading.Lock()


def _monitor(device):
    key = device.index if device.index is not None else torch.cuda.current_device()
    with _monitors_lock:
        m = _monitors.get(key)
        if m is None:
            m = _monitors[key] = _StatusMonitor(torch.device("cuda", key))
    return m


def check_status(device=None, wait=True):
    """Raise ValueError if any earlier deferred-validation call on ``device``
    (default: the current device) found bad ids, counts or head ids.  With
    ``wait`` (default) it first waits for every pending status copy."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None \
        else torch.device(device)
    _monitor(dev).poll(wait=wait)


def _status_message(bits):
    parts = []
    if bits & _lib.STATUS_BAD_INDEX:
        parts.append("a selected block id is outside [0, n_blocks)")
    if bits & _lib.STATUS_BAD_COUNT:
        parts.append("a count is negative or exceeds indices.shape[-1]")
    if bits & _lib.STATUS_BAD_HEAD:
        parts.append("a head id is outside [0, heads)")
    if bits & _lib.STATUS_TIMEOUT:
        parts.append("a device pipeline wait timed out")
    return "; ".join(parts)


def block_attention(q, patch_k, patch_v, special_k, special_v, indices, counts, head_ids, *,
                    query_block=64, key_block=64, scale=None, out=None, head_dense=None,
                    return_evidence=True, kernel="auto", validate="deferred"):
    """Shared-within-query-block, head-specific exact sparse attention.

    Extensions beyond the reference signature (all keyword-only, defaults
    keep the reference behaviour): ``counts`` may be [sparseH, n_qblocks];
    ``head_dense`` [sparseH] bool routes a slot to the dense path of the same
    kernel; ``return_evidence=False`` skips the evidence pass (evidence is
    then all -inf); ``kernel`` picks 'auto' | 'tcgen05' | 'mma_sync';
    ``validate``: "deferred" (default) reports a bad id, count or head as a
    ValueError from a later call or ``check_status`` without blocking the
    host; True reads the status back now (one host sync) and raises from
    this call; False reports nothing.  Use "deferred" or False inside CUDA
    graph capture.
    """
    if validate not in (True, False, "deferred"):
        raise ValueError("validate must be True, False or 'deferred'")
    if q.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError('Tensor-core sparse execution requires BF16 or FP16')
    h, n, d = q.shape
    if out is None:
        out = torch.empty_like(q)
    evidence = torch.full(indices.shape, -math.inf, device=q.device, dtype=torch.float32)
    monitor = None
    status = None
    if validate == "deferred" and q.is_cuda:  # CPU tensors are rejected by the launcher
        monitor = _monitor(q.device)
        if not torch.cuda.is_current_stream_capturing():
            monitor.poll()  # errors of earlier calls whose status copy has landed
        status = monitor.word
    elif validate is True:
        status = torch.zeros(1, device=q.device, dtype=torch.int32)
    if special_k is None:
        special_k = q.new_empty((h, 0, d))
        special_v = q.new_empty((h, 0, d))
    ops.launch_block_attention(q, patch_k, patch_v, special_k, special_v, indices, counts,
                               head_ids, head_dense=head_dense, query_block=query_block,
                               key_block=key_block, scale=scale, out=out,
                               evidence=evidence if return_evidence else None, status=status,
                               kernel=kernel)
    if monitor is not None:
        if not torch.cuda.is_current_stream_capturing():
            monitor.enqueue_copy()
    elif validate is True:
        bits = int(status.item())
        if bits:
            raise ValueError("block_attention: " + _status_message(bits))
    return out, evidence
