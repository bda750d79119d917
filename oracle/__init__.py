"""CPU oracle for the vggt_sparse hot path — TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the reference's algorithms for the sparse
global-attention path of Liangyu-Xiang/Sparse-Attention-VGGT (SAF3R):

* ``estimator``  block mean pooling, pooled scores, top-k / mass selection
  (saf3r/patch/adaptive_block_value.py:16-23, :54-56, :170;
  saf3r/patch/coarse_sensing.py:25-31; saf3r/patch/region_history_attention.py:39-42)
* ``attention``  fp32 block-sparse attention with specials and same-pass
  evidence (saf3r/patch/adaptive_block_value.py:371-385;
  saf3r/triton/adaptive_block_attention.py:7-60; tests/test_adaptive_block_value.py:172-184)
* ``layout``     frame-major patch/special split
  (saf3r/patch/value_evolving_attention.py:17-20)
* ``assembly``   select_block_mask with history and value order, and the
  same-pass history update (saf3r/patch/adaptive_block_value.py:42-91, :389-396)
* ``token_attention``  per-token sparse attention
  (saf3r/triton/sparse_topk_attention.py:115-166, :261-286)
* ``frame_topk``  per-frame QK top-k (saf3r/triton/fused_qk_topk.py:24-217,
  saf3r/triton/topk_utils.py:24-28)

It is the CHECKER: only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it.
The product package (``vggt_sparse``) never imports it and has no CPU path.

Parity is pinned against golden vectors produced by running the reference's
own functions in the build container (``tests/golden/make_golden.py``).
"""
from .attention import block_sparse_attention, dense_attention  # noqa: F401
from .estimator import (block_mean, pooled_scores, select_mass, select_topk,  # noqa: F401
                        estimate_masks, mass_weights, topk_budget, score_keys)
from .layout import token_layout  # noqa: F401
from .qkv import project_qkv  # noqa: F401
from .token_attention import token_sparse_attention  # noqa: F401
from .frame_topk import qk_topk_per_frame, score_keys32  # noqa: F401
