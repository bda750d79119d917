"""vggt_sparse — B200-native (sm_100a) sparse global attention for VGGT-style
multi-view transformers.

Drop-in for the reference operator saf3r.triton.adaptive_block_attention
(``block_attention``), plus the device block-mask estimator, head-profile
dispatch and multi-GPU sharding.  All compute runs in ``libvggt_sparse.so``
(hand-written CUDA for sm_100a behind a C ABI); there is no CPU fallback.
"""
from . import ops  # noqa: F401  (registers torch.ops.vggt_sparse.*)
from ._lib import ExtensionMissing, load as load_library  # noqa: F401
from .assembly import assemble_masks, history_update, select_block_mask  # noqa: F401
from .block_attention import block_attention, check_status  # noqa: F401
from .configs import CONFIGS, LayerConfig  # noqa: F401
from .estimator import BlockMasks, block_mask_estimate, block_select  # noqa: F401
from .frame_topk import compute_qk_topk_indices_fused  # noqa: F401
from .layer import SparseGlobalLayer, topk_budget  # noqa: F401
from .layout import LayerShape, split_keys, token_layout  # noqa: F401
from .pipeline import HostPipeline  # noqa: F401
from .qkv import QkvOut, project_qkv, rope_tables  # noqa: F401
from .token_attention import token_sparse_attention  # noqa: F401
from .profile import (dense_heads_from_decisions, dense_heads_from_profile,  # noqa: F401
                      head_modes_from_profile, split_heads)

__version__ = "1.0.0"
