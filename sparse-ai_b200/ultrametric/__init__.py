"""B200-native (sm_100a) block-sparse attention with sparse-ai's ``ultrametric`` operator
surface: routing -> block lists, block-list prefill forward/backward, routed paged decode.

Only the hot-path modules of the reference package are provided (``block_list``,
``kernel``, ``kernel_decode``); the toy models and routers of the reference
(``topology``, ``layer``, ``model``) are outside this library.
"""

from .block_list import (
    HAS_TRITON,
    BlockLists,
    block_list_attention,
    build_block_lists,
    build_block_lists_from_mask,
    build_transposed_block_lists,
    routed_block_attention,
)
from .kernel import (
    CurriculumSparseAttention,
    block_sparse_attention,
    routing_to_block_indices,
    ultrametric_attention_triton,
)
from .kernel_decode import ultrametric_decode

__all__ = [
    "HAS_TRITON",
    "BlockLists",
    "build_block_lists",
    "build_block_lists_from_mask",
    "build_transposed_block_lists",
    "block_list_attention",
    "routed_block_attention",
    "block_sparse_attention",
    "routing_to_block_indices",
    "ultrametric_attention_triton",
    "CurriculumSparseAttention",
    "ultrametric_decode",
]
