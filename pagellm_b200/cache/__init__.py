"""Drop-in for pagellm's ``pagellm.cache`` paged KV cache, backed by libpagekv (CUDA, sm_100a)."""

from .block_manager import BlockAllocator, BlockManager, BlockTable, OutOfBlocks, block_hash
from .paged import PagedBatch, PagedKVPool, batched_decode_attention, paged_attention, slot_mapping

__all__ = [
    "BlockAllocator",
    "BlockManager",
    "BlockTable",
    "OutOfBlocks",
    "PagedBatch",
    "PagedKVPool",
    "batched_decode_attention",
    "block_hash",
    "paged_attention",
    "slot_mapping",
]
