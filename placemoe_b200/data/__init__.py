from .packing import PackedSyntheticTokens, pack_documents
from .synthetic import PinnedBatchPool, SyntheticTokens

__all__ = ["PackedSyntheticTokens", "PinnedBatchPool", "SyntheticTokens", "pack_documents"]
