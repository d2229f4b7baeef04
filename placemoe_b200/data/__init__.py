from .synthetic import PinnedBatchPool, SyntheticTokens

__all__ = ["PinnedBatchPool", "SyntheticTokens"]
