"""KV-cache eviction selection (``cab_attention/eviction`` of the reference)."""

from .policy import EvictionConfig, ThreeComponentEvictionPolicy, select_indices_batched  # noqa: F401
