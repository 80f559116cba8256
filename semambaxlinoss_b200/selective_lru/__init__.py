"""Selective-LRU layers and scan operators (drop-in for the reference's models/selective_lru)."""
from .scan import fused_selective_lru, fused_selective_lru_real
from .selective_lru import SelectiveLRU

__all__ = ["SelectiveLRU", "fused_selective_lru", "fused_selective_lru_real"]
