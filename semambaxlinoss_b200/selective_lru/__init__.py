"""Selective-LRU layers and scan operators (drop-in for the reference's models/selective_lru)."""
from .mimo import (
    drive_weight,
    fused_selective_lru_mimo,
    mimo_layer,
    proj_width,
    selective_scan,
    selective_scan_real,
    selective_scan_triton,
    selective_scan_triton_real,
)
from .scan import fused_selective_lru, fused_selective_lru_real
from .selective_lru import SelectiveLRU, SelectiveLRUMIMO

__all__ = [
    "SelectiveLRU", "SelectiveLRUMIMO", "fused_selective_lru", "fused_selective_lru_real",
    "fused_selective_lru_mimo", "selective_scan", "selective_scan_real",
    "selective_scan_triton", "selective_scan_triton_real", "mimo_layer", "proj_width",
    "drive_weight",
]
