"""LinOSS layer and scan operators (drop-in for the reference's models/linoss)."""
from .linoss import LinOSS, _map_theta_to_A
from .scan import linoss_scan, linoss_scan_fused, linoss_scan_triton

__all__ = ["LinOSS", "linoss_scan", "linoss_scan_fused", "linoss_scan_triton", "_map_theta_to_A"]
