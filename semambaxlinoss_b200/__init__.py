"""semambaxlinoss_b200 — B200-native (sm_100a) recurrent scans of the SEMamba TF-blocks.

Drop-in layers for a-baur/SEMambaXLinOSS's hot path (selective-LRU SISO / MIMO and
LinOSS scans, forward and backward) running on hand-written CUDA kernels reached through
the C ABI in include/semx.h (libsemx.so, loaded with ctypes).
"""
__version__ = "0.1.0"
