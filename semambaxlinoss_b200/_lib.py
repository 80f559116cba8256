"""ctypes binding of ``libsemx.so`` (declared in ``include/semx.h``).

This is the only place Python touches the C ABI. It mirrors the argument structs,
checks at load time that the library's struct sizes and ABI version match these
mirrors, and turns non-zero status codes into Python exceptions. There is no fallback:
if the library is missing or a call fails, the caller gets an exception.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

import os

# The in-tree library; SEMX_LIB may name another build of the same ABI (e.g. to compare
# builds side by side).
LIB_PATH = Path(os.environ.get("SEMX_LIB", Path(__file__).resolve().parent / "libsemx.so"))
ABI_VERSION = 2

c_f32p = ctypes.POINTER(ctypes.c_float)

# Status codes (enum semx_status).
SEMX_OK = 0
SEMX_ERR_ABI = 1
SEMX_ERR_NULL = 2
SEMX_ERR_SHAPE = 3
SEMX_ERR_UNSUPPORTED = 4
SEMX_ERR_ALIGN = 5
SEMX_ERR_LAUNCH = 6
SEMX_ERR_WORKSPACE = 7
SEMX_ERR_DEVICE = 8

# enum semx_linoss_variant
LINOSS_GENERIC = 0
LINOSS_IM = 1
LINOSS_IMEX = 2
LINOSS_DAMPED_IMEX = 3


class SemxError(RuntimeError):
    """A semx entry point returned a non-zero status."""

    def __init__(self, fn: str, status: int, message: str):
        super().__init__(f"{fn} failed with status {status}: {message}")
        self.status = status


class SemxLinossArgs(ctypes.Structure):
    _fields_ = [
        ("struct_size", ctypes.c_uint32),
        ("variant", ctypes.c_int32),
        ("a_from_g", ctypes.c_int32),
        ("chunk", ctypes.c_int32),
        ("S", ctypes.c_int64),
        ("L", ctypes.c_int64),
        ("P", ctypes.c_int64),
        ("M11", ctypes.c_void_p),
        ("M12", ctypes.c_void_p),
        ("M21", ctypes.c_void_p),
        ("M22", ctypes.c_void_p),
        ("F1", ctypes.c_void_p),
        ("F2", ctypes.c_void_p),
        ("steps", ctypes.c_void_p),
        ("A_diag", ctypes.c_void_p),
        ("G_diag", ctypes.c_void_p),
        ("Bu", ctypes.c_void_p),
        ("Y2", ctypes.c_void_p),
        ("ckpt", ctypes.c_void_p),
        ("dY2", ctypes.c_void_p),
        ("dF1", ctypes.c_void_p),
        ("dF2", ctypes.c_void_p),
        ("dBu", ctypes.c_void_p),
        ("dM", ctypes.c_void_p),
        ("dparams", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p),
        ("reverse", ctypes.c_int32),
    ]


# enum semx_input_gain
GAIN_CODES = {"gamma": 0, "mamba": 1, "zoh": 2, "none": 3}


# Token layout fields shared by the selective-LRU and conv + SiLU argument structs.
_LAYOUT_FIELDS = [
    ("reverse", ctypes.c_int32),
    ("seq_group", ctypes.c_int64),
    ("group_stride", ctypes.c_int64),
    ("seq_stride", ctypes.c_int64),
    ("step_stride", ctypes.c_int64),
]


def set_layout(args, layout) -> None:
    """Copies a TokenLayout (or None: the default sequence-major layout) into an argument
    struct's layout fields."""
    if layout is None:
        return
    args.reverse = int(layout.reverse)
    args.seq_group, args.group_stride = layout.seq_group, layout.group_stride
    args.seq_stride, args.step_stride = layout.seq_stride, layout.step_stride


class SemxSelectiveLruArgs(ctypes.Structure):
    _fields_ = [
        ("struct_size", ctypes.c_uint32),
        ("real", ctypes.c_int32),
        ("input_gain", ctypes.c_int32),
        ("chunk", ctypes.c_int32),
        ("S", ctypes.c_int64),
        ("L", ctypes.c_int64),
        ("C", ctypes.c_int64),
        ("N", ctypes.c_int64),
    ] + [(name, ctypes.c_void_p) for name in (
        "delta_nu", "delta_theta", "a", "omega", "B_re", "B_im", "C_re", "C_im", "x", "D",
        "g", "s", "h0_re", "h0_im", "y", "hf_re", "hf_im", "ckpt", "dy", "dhf_re", "dhf_im",
        "d_delta_nu", "d_delta_theta", "dx", "dB_re", "dB_im", "dC_re", "dC_im", "da",
        "domega", "dD", "dg", "ds", "dh0_re", "dh0_im", "workspace",
    )] + _LAYOUT_FIELDS


class SemxComplexScanArgs(ctypes.Structure):
    _fields_ = [
        ("struct_size", ctypes.c_uint32),
        ("reserved", ctypes.c_int32),
        ("S", ctypes.c_int64),
        ("L", ctypes.c_int64),
        ("N", ctypes.c_int64),
    ] + [(name, ctypes.c_void_p) for name in (
        "lam_re", "lam_im", "Bu_re", "Bu_im", "h_re", "h_im", "dh_re", "dh_im",
        "dlam_re", "dlam_im", "dBu_re", "dBu_im",
    )]


class SemxMimoArgs(ctypes.Structure):
    _fields_ = [
        ("struct_size", ctypes.c_uint32),
        ("reserved", ctypes.c_int32),
        ("S", ctypes.c_int64),
        ("L", ctypes.c_int64),
        ("H", ctypes.c_int64),
        ("Nh", ctypes.c_int64),
        ("Fh", ctypes.c_int64),
    ] + [(name, ctypes.c_void_p) for name in (
        "lam_re", "lam_im", "Bu_re", "Bu_im", "C_re", "C_im", "x", "D", "y", "h_re", "h_im",
        "dy", "dh_re", "dh_im", "dlam_re", "dlam_im", "dBu_re", "dBu_im", "dx", "dC_re",
        "dC_im", "dD", "workspace",
    )]


class SemxMimoLayerArgs(ctypes.Structure):
    _fields_ = [
        ("struct_size", ctypes.c_uint32),
        ("input_gain", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("detune", ctypes.c_int32),
        ("envelope", ctypes.c_int32),
        ("bf16", ctypes.c_int32),
        ("rate_scale", ctypes.c_float),
        ("reserved", ctypes.c_int32),
        ("S", ctypes.c_int64),
        ("L", ctypes.c_int64),
        ("H", ctypes.c_int64),
        ("Nh", ctypes.c_int64),
        ("Fh", ctypes.c_int64),
    ] + [(name, ctypes.c_void_p) for name in (
        "x", "proj", "A_log", "omega", "detune_gain", "C", "D", "c_out", "env_gain", "dt_bias",
        "y", "ckpt", "dy", "dx", "dproj", "dA_log", "domega", "ddetune", "dC", "dD", "dc_out",
        "denv", "d_dt_bias", "workspace",
    )]


class SemxConvSiluArgs(ctypes.Structure):
    _fields_ = [
        ("struct_size", ctypes.c_uint32),
        ("K", ctypes.c_int32),
        ("left", ctypes.c_int32),
        ("bf16", ctypes.c_int32),
        ("S", ctypes.c_int64),
        ("L", ctypes.c_int64),
        ("C", ctypes.c_int64),
        ("ld", ctypes.c_int64),
    ] + [(name, ctypes.c_void_p) for name in ("xz", "w", "b", "v", "dv", "dxz", "dw", "db", "workspace")] + \
        _LAYOUT_FIELDS


class SemxGateSiluArgs(ctypes.Structure):
    _fields_ = [
        ("struct_size", ctypes.c_uint32),
        ("bf16", ctypes.c_int32),
        ("n", ctypes.c_int64),
        ("C", ctypes.c_int64),
        ("ld", ctypes.c_int64),
    ] + [(name, ctypes.c_void_p) for name in ("y", "xz", "o", "dout", "dy", "dxz")]


class SemxRmsNormArgs(ctypes.Structure):
    _fields_ = [
        ("struct_size", ctypes.c_uint32),
        ("bf16", ctypes.c_int32),
        ("eps", ctypes.c_float),
        ("reserved", ctypes.c_int32),
        ("n", ctypes.c_int64),
        ("d", ctypes.c_int64),
    ] + [(name, ctypes.c_void_p) for name in ("x", "weight", "y", "rstd", "dy", "dx", "dweight", "workspace")]


class SemxStepProjArgs(ctypes.Structure):
    _fields_ = [
        ("struct_size", ctypes.c_uint32),
        ("bf16", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("scale", ctypes.c_float),
        ("rows", ctypes.c_int64),
        ("C", ctypes.c_int64),
        ("ldz", ctypes.c_int64),
    ] + [(n, ctypes.c_void_p) for n in (
        "z_nu", "z_th", "W_nu", "b_nu", "W_th", "b_th", "delta_nu", "delta_th",
        "d_delta_nu", "d_delta_th", "dz_nu", "dz_th", "dW_nu", "db_nu", "dW_th", "db_th",
        "workspace")]


class SemxLinossReadoutArgs(ctypes.Structure):
    _fields_ = [
        ("struct_size", ctypes.c_uint32),
        ("reserved", ctypes.c_int32),
        ("rows", ctypes.c_int64),
        ("H", ctypes.c_int64),
        ("P", ctypes.c_int64),
    ] + [(n, ctypes.c_void_p) for n in ("x", "y2", "C", "D", "y", "dy", "dx", "dC", "dD", "workspace")]


# (python struct, C size query) for every argument struct in semx.h.
STRUCTS = {
    "SemxLinossArgs": (SemxLinossArgs, "semx_linoss_args_size"),
    "SemxSelectiveLruArgs": (SemxSelectiveLruArgs, "semx_selective_lru_args_size"),
    "SemxComplexScanArgs": (SemxComplexScanArgs, "semx_complex_scan_args_size"),
    "SemxMimoArgs": (SemxMimoArgs, "semx_mimo_args_size"),
    "SemxMimoLayerArgs": (SemxMimoLayerArgs, "semx_mimo_layer_args_size"),
    "SemxConvSiluArgs": (SemxConvSiluArgs, "semx_conv_silu_args_size"),
    "SemxGateSiluArgs": (SemxGateSiluArgs, "semx_gate_silu_args_size"),
    "SemxRmsNormArgs": (SemxRmsNormArgs, "semx_rms_norm_args_size"),
    "SemxStepProjArgs": (SemxStepProjArgs, "semx_step_proj_args_size"),
    "SemxLinossReadoutArgs": (SemxLinossReadoutArgs, "semx_linoss_readout_args_size"),
}

# Every symbol semx.h declares, with its ctypes signature.
_SIGNATURES = {
    "semx_abi_version": (ctypes.c_int, []),
    "semx_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "semx_last_error": (ctypes.c_char_p, []),
    "semx_launch_count": (ctypes.c_uint64, []),
    "semx_tc_timeouts": (ctypes.c_int, [ctypes.POINTER(ctypes.c_uint32)]),
    "semx_linoss_args_size": (ctypes.c_size_t, []),
    "semx_linoss_ckpt_bytes": (
        ctypes.c_size_t,
        [ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int32],
    ),
    "semx_linoss_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(SemxLinossArgs)]),
    "semx_linoss_fwd": (ctypes.c_int, [ctypes.POINTER(SemxLinossArgs), ctypes.c_void_p]),
    "semx_linoss_bwd": (ctypes.c_int, [ctypes.POINTER(SemxLinossArgs), ctypes.c_void_p]),
    "semx_linoss_bwd_noalloc": (ctypes.c_int, [ctypes.POINTER(SemxLinossArgs), ctypes.c_void_p]),
    "semx_selective_lru_args_size": (ctypes.c_size_t, []),
    "semx_selective_lru_ckpt_bytes": (ctypes.c_size_t, [ctypes.POINTER(SemxSelectiveLruArgs)]),
    "semx_selective_lru_workspace_bytes": (
        ctypes.c_size_t, [ctypes.POINTER(SemxSelectiveLruArgs)]),
    "semx_selective_lru_fwd": (
        ctypes.c_int, [ctypes.POINTER(SemxSelectiveLruArgs), ctypes.c_void_p]),
    "semx_selective_lru_bwd": (
        ctypes.c_int, [ctypes.POINTER(SemxSelectiveLruArgs), ctypes.c_void_p]),
    "semx_complex_scan_args_size": (ctypes.c_size_t, []),
    "semx_complex_scan_fwd": (
        ctypes.c_int, [ctypes.POINTER(SemxComplexScanArgs), ctypes.c_void_p]),
    "semx_complex_scan_bwd": (
        ctypes.c_int, [ctypes.POINTER(SemxComplexScanArgs), ctypes.c_void_p]),
    "semx_mimo_args_size": (ctypes.c_size_t, []),
    "semx_mimo_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(SemxMimoArgs)]),
    "semx_mimo_fwd": (ctypes.c_int, [ctypes.POINTER(SemxMimoArgs), ctypes.c_void_p]),
    "semx_mimo_bwd": (ctypes.c_int, [ctypes.POINTER(SemxMimoArgs), ctypes.c_void_p]),
    "semx_conv_silu_args_size": (ctypes.c_size_t, []),
    "semx_conv_silu_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(SemxConvSiluArgs)]),
    "semx_conv_silu_fwd": (ctypes.c_int, [ctypes.POINTER(SemxConvSiluArgs), ctypes.c_void_p]),
    "semx_conv_silu_bwd": (ctypes.c_int, [ctypes.POINTER(SemxConvSiluArgs), ctypes.c_void_p]),
    "semx_gate_silu_args_size": (ctypes.c_size_t, []),
    "semx_gate_silu_fwd": (ctypes.c_int, [ctypes.POINTER(SemxGateSiluArgs), ctypes.c_void_p]),
    "semx_gate_silu_bwd": (ctypes.c_int, [ctypes.POINTER(SemxGateSiluArgs), ctypes.c_void_p]),
    "semx_rms_norm_args_size": (ctypes.c_size_t, []),
    "semx_rms_norm_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(SemxRmsNormArgs)]),
    "semx_rms_norm_fwd": (ctypes.c_int, [ctypes.POINTER(SemxRmsNormArgs), ctypes.c_void_p]),
    "semx_rms_norm_bwd": (ctypes.c_int, [ctypes.POINTER(SemxRmsNormArgs), ctypes.c_void_p]),
    "semx_step_proj_args_size": (ctypes.c_size_t, []),
    "semx_step_proj_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(SemxStepProjArgs)]),
    "semx_step_proj_fwd": (ctypes.c_int, [ctypes.POINTER(SemxStepProjArgs), ctypes.c_void_p]),
    "semx_step_proj_bwd": (ctypes.c_int, [ctypes.POINTER(SemxStepProjArgs), ctypes.c_void_p]),
    "semx_linoss_readout_args_size": (ctypes.c_size_t, []),
    "semx_linoss_readout_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(SemxLinossReadoutArgs)]),
    "semx_linoss_readout_fwd": (ctypes.c_int, [ctypes.POINTER(SemxLinossReadoutArgs), ctypes.c_void_p]),
    "semx_linoss_readout_bwd": (ctypes.c_int, [ctypes.POINTER(SemxLinossReadoutArgs), ctypes.c_void_p]),
    "semx_mimo_layer_args_size": (ctypes.c_size_t, []),
    "semx_mimo_layer_ckpt_bytes": (ctypes.c_size_t, [ctypes.POINTER(SemxMimoLayerArgs)]),
    "semx_mimo_layer_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(SemxMimoLayerArgs)]),
    "semx_mimo_layer_fwd": (ctypes.c_int, [ctypes.POINTER(SemxMimoLayerArgs), ctypes.c_void_p]),
    "semx_mimo_layer_bwd": (ctypes.c_int, [ctypes.POINTER(SemxMimoLayerArgs), ctypes.c_void_p]),
}

_lib = None
_lock = threading.Lock()


def declared_symbols() -> list[str]:
    return sorted(_SIGNATURES)


def load() -> ctypes.CDLL:
    """Loads and checks ``libsemx.so``; raises if it is missing or mismatched."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"semx CUDA library not found at {LIB_PATH}; build it with "
                "`python -m semambaxlinoss_b200.build` (or __graft_entry__.build())"
            )
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, argtypes) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = argtypes
        if lib.semx_abi_version() != ABI_VERSION:
            raise RuntimeError(
                f"libsemx ABI version {lib.semx_abi_version()} != binding {ABI_VERSION}"
            )
        for sname, (cls, query) in STRUCTS.items():
            if getattr(lib, query)() != ctypes.sizeof(cls):
                raise RuntimeError(
                    f"{sname}: library size {getattr(lib, query)()} != binding "
                    f"{ctypes.sizeof(cls)}"
                )
        _lib = lib
        return lib


def check(fn: str, status: int) -> None:
    if status != SEMX_OK:
        lib = load()
        msg = lib.semx_last_error().decode(errors="replace")
        raise SemxError(fn, status, msg or lib.semx_status_string(status).decode())


def ptr(t: torch.Tensor | None) -> int | None:
    """Device address of a tensor's storage (None for a missing optional tensor)."""
    if t is None:
        return None
    return t.data_ptr()


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def call(fn_name: str, args, device) -> None:
    """Runs a semx entry point on the current stream of `device`; raises on failure."""
    lib = load()
    status = getattr(lib, fn_name)(ctypes.byref(args), stream_handle(device))
    check(fn_name, status)


def empty_f32(nbytes: int, device) -> torch.Tensor:
    """Scratch of at least `nbytes` (never zero-sized, so the pointer is never NULL)."""
    return torch.empty(max((nbytes + 3) // 4, 1), dtype=torch.float32, device=device)


def new_args(cls):
    a = cls()
    a.struct_size = ctypes.sizeof(cls)
    return a


def launch_count() -> int:
    """Kernels the library has launched in this process so far (all threads, devices)."""
    return int(load().semx_launch_count())


def tc_timeouts(device=None) -> int:
    """Tensor-core completion waits that ran out of time on `device` (default: current) in
    this process; 0 in a healthy run."""
    if device is not None:
        torch.cuda.set_device(device)
    n = ctypes.c_uint32(0)
    check("semx_tc_timeouts", load().semx_tc_timeouts(ctypes.byref(n)))
    return int(n.value)
