"""semx_linoss_bwd_noalloc: the LinOSS backward for callers that cannot allocate device
memory (for example a real-time audio callback, where cudaMalloc may synchronise the
device and miss the buffer deadline, or a host whose own memory pool owns the GPU).

The entry point takes no workspace; its scratch is a fixed pool inside the library. This
file calls it through the C ABI and checks that two calls in a row reproduce the
gradients of the workspace-taking entry point semx_linoss_bwd, and that a problem too big
for the pool is refused before anything is launched. It is collected after every other
test file, and it also runs on its own in a fresh process.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from tests.parity import FP32_TOL, assert_close

pytestmark = pytest.mark.gpu


def _problem(S, L, P, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    return {
        "steps": torch.randn(P, generator=g, device=dev),
        "A": torch.randn(P, generator=g, device=dev),
        "Bu": torch.randn(S, L, P, dtype=torch.complex64, generator=g, device=dev),
        "dY2": torch.randn(S, L, P, dtype=torch.complex64, generator=g, device=dev),
    }


def _args(t, S, L, P, chunk, Y2, ckpt, dBu, dparams):
    from semambaxlinoss_b200 import _lib

    a = _lib.new_args(_lib.SemxLinossArgs)
    a.variant, a.a_from_g, a.chunk, a.S, a.L, a.P = _lib.LINOSS_IMEX, 1, chunk, S, L, P
    a.steps, a.A_diag, a.Bu = t["steps"].data_ptr(), t["A"].data_ptr(), t["Bu"].data_ptr()
    a.Y2, a.ckpt, a.dY2 = Y2.data_ptr(), ckpt.data_ptr(), t["dY2"].data_ptr()
    a.dBu, a.dparams = dBu.data_ptr(), dparams.data_ptr()
    return a


def test_noalloc_backward_matches_workspace_backward():
    from semambaxlinoss_b200 import _lib

    if not torch.cuda.is_available():
        raise RuntimeError("this test needs a CUDA GPU")
    dev = torch.device("cuda:0")
    lib = _lib.load()
    stream = torch.cuda.current_stream(dev).cuda_stream
    for S, L, P, chunk, seed in [(37, 100, 48, 16, 1), (300, 21, 256, 8, 2)]:
        t = _problem(S, L, P, seed, dev)
        Y2 = torch.empty_like(t["Bu"])
        ckpt = torch.empty(lib.semx_linoss_ckpt_bytes(S, L, P, chunk) // 4, device=dev)
        a = _args(t, S, L, P, chunk, Y2, ckpt, torch.empty_like(t["Bu"]), torch.zeros(3, P, device=dev))
        _lib.check("semx_linoss_fwd", lib.semx_linoss_fwd(ctypes.byref(a), stream))

        # Gradients from the entry point that takes a caller-allocated workspace.
        dBu_ref, dp_ref = torch.empty_like(t["Bu"]), torch.zeros(3, P, device=dev)
        a = _args(t, S, L, P, chunk, Y2, ckpt, dBu_ref, dp_ref)
        ws = torch.empty(lib.semx_linoss_workspace_bytes(ctypes.byref(a)) // 4 + 1, device=dev)
        a.workspace = ws.data_ptr()
        _lib.check("semx_linoss_bwd", lib.semx_linoss_bwd(ctypes.byref(a), stream))

        # Two calls in a row through the scratch-free entry point (workspace left NULL).
        for _ in range(2):
            dBu = torch.full_like(t["Bu"], float("nan"))
            dp = torch.full((3, P), float("nan"), device=dev)
            a = _args(t, S, L, P, chunk, Y2, ckpt, dBu, dp)
            _lib.check("semx_linoss_bwd_noalloc", lib.semx_linoss_bwd_noalloc(ctypes.byref(a), stream))
            torch.cuda.synchronize(dev)
            assert_close(dBu, dBu_ref, FP32_TOL, "dBu")
            assert_close(dp[:2], dp_ref[:2], FP32_TOL, "d steps / d A_diag")


def test_noalloc_rejects_problems_larger_than_the_pool():
    from semambaxlinoss_b200 import _lib

    lib = _lib.load()
    a = _lib.new_args(_lib.SemxLinossArgs)
    a.variant, a.chunk, a.S, a.L, a.P = _lib.LINOSS_IMEX, 64, 100_000, 10, 256
    assert lib.semx_linoss_workspace_bytes(ctypes.byref(a)) > (8 << 20)
    assert lib.semx_linoss_bwd_noalloc(ctypes.byref(a), None) == _lib.SEMX_ERR_SHAPE
    assert b"pool" in lib.semx_last_error()
