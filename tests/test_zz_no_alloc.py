"""semx_linoss_bwd_noalloc: the LinOSS backward for callers that cannot allocate device
memory (for example a real-time audio callback, where cudaMalloc may synchronise the
device and miss the buffer deadline, or a host whose own memory pool owns the GPU).

The entry point takes no workspace; its scratch is a fixed pool inside the library. This
file calls it through the C ABI and checks that it reproduces, bit for bit, the gradients
of the workspace-taking entry point semx_linoss_bwd on two calls in a row, at the largest
problem the pool holds, with a workspace pointer it must ignore, and with L = 0 after a
call that left data in the pool; and (on the CPU) that a problem too big for the pool,
or one whose size would overflow, is refused before anything is launched. It is
collected after every other test file, and it also runs on its own in a fresh process.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

POOL_BYTES = 8 << 20


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


def _dev():
    if not torch.cuda.is_available():
        raise RuntimeError("this test needs a CUDA GPU")
    return torch.device("cuda:0")


def _forward_and_reference(lib, t, S, L, P, chunk, dev, stream):
    """Runs the forward and the workspace-taking backward; returns (Y2, ckpt, dBu, dparams)."""
    from semambaxlinoss_b200 import _lib

    Y2 = torch.empty_like(t["Bu"])
    ckpt = torch.empty(max(1, lib.semx_linoss_ckpt_bytes(S, L, P, chunk) // 4), device=dev)
    a = _args(t, S, L, P, chunk, Y2, ckpt, torch.empty_like(t["Bu"]), torch.zeros(3, P, device=dev))
    _lib.check("semx_linoss_fwd", lib.semx_linoss_fwd(ctypes.byref(a), stream))
    dBu_ref, dp_ref = torch.empty_like(t["Bu"]), torch.zeros(3, P, device=dev)
    a = _args(t, S, L, P, chunk, Y2, ckpt, dBu_ref, dp_ref)
    ws = torch.empty(lib.semx_linoss_workspace_bytes(ctypes.byref(a)) // 4 + 1, device=dev)
    a.workspace = ws.data_ptr()
    _lib.check("semx_linoss_bwd", lib.semx_linoss_bwd(ctypes.byref(a), stream))
    return Y2, ckpt, dBu_ref, dp_ref


def _noalloc(lib, t, S, L, P, chunk, Y2, ckpt, stream, dev, workspace=None):
    from semambaxlinoss_b200 import _lib

    dBu = torch.full_like(t["Bu"], float("nan"))
    dp = torch.full((3, P), float("nan"), device=dev)
    a = _args(t, S, L, P, chunk, Y2, ckpt, dBu, dp)
    if workspace is not None:
        a.workspace = workspace.data_ptr()
    _lib.check("semx_linoss_bwd_noalloc", lib.semx_linoss_bwd_noalloc(ctypes.byref(a), stream))
    torch.cuda.synchronize(dev)
    return dBu, dp


@pytest.mark.gpu
def test_noalloc_backward_matches_workspace_backward():
    from semambaxlinoss_b200 import _lib

    dev = _dev()
    lib = _lib.load()
    stream = torch.cuda.current_stream(dev).cuda_stream
    for S, L, P, chunk, seed in [(37, 100, 48, 16, 1), (300, 21, 256, 8, 2)]:
        t = _problem(S, L, P, seed, dev)
        Y2, ckpt, dBu_ref, dp_ref = _forward_and_reference(lib, t, S, L, P, chunk, dev, stream)
        # Two calls in a row through the scratch-free entry point (workspace left NULL):
        # the same kernels on the same data, so the gradients are bitwise equal.
        for _ in range(2):
            dBu, dp = _noalloc(lib, t, S, L, P, chunk, Y2, ckpt, stream, dev)
            assert torch.equal(dBu, dBu_ref)
            assert torch.equal(dp[:2], dp_ref[:2])


@pytest.mark.gpu
def test_noalloc_at_the_pool_limit_ignoring_a_workspace():
    """The largest sequence count whose scratch fits the pool (P = 256), with a device
    buffer passed as args->workspace: the entry point must neither use nor touch it."""
    from semambaxlinoss_b200 import _lib

    dev = _dev()
    lib = _lib.load()
    stream = torch.cuda.current_stream(dev).cuda_stream
    P, L, chunk = 256, 9, 8
    probe = _lib.new_args(_lib.SemxLinossArgs)
    probe.P = P
    S = 1
    while True:
        probe.S = S + 1
        if lib.semx_linoss_workspace_bytes(ctypes.byref(probe)) > POOL_BYTES:
            break
        S += 1
    probe.S = S
    assert lib.semx_linoss_workspace_bytes(ctypes.byref(probe)) <= POOL_BYTES
    t = _problem(S, L, P, 3, dev)
    Y2, ckpt, dBu_ref, dp_ref = _forward_and_reference(lib, t, S, L, P, chunk, dev, stream)
    decoy = torch.full((1024,), 7.0, device=dev)
    dBu, dp = _noalloc(lib, t, S, L, P, chunk, Y2, ckpt, stream, dev, workspace=decoy)
    assert torch.equal(dBu, dBu_ref)
    assert torch.equal(dp[:2], dp_ref[:2])
    assert torch.equal(decoy, torch.full_like(decoy, 7.0))


@pytest.mark.gpu
def test_noalloc_zero_steps_after_a_call_that_filled_the_pool():
    """L = 0 takes the path that clears the pool's partial rows instead of writing them
    from a kernel; run right after a call that left non-zero partials there, the
    parameter gradients must come back exactly zero."""
    from semambaxlinoss_b200 import _lib

    dev = _dev()
    lib = _lib.load()
    stream = torch.cuda.current_stream(dev).cuda_stream
    S, L, P, chunk = 64, 40, 128, 8
    t = _problem(S, L, P, 4, dev)
    Y2, ckpt, _, dp_ref = _forward_and_reference(lib, t, S, L, P, chunk, dev, stream)
    _, dp = _noalloc(lib, t, S, L, P, chunk, Y2, ckpt, stream, dev)
    assert torch.equal(dp[:2], dp_ref[:2])
    assert dp[:2].abs().max().item() > 0
    t0 = _problem(S, 1, P, 5, dev)
    _, dp0 = _noalloc(lib, t0, S, 0, P, chunk, torch.empty_like(t0["Bu"]),
                      torch.zeros(S * 2 * P * 4, device=dev), stream, dev)
    assert torch.equal(dp0[:2], torch.zeros_like(dp0[:2]))


def test_noalloc_rejects_problems_larger_than_the_pool():
    """Refused on the host before any CUDA call (runs without a GPU)."""
    from semambaxlinoss_b200 import _lib

    lib = _lib.load()
    a = _lib.new_args(_lib.SemxLinossArgs)
    a.variant, a.chunk, a.S, a.L, a.P = _lib.LINOSS_IMEX, 64, 100_000, 10, 256
    assert lib.semx_linoss_workspace_bytes(ctypes.byref(a)) > POOL_BYTES
    assert lib.semx_linoss_bwd_noalloc(ctypes.byref(a), None) == _lib.SEMX_ERR_SHAPE
    assert b"pool" in lib.semx_last_error()
    # Sizes whose scratch byte count would wrap around 2^64 are refused as well.
    a.S, a.P = 1 << 40, 1 << 30
    assert lib.semx_linoss_bwd_noalloc(ctypes.byref(a), None) == _lib.SEMX_ERR_SHAPE
    assert b"pool" in lib.semx_last_error()
