"""Token layouts on the CPU: the row map of TokenLayout, which layers read which layouts,
and the library's refusal of layouts that reach outside the token rows (host checks that
run before any device access)."""
from __future__ import annotations

import ctypes

import pytest
import torch

from semambaxlinoss_b200 import _lib
from semambaxlinoss_b200.layout import TokenLayout, check_rows


@pytest.mark.parametrize("b,t,f", [(2, 5, 3), (1, 7, 1), (3, 1, 4)])
@pytest.mark.parametrize("reverse", [False, True])
def test_time_axis_rows_are_the_permuted_grid(b, t, f, reverse):
    lay = TokenLayout.time_axis(b, t, f, reverse)
    grid = torch.arange(b * t * f).view(b, t, f).permute(0, 2, 1).reshape(b * f, t)
    if reverse:
        grid = torch.flip(grid, [1])
    rows = [[lay.row(s, k) for k in range(t)] for s in range(lay.S)]
    assert torch.equal(torch.tensor(rows), grid)
    assert sorted(r for rr in rows for r in rr) == list(range(lay.rows))
    assert lay.is_contiguous == (f == 1)


def test_contiguous_and_flipped():
    lay = TokenLayout.contiguous(4, 6)
    assert lay.is_default and lay.is_contiguous
    rev = lay.flipped()
    assert rev.reverse and rev.is_contiguous and not rev.is_default
    assert rev.flipped() == lay
    assert [rev.row(1, k) for k in range(6)] == [11, 10, 9, 8, 7, 6]
    assert TokenLayout.freq_axis(2, 3, 5) == TokenLayout.contiguous(6, 5)
    # A grid that happens to be sequence-major is contiguous.
    assert TokenLayout(6, 5, seq_group=3, group_stride=15, seq_stride=5, step_stride=1).is_contiguous
    with pytest.raises(ValueError):
        check_rows("x", torch.zeros(5, 4), lay)
    check_rows("x", torch.zeros(2, 12, 3), lay)


def _slru_args(S, L, layout):
    a = _lib.new_args(_lib.SemxSelectiveLruArgs)
    a.S, a.L, a.C, a.N, a.chunk, a.real = S, L, 4, 4, 8, 1
    _lib.set_layout(a, layout)
    return a


def _conv_args(S, L, layout):
    a = _lib.new_args(_lib.SemxConvSiluArgs)
    a.S, a.L, a.C, a.ld, a.K, a.left = S, L, 4, 8, 4, 3
    _lib.set_layout(a, layout)
    return a


@pytest.mark.parametrize("entry,build", [("semx_selective_lru_fwd", _slru_args),
                                         ("semx_selective_lru_bwd", _slru_args),
                                         ("semx_conv_silu_fwd", _conv_args),
                                         ("semx_conv_silu_bwd", _conv_args)])
def test_library_refuses_layouts_outside_the_rows(entry, build):
    lib = _lib.load()
    fn = getattr(lib, entry)
    cases = [
        # rows past S * L: (5 // 3) * 16 + 2 + 4 * 3 = 30 >= 30
        TokenLayout(6, 5, seq_group=3, group_stride=16, seq_stride=1, step_stride=3),
        # S not a multiple of the group
        TokenLayout(6, 5, seq_group=4, group_stride=20, seq_stride=1, step_stride=4),
        # a negative field
        TokenLayout(6, 5, seq_group=3, group_stride=-1, seq_stride=1, step_stride=3),
        # a field large enough to wrap 64-bit arithmetic
        TokenLayout(6, 5, seq_group=3, group_stride=1 << 62, seq_stride=1, step_stride=3),
    ]
    for lay in cases:
        assert fn(ctypes.byref(build(6, 5, lay)), None) == _lib.SEMX_ERR_SHAPE, lay
        assert b"layout" in lib.semx_last_error() or b"seq_group" in lib.semx_last_error()
    # The valid time-axis grid passes the layout check and stops at the missing pointers.
    ok = TokenLayout.time_axis(2, 5, 3)
    assert fn(ctypes.byref(build(6, 5, ok)), None) == _lib.SEMX_ERR_NULL


def test_which_layers_read_which_layouts():
    from semambaxlinoss_b200.linoss import LinOSS
    from semambaxlinoss_b200.mamba_block import MambaBlock, TFMambaBlock
    from semambaxlinoss_b200.selective_lru import SelectiveLRU, SelectiveLRUMIMO

    time = TokenLayout.time_axis(2, 5, 3)
    rev = TokenLayout.contiguous(4, 5, reverse=True)
    slru = SelectiveLRU(8, 4)
    assert slru.accepts_layout(time) and slru.accepts_layout(rev) and slru.accepts_layout(time.flipped())
    slru.stream_chunk = 16
    assert not slru.accepts_layout(time) and slru.accepts_layout(TokenLayout.contiguous(4, 5))
    lin = LinOSS(8, 4)
    assert lin.accepts_layout(rev) and not lin.accepts_layout(time)
    mimo = SelectiveLRUMIMO(8, 4, n_heads=2)
    assert not mimo.accepts_layout(rev) and mimo.accepts_layout(TokenLayout.contiguous(4, 5))

    def cfg(ssm):
        return dict(ssm=ssm, d_state=4, d_conv=4, expand=2, bidirectional=True, ssm_params={})

    assert MambaBlock(8, cfg("selective_lru")).accepts_layout(time)
    assert not MambaBlock(8, cfg("linoss")).accepts_layout(time)
    assert MambaBlock(8, cfg("linoss")).accepts_layout(TokenLayout.contiguous(4, 5))
    assert not MambaBlock(8, cfg("selective_lru_mimo")).accepts_layout(time)
    tf = TFMambaBlock({"model_cfg": dict(hid_feature=8, time_mixer=cfg("selective_lru"),
                                         freq_mixer=cfg("linoss"))})
    assert tf.time_mamba.accepts_layout(time)
