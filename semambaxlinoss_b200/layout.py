"""Token layouts: where step t of sequence s lives among the rows of a token tensor.

Every per-token tensor a scan reads or writes (x, the selective steps, B_t / C_t, y, the
in_proj output and its gradients) is a (rows, width) matrix. By default the rows are
sequence-major, row = s * L + t, which is what a (S, L, width) contiguous tensor gives.
A :class:`TokenLayout` describes two other orders the kernels read directly, so that the
callers need no copies:

* ``reverse``: the scan visits the rows of a sequence last to first
  (t' = L - 1 - t). A scan of a time-reversed sequence written back in reversed order,
  ``flip(scan(flip(x)))``, equals the reverse scan of x with its output in x's own row
  order, which is how the backward branch of a bi-directional block
  (models/mamba_block.py:387-396 of the reference) runs without its two ``torch.flip``
  copies.
* a row grid: row(s, t) = (s // G) * A + (s % G) * B + t' * C. With the TF-block
  activations kept as one (batch, frames, bins, channels) tensor, the frequency-axis
  sequences are contiguous (the default) and the time-axis sequences are the grid
  G = bins, A = frames * bins, B = 1, C = bins (:meth:`TokenLayout.time_axis`), which
  removes the permute + contiguous copies around the two axes
  (models/mamba_block.py:496-507 of the reference).

The fields map one to one onto the ``reverse``, ``seq_group``, ``group_stride``,
``seq_stride`` and ``step_stride`` fields of the C argument structs; zeros select the
defaults (G = 1, A = L, C = 1).
"""
from __future__ import annotations

from dataclasses import dataclass, replace


@dataclass(frozen=True)
class TokenLayout:
    S: int
    L: int
    reverse: bool = False
    seq_group: int = 0
    group_stride: int = 0
    seq_stride: int = 0
    step_stride: int = 0

    @staticmethod
    def contiguous(S: int, L: int, reverse: bool = False) -> "TokenLayout":
        """row = s * L + t (a contiguous (S, L, width) tensor), optionally reversed."""
        return TokenLayout(int(S), int(L), bool(reverse))

    @staticmethod
    def time_axis(batch: int, frames: int, bins: int, reverse: bool = False) -> "TokenLayout":
        """Sequences (b, f) over the frames t of a (batch, frames, bins, width) tensor:
        sequence s = b * bins + f, row = b * frames * bins + t * bins + f."""
        return TokenLayout(int(batch) * int(bins), int(frames), bool(reverse),
                           seq_group=int(bins), group_stride=int(frames) * int(bins),
                           seq_stride=1, step_stride=int(bins))

    @staticmethod
    def freq_axis(batch: int, frames: int, bins: int, reverse: bool = False) -> "TokenLayout":
        """Sequences (b, t) over the bins f of a (batch, frames, bins, width) tensor: the
        contiguous layout with S = batch * frames, L = bins."""
        return TokenLayout.contiguous(int(batch) * int(frames), int(bins), reverse)

    @property
    def rows(self) -> int:
        return self.S * self.L

    @property
    def is_contiguous(self) -> bool:
        """True when the rows are sequence-major (row = s * L + t'), reversed or not."""
        G = self.seq_group or 1
        A = self.group_stride or self.L
        B = self.seq_stride
        C = self.step_stride or 1
        if C != 1:
            return False
        if G == 1:
            return A == self.L or self.S <= 1
        return B == self.L and A == G * self.L

    @property
    def is_default(self) -> bool:
        return self.is_contiguous and not self.reverse

    def flipped(self) -> "TokenLayout":
        """The same rows visited in the opposite step order."""
        return replace(self, reverse=not self.reverse)

    def row(self, s: int, t: int) -> int:
        """Row of step t (logical, before reversal) of sequence s."""
        G = self.seq_group or 1
        A = self.group_stride or self.L
        C = self.step_stride or 1
        tt = self.L - 1 - t if self.reverse else t
        return (s // G) * A + (s % G) * self.seq_stride + tt * C


def check_rows(name: str, t, layout: TokenLayout, width: int | None = None) -> None:
    """Raises ValueError unless ``t`` holds exactly layout.rows rows of ``width`` values."""
    w = t.shape[-1] if width is None else width
    if t.shape[-1] != w or t.numel() != layout.rows * w:
        raise ValueError(
            f"{name}: expected {layout.rows} rows of {w} values for a layout of "
            f"{layout.S} sequences x {layout.L} steps, got shape {tuple(t.shape)}")
