"""CPU model of the warp reduction network used by the selective-LRU backward
(`lane_reduce` in semambaxlinoss_b200/csrc/selective_lru_scan.cu): emulates the
__shfl_xor_sync rounds lane by lane and checks which value index each lane ends with,
for every (values per lane, channel lanes, lanes per channel) the kernels instantiate."""
from __future__ import annotations

import itertools

import pytest


def emulate(V, CW, NG, values):
    """values[lane][i]; lane = cl * NG + g. Returns the per-lane registers after the network."""
    v = [list(x) for x in values]
    kT = V if V < CW else CW
    r = 0
    while (1 << r) < kT:
        m = CW >> (r + 1)
        n = V >> (r + 1)
        new = [list(x) for x in v]
        for lane in range(32):
            cl = lane // NG
            up = (cl & m) != 0
            partner = lane ^ (m * NG)
            pcl = partner // NG
            pup = (pcl & m) != 0
            for i in range(n):
                keep = v[lane][i + n] if up else v[lane][i]
                send_from_partner = v[partner][i] if pup else v[partner][i + n]
                new[lane][i] = keep + send_from_partner
        v = new
        r += 1
    m = (CW // kT) // 2
    while m >= 1:
        new = [list(x) for x in v]
        for lane in range(32):
            new[lane][0] = v[lane][0] + v[lane ^ (m * NG)][0]
        v = new
        m //= 2
    return v


@pytest.mark.parametrize("NG,real", list(itertools.product([1, 2, 4, 8], [True, False])))
def test_lane_reduce_mapping(NG, real):
    GM = 4
    V = (2 if real else 4) * GM
    CW = 32 // NG
    # value i of lane (cl, g) = distinct prime-ish weights so sums identify their terms
    values = [[(lane // NG) * 1000 + (lane % NG) * 100 + i for i in range(V)] for lane in range(32)]
    out = emulate(V, CW, NG, values)
    for lane in range(32):
        cl, g = lane // NG, lane % NG

        def total(idx):
            return sum(values[c * NG + g][idx] for c in range(CW))

        if V >= CW:
            per = V // CW
            for i in range(per):
                assert out[lane][i] == total(cl * per + i)
        else:
            assert out[lane][0] == total(cl // (CW // V))
