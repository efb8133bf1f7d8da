"""The CPU restatements of the MTP step kernels (oracle/spec.py) on the cases the
reference's shader comment spells out (spec_accept.wgsl:1-8): an accepted draft
emits two tokens and advances two positions, a rejected one emits one."""

import numpy as np

from oracle import spec


def test_spec_accept_accepted():
    tok, ctl, out = spec.spec_accept([5, 9], [9, 11], [21, 22], (100, 102, 2, 1))
    assert tok.tolist() == [11, 22]
    assert ctl.tolist() == [102, 104, 2, 0]
    assert out.tolist() == [2, 9, 11, 102, 0]


def test_spec_accept_rejected():
    tok, ctl, out = spec.spec_accept([5, 8], [9, 11], [21, 22], (100, 102, 2, 2))
    assert tok.tolist() == [9, 21]
    assert ctl.tolist() == [101, 103, 2, 0]
    assert out.tolist() == [1, 9, 11, 101, 0]


def test_gather_rows_picks_rows():
    q = np.arange(40, dtype=np.uint32).reshape(10, 4)
    s = np.arange(20, dtype=np.uint16).reshape(10, 2)
    gq, gs = spec.gather_rows(q, s, [7, 0, 7])
    assert gq.tolist() == [q[7].tolist(), q[0].tolist(), q[7].tolist()]
    assert gs.tolist() == [s[7].tolist(), s[0].tolist(), s[7].tolist()]
