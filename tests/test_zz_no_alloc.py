"""GPU: w4a8_lmhead_argmax_noalloc, the lm_head argmax for callers that cannot
allocate device memory (its scratch is a fixed array inside the library), called
through the C ABI and compared with w4a8_lmhead_argmax on two calls in a row.

This file is collected last on purpose, so a run that stops at the first failure
has already run every other test; it passes alone in a fresh process too."""

import ctypes

import numpy as np
import pytest
import torch

from oracle import c as orc
from webyiq_b200 import _lib

from helpers import make_weight, make_x

pytestmark = pytest.mark.gpu


def _dev(a, device):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


@pytest.mark.parametrize("group,has_min,act,m", [(128, False, 1, 1), (128, True, 1, 3), (32, True, 0, 2),
                                                 (128, False, 1, 16)])
def test_noalloc_matches_workspace_entry_point(cuda, group, has_min, act, m):
    L = _lib.load()
    n, k = 5003, 1024
    q, s, _ = make_weight(n, k, group, has_min, seed=m + group)
    xq, xs = orc.quant(make_x(m, k, seed=m), act=act)
    qd = _dev(q.view(np.int32), cuda)
    sd = _dev(s.view(np.int32) if has_min else s.view(np.int16), cuda)
    w = _lib.Weight()
    _lib.check(L.w4a8_weight_view(ctypes.c_void_p(qd.data_ptr()), ctypes.c_void_p(sd.data_ptr()), n, k, group,
                                  int(has_min), ctypes.byref(w)))
    dxq, dxs = _dev(xq, cuda), _dev(xs, cuda)
    ids = _dev(np.arange(n, dtype=np.uint32) * 3 + 7, cuda)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731

    # the existing entry point, with a caller-provided workspace
    ws = torch.zeros(L.w4a8_lmhead_workspace_bytes(n, m), dtype=torch.uint8, device=cuda)
    ref_key = torch.empty(m, dtype=torch.int64, device=cuda)
    ref_tok = torch.empty(m, dtype=torch.int32, device=cuda)
    ref_lg = torch.empty((m, n), dtype=torch.float32, device=cuda)
    _lib.check(L.w4a8_lmhead_argmax(ctypes.byref(w), 11, P(dxq), P(dxs), act, m, P(ref_lg), P(ref_key), P(ref_tok),
                                    P(ids), P(ws), ws.numel(), stream))
    torch.cuda.synchronize()

    for _ in range(2):  # two calls in a row share the library's scratch
        key = torch.full((m,), -1, dtype=torch.int64, device=cuda)
        tok = torch.full((m,), -1, dtype=torch.int32, device=cuda)
        lg = torch.zeros((m, n), dtype=torch.float32, device=cuda)
        _lib.check(L.w4a8_lmhead_argmax_noalloc(ctypes.byref(w), 11, P(dxq), P(dxs), act, m, P(lg), P(key), P(tok),
                                                P(ids), stream))
        torch.cuda.synchronize()
        # exact: same kernel, same sums (tolerance 0)
        np.testing.assert_array_equal(key.cpu().numpy(), ref_key.cpu().numpy())
        np.testing.assert_array_equal(tok.cpu().numpy(), ref_tok.cpu().numpy())
        np.testing.assert_array_equal(lg.cpu().numpy().view(np.uint32), ref_lg.cpu().numpy().view(np.uint32))

    # beyond the scratch's 16 tokens: rejected before any launch
    st = L.w4a8_lmhead_argmax_noalloc(ctypes.byref(w), 0, P(dxq), P(dxs), act, 17, None, P(key), None, None, stream)
    assert st == _lib.EINVAL
    assert b"16 tokens" in L.w4a8_last_error()
