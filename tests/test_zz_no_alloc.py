"""GPU: w4a8_lmhead_argmax_noalloc, the lm_head argmax for callers that cannot
allocate device memory (its scratch is a fixed array inside the library), called
through the C ABI and compared with w4a8_lmhead_argmax on two calls in a row, and
with the CPU oracle directly (GEMV then argmax), up to config 3's full 248,320-row
vocabulary.

Cases cover both kernels the entry point reaches: the streaming lm_head kernel
(group 128, per-token activations, one or two tokens, rows a multiple of 8) and the
GEMV kernels with the fused argmax (everything else).

This file is collected last on purpose, so a run that stops at the first failure
has already run every other test; it passes alone in a fresh process too."""

import ctypes

import numpy as np
import pytest
import torch

from oracle import c as orc
from webyiq_b200 import _lib

from helpers import make_weight, make_x, shard_key, to_i64

pytestmark = pytest.mark.gpu


def _dev(a, device):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def _view(L, qd, sd, n, k, group, has_min):
    w = _lib.Weight()
    _lib.check(L.w4a8_weight_view(ctypes.c_void_p(qd.data_ptr()), ctypes.c_void_p(sd.data_ptr()), n, k, group,
                                  int(has_min), ctypes.byref(w)))
    return w


def _P(t):
    return ctypes.c_void_p(t.data_ptr())


# (n, group, has_min, act, m): n = 5003 takes the GEMV kernels; n = 5008 (a multiple
# of 8) with group 128 and per-token activations for one or two tokens takes the
# streaming kernel.
CASES = [(5003, 128, False, 1, 1), (5003, 128, True, 1, 3), (5003, 32, True, 0, 2), (5003, 128, False, 1, 16),
         (5008, 128, False, 1, 1), (5008, 128, False, 1, 2), (5008, 128, True, 1, 1)]


@pytest.mark.parametrize("n,group,has_min,act,m", CASES)
def test_noalloc_matches_workspace_entry_point(cuda, n, group, has_min, act, m):
    L = _lib.load()
    k = 1024
    q, s, _ = make_weight(n, k, group, has_min, seed=m + group + n)
    xq, xs = orc.quant(make_x(m, k, seed=m), act=act)
    qd = _dev(q.view(np.int32), cuda)
    sd = _dev(s.view(np.int32) if has_min else s.view(np.int16), cuda)
    w = _view(L, qd, sd, n, k, group, has_min)
    dxq, dxs = _dev(xq, cuda), _dev(xs, cuda)
    ids = _dev(np.arange(n + 11, dtype=np.uint32) * 3 + 7, cuda)  # indexed by the global row id (offset 11)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    # the existing entry point, with a caller-provided workspace
    ws = torch.zeros(L.w4a8_lmhead_workspace_bytes(n, m), dtype=torch.uint8, device=cuda)
    ref_key = torch.empty(m, dtype=torch.int64, device=cuda)
    ref_tok = torch.empty(m, dtype=torch.int32, device=cuda)
    ref_lg = torch.empty((m, n), dtype=torch.float32, device=cuda)
    _lib.check(L.w4a8_lmhead_argmax(ctypes.byref(w), 11, _P(dxq), _P(dxs), act, m, _P(ref_lg), _P(ref_key),
                                    _P(ref_tok), _P(ids), _P(ws), ws.numel(), stream))
    torch.cuda.synchronize()

    for _ in range(2):  # two calls in a row share the library's scratch
        key = torch.full((m,), -1, dtype=torch.int64, device=cuda)
        tok = torch.full((m,), -1, dtype=torch.int32, device=cuda)
        lg = torch.zeros((m, n), dtype=torch.float32, device=cuda)
        _lib.check(L.w4a8_lmhead_argmax_noalloc(ctypes.byref(w), 11, _P(dxq), _P(dxs), act, m, _P(lg), _P(key),
                                                _P(tok), _P(ids), stream))
        torch.cuda.synchronize()
        # exact: same kernel, same sums (tolerance 0)
        np.testing.assert_array_equal(key.cpu().numpy(), ref_key.cpu().numpy())
        np.testing.assert_array_equal(tok.cpu().numpy(), ref_tok.cpu().numpy())
        np.testing.assert_array_equal(lg.cpu().numpy().view(np.uint32), ref_lg.cpu().numpy().view(np.uint32))

    if act == 1:
        # and against the oracle directly: per-token logits are exact, so bit for bit
        ref = orc.gemv(q, s, k, group, has_min, xq, xs, act=1)
        np.testing.assert_array_equal(lg.cpu().numpy().view(np.uint32), ref.view(np.uint32))
        idx = orc.argmax(ref).astype(np.int64)
        np.testing.assert_array_equal(tok.cpu().numpy(), (idx + 11) * 3 + 7)
        assert key.cpu().tolist() == [to_i64(shard_key(r, 11)) for r in ref]

    # beyond the scratch's 16 tokens: rejected before any launch
    st = L.w4a8_lmhead_argmax_noalloc(ctypes.byref(w), 0, _P(dxq), _P(dxs), act, 17, None, _P(key), None, None,
                                      stream)
    assert st == _lib.EINVAL
    assert b"16 tokens" in L.w4a8_last_error()


@pytest.mark.parametrize("m", [1, 2])
def test_noalloc_full_vocabulary_against_oracle(cuda, m):
    """Config 3's lm_head (248,320 x 2048, group 128, symmetric, per-token int8) through
    the no-allocation entry point twice in a row: the token of every call is the
    oracle's argmax of the oracle's logits, and the logits are bit-identical."""
    L = _lib.load()
    n, k = 248320, 2048
    rng = np.random.default_rng(31 + m)
    q = rng.integers(0, 2 ** 32, size=(n, k // 8), dtype=np.uint32)  # uniform nibbles
    s = (np.abs(rng.standard_normal((n, k // 128))) * 0.01).astype(np.float16)
    xq, xs = orc.quant(make_x(m, k, seed=40 + m), act=1)
    ref = orc.gemv(q, s.view(np.uint16), k, 128, False, xq, xs, act=1)
    ref_tok = orc.argmax(ref).astype(np.int64)

    qd = _dev(q.view(np.int32), cuda)
    sd = _dev(s.view(np.int16), cuda)
    w = _view(L, qd, sd, n, k, 128, False)
    dxq, dxs = _dev(xq, cuda), _dev(xs, cuda)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for call in range(2):
        key = torch.full((m,), -1, dtype=torch.int64, device=cuda)
        tok = torch.full((m,), -1, dtype=torch.int32, device=cuda)
        lg = torch.zeros((m, n), dtype=torch.float32, device=cuda)
        _lib.check(L.w4a8_lmhead_argmax_noalloc(ctypes.byref(w), 0, _P(dxq), _P(dxs), 1, m, _P(lg), _P(key),
                                                _P(tok), None, stream))
        torch.cuda.synchronize()
        np.testing.assert_array_equal(tok.cpu().numpy().astype(np.int64), ref_tok, err_msg=f"call {call}")
        np.testing.assert_array_equal(lg.cpu().numpy().view(np.uint32), ref.view(np.uint32), err_msg=f"call {call}")
        keys = key.cpu().numpy().view(np.uint64)
        assert [int(~int(kk) & 0xFFFFFFFF) for kk in keys] == ref_tok.tolist()
