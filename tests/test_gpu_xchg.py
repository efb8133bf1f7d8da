"""The peer-memory key exchange of the column-split lm_head (w4a8_lmhead_argmax_xchg)
on one GPU, world 1 (the rank's own buffer only, opened without torch.distributed).

Where the streaming lm_head covers the call (one or two tokens, whole 8-row blocks)
its last CTA runs the merge, so the call is one kernel; other calls (three tokens,
or rows not in whole 8-row blocks) leave the shard's key to the separate merge
kernel.  Either way the key and token must equal w4a8_lmhead_argmax's and the
oracle's bit for bit, over consecutive calls (both halves of the double-buffered
key slots), with a row offset, and over CUDA graph replays.  The multi-rank
exchange and its timeout run in test_gpu_multi.py."""

import ctypes

import numpy as np
import pytest
import torch

from oracle import c as orc
from webyiq_b200 import _lib, ops

from helpers import make_weight, make_x, shard_key, to_i64

pytestmark = pytest.mark.gpu


class _OneRankExchange:
    """A world-1 exchange: the C-ABI create/open with this rank's own handle."""

    def __init__(self):
        self.ptr = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(ops.XCHG_HANDLE_BYTES)
        _lib.check(_lib.load().w4a8_xchg_create(1, 0, handle, ctypes.byref(self.ptr)))
        _lib.check(_lib.load().w4a8_xchg_open(self.ptr, handle))

    def close(self):
        _lib.check(_lib.load().w4a8_xchg_destroy(self.ptr))


def _dev_weight(q, s, n, k, cuda):
    return ops.QWeight(torch.from_numpy(np.ascontiguousarray(q).view(np.int32)).to(cuda),
                       torch.from_numpy(np.ascontiguousarray(s).view(np.int16)).to(cuda), n, k, 128, False)


@pytest.mark.parametrize("n,m", [(8 * 1037, 1), (8 * 1037, 2), (8 * 1037, 3), (8 * 1037 + 5, 1)])
def test_exchange_one_rank(cuda, n, m):
    k, off = 2048, 1000
    q, s, _ = make_weight(n, k, 128, False, seed=n + m)
    xq, xs = orc.quant(make_x(m, k, seed=m + 5), act=1)
    logits = orc.gemv(q, s, k, 128, False, xq, xs, act=1)
    ref_tok = (orc.argmax(logits).astype(np.int64) + off).tolist()
    ref_key = [to_i64(shard_key(row, off)) for row in logits]
    w = _dev_weight(q, s, n, k, cuda)
    xq_d, xs_d = torch.from_numpy(xq).to(cuda), torch.from_numpy(xs).to(cuda)
    ws = ops.lmhead_workspace(w, m, cuda)
    key0, tok0 = ops.lmhead_argmax(w, xq_d, xs_d, act=1, row_offset=off, workspace=ws)
    torch.cuda.synchronize()
    assert key0.tolist() == ref_key and tok0.tolist() == ref_tok
    x = _OneRankExchange()
    try:
        key = torch.empty(m, dtype=torch.int64, device=cuda)
        tok = torch.empty(m, dtype=torch.int32, device=cuda)
        for _ in range(3):
            key.zero_()
            tok.zero_()
            ops.lmhead_argmax_xchg(w, xq_d, xs_d, x, act=1, row_offset=off, workspace=ws, best_key=key, tok=tok,
                                   check=True)
            assert key.tolist() == ref_key and tok.tolist() == ref_tok
        g = torch.cuda.CUDAGraph()
        st = torch.cuda.Stream()
        st.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(st):
            with torch.cuda.graph(g, stream=st):
                ops.lmhead_argmax_xchg(w, xq_d, xs_d, x, act=1, row_offset=off, workspace=ws, best_key=key, tok=tok)
        for _ in range(2):
            key.zero_()
            tok.zero_()
            g.replay()
            torch.cuda.synchronize()
            assert key.tolist() == ref_key and tok.tolist() == ref_tok
        del g
        assert ops.device_error() == 0
    finally:
        torch.cuda.synchronize()
        x.close()


def test_exchange_rejects_ids_past_2_24(cuda):
    """The exchanged keys carry the call's tag in the top 8 bits of their id half, so
    a shard whose vocabulary ids reach 2^24 is refused before anything runs."""
    from webyiq_b200._lib import EINVAL, W4A8Error

    n, k = 64, 256
    q, s, _ = make_weight(n, k, 128, False, seed=3)
    xq, xs = orc.quant(make_x(1, k, seed=4), act=1)
    w = _dev_weight(q, s, n, k, cuda)
    x = _OneRankExchange()
    try:
        with pytest.raises(W4A8Error) as exc:
            ops.lmhead_argmax_xchg(w, torch.from_numpy(xq).to(cuda), torch.from_numpy(xs).to(cuda), x, act=1,
                                   row_offset=(1 << 24) - n + 1)
        assert exc.value.status == EINVAL
    finally:
        x.close()
