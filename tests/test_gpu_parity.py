"""GPU parity: every CUDA kernel, called through the C ABI, against the CPU oracle
(oracle/w4a8_oracle.c) on the same seeded inputs.

Bars: bit-exact for the quantizer, the int32 group dots, every per-token
(W4A8_ACT_TOKEN) STORE/ADD output and every argmax id; the per-group-32 f32 path
and SWIGLU (expf) within 1e-3 relative (helpers.assert_rel_close)."""

import numpy as np
import pytest
import torch

from oracle import c as orc
from webyiq_b200 import ops
from webyiq_b200._lib import W4A8Error

from helpers import assert_rel_close, make_weight, make_x

pytestmark = pytest.mark.gpu


def dev_weight(q, s, n, k, group, has_min, device):
    qt = torch.from_numpy(np.ascontiguousarray(q).view(np.int32)).to(device)
    st = torch.from_numpy(np.ascontiguousarray(s).view(np.int32 if has_min else np.int16)).to(device)
    return ops.QWeight(qt, st, n, k, group, has_min)


def to_dev(a, device):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def bits(a):
    a = np.ascontiguousarray(a)
    return a.view(np.uint32) if a.dtype == np.float32 else a


@pytest.mark.parametrize("act", [0, 1])
@pytest.mark.parametrize("norm", [False, True])
@pytest.mark.parametrize("m,k", [(1, 32), (3, 2048), (2, 6144), (5, 4096), (1, 96)])
def test_quant_bit_exact(cuda, act, norm, m, k):
    x = make_x(m, k, seed=k + m)
    x[0, :32] = 0.0  # a zero group
    nw = (1 + 0.2 * make_x(1, k, seed=5)[0]).astype(np.float32) if norm else None
    ref_q, ref_s = orc.quant(x, nw, 1e-6, act=act)
    xq, xs = ops.quant(to_dev(x, cuda), None if nw is None else to_dev(nw, cuda), 1e-6, act=act)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(xq.cpu().numpy(), ref_q)
    np.testing.assert_array_equal(bits(xs.cpu().numpy()), bits(ref_s))


SHAPES_128 = [(37, 256), (100, 2048), (64, 6144), (8, 4096), (3, 128)]
SHAPES_32 = [(37, 96), (100, 2048), (16, 32), (48, 6144)]


@pytest.mark.parametrize("has_min", [False, True])
@pytest.mark.parametrize("group,shape", [(128, s) for s in SHAPES_128] + [(32, s) for s in SHAPES_32])
@pytest.mark.parametrize("m", [1, 3, 16])
def test_group_dots_exact(cuda, group, shape, has_min, m):
    n, k = shape
    q, s, _ = make_weight(n, k, group, has_min, seed=n * 7 + k)
    xq, _ = orc.quant(make_x(m, k, seed=m), act=1)
    ref = orc.group_dots(q, k, group, has_min, xq)
    w = dev_weight(q, s, n, k, group, has_min, cuda)
    out = ops.group_dots(w, to_dev(xq, cuda))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), ref)


@pytest.mark.parametrize("group,has_min", [(128, False), (128, True), (32, True), (32, False)])
@pytest.mark.parametrize("m", [1, 2, 3, 4, 8, 16])
@pytest.mark.parametrize("mode", [0, 1, 2])
def test_gemv_token(cuda, group, has_min, m, mode):
    n, k = (96, 2048) if group == 128 else (64, 1024)
    q, s, _ = make_weight(n, k, group, has_min, seed=m + 10 * mode)
    xq, xs = orc.quant(make_x(m, k, seed=m), act=1)
    base = make_x(m, n // 2 if mode == 2 else n, seed=99) if mode == 1 else None
    ref = orc.gemv(q, s, k, group, has_min, xq, xs, act=1, mode=mode, y=base)
    w = dev_weight(q, s, n, k, group, has_min, cuda)
    y = None if base is None else to_dev(base, cuda)
    y = ops.gemv(w, to_dev(xq, cuda), to_dev(xs, cuda), act=1, mode=mode, y=y)
    torch.cuda.synchronize()
    if mode == 2:
        assert_rel_close(y.cpu().numpy(), ref, 1e-3)
    else:
        np.testing.assert_array_equal(bits(y.cpu().numpy()), bits(ref))


@pytest.mark.parametrize("group,has_min", [(32, True), (32, False), (128, True), (128, False)])
@pytest.mark.parametrize("m", [1, 2, 5, 16])
@pytest.mark.parametrize("mode", [0, 1, 2])
def test_gemv_group32(cuda, group, has_min, m, mode):
    n, k = 64, 2048
    q, s, _ = make_weight(n, k, group, has_min, seed=m + 3)
    xq, xs = orc.quant(make_x(m, k, seed=m + 1), act=0)
    base = make_x(m, n // 2 if mode == 2 else n, seed=98) if mode == 1 else None
    ref = orc.gemv(q, s, k, group, has_min, xq, xs, act=0, mode=mode, y=base)
    w = dev_weight(q, s, n, k, group, has_min, cuda)
    y = None if base is None else to_dev(base, cuda)
    y = ops.gemv(w, to_dev(xq, cuda), to_dev(xs, cuda), act=0, mode=mode, y=y)
    torch.cuda.synchronize()
    assert_rel_close(y.cpu().numpy(), ref, 1e-3)


def test_gemv_golden_reference_fakequant(cuda):
    """The engine's own format (convert.py group 32) through quant + GEMV on the GPU,
    against the reference's fake-quant linear (tests/golden/fakequant.npz)."""
    import os

    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "fakequant.npz"))
    x, k = g["x"], g["x"].shape[1]
    xq, xs = ops.quant(to_dev(x, cuda), act=0)
    w = dev_weight(g["packed"], g["scales"], g["packed"].shape[0], k, 32, True, cuda)
    y = ops.gemv(w, xq, xs, act=0)
    torch.cuda.synchronize()
    assert_rel_close(y.cpu().numpy(), g["y"], 1e-3)


def test_gemv_c1_full_size_bit_exact(cuda):
    """K=2048, N=6144, symmetric int4 group 128, per-token int8."""
    n, k = 6144, 2048
    q, s, _ = make_weight(n, k, 128, False, seed=0)
    xq, xs = orc.quant(make_x(1, k, seed=1), act=1)
    ref = orc.gemv(q, s, k, 128, False, xq, xs, act=1)
    w = dev_weight(q, s, n, k, 128, False, cuda)
    y = ops.gemv(w, to_dev(xq, cuda), to_dev(xs, cuda), act=1)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(bits(y.cpu().numpy()), bits(ref))
    # run-to-run and PDL on/off identical
    ops.set_pdl(False)
    y2 = ops.gemv(w, to_dev(xq, cuda), to_dev(xs, cuda), act=1)
    ops.set_pdl(True)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(bits(y2.cpu().numpy()), bits(ref))


@pytest.mark.parametrize("m", [1, 2, 17, 64, 130])
def test_gemm_and_matmul(cuda, m):
    n, k = 96, 2048
    q, s, _ = make_weight(n, k, 128, False, seed=m)
    xq, xs = orc.quant(make_x(m, k, seed=m), act=1)
    ref = orc.gemv(q, s, k, 128, False, xq, xs, act=1)
    w = dev_weight(q, s, n, k, 128, False, cuda)
    y1 = ops.gemm(w, to_dev(xq, cuda), to_dev(xs, cuda), act=1)
    y2 = ops.matmul(w, to_dev(xq, cuda), to_dev(xs, cuda), act=1)
    torch.cuda.synchronize()
    assert_rel_close(y1.cpu().numpy(), ref, 1e-5)
    assert_rel_close(y2.cpu().numpy(), ref, 1e-5)


# ---------------------------------------------------------------------------
# lm_head with fused argmax


def lmhead_case(n, k, m, seed, tie_rows=()):
    q, s, _ = make_weight(n, k, 128, False, seed=seed)
    for dst, src in tie_rows:  # identical rows give identical logits: a tie
        q[dst] = q[src]
        s[dst] = s[src]
    xq, xs = orc.quant(make_x(m, k, seed=seed + 1), act=1)
    return q, s, xq, xs


@pytest.mark.parametrize("m", [1, 2, 4])
def test_lmhead_argmax_exact(cuda, m):
    n, k = 4099, 1024
    q, s, xq, xs = lmhead_case(n, k, m, seed=4)
    logits = orc.gemv(q, s, k, 128, False, xq, xs, act=1)
    best = int(orc.argmax(logits)[0])
    # force a tie with the best row of token 0 at a higher and a lower index
    q, s, xq, xs = lmhead_case(n, k, m, seed=4, tie_rows=[(n - 1, best), (best // 2, best)])
    logits = orc.gemv(q, s, k, 128, False, xq, xs, act=1)
    ref_tok = orc.argmax(logits)
    assert ref_tok[0] == best // 2
    ids = (np.arange(n, dtype=np.uint32) * 3 + 1)
    w = dev_weight(q, s, n, k, 128, False, cuda)
    dxq, dxs = to_dev(xq, cuda), to_dev(xs, cuda)
    lg = torch.empty((m, n), dtype=torch.float32, device=cuda)
    ws = ops.lmhead_workspace(w, m, cuda)
    for rep in range(3):  # the workspace resets itself between calls
        key, tok = ops.lmhead_argmax(w, dxq, dxs, act=1, logits=lg, workspace=ws)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(bits(lg.cpu().numpy()), bits(logits))
        np.testing.assert_array_equal(tok.cpu().numpy().astype(np.uint32), ref_tok)
        assert [ops.key_index(int(v)) for v in key.cpu().numpy()] == list(ref_tok)
    _, tok = ops.lmhead_argmax(w, dxq, dxs, act=1, ids=to_dev(ids, cuda), workspace=ws)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(tok.cpu().numpy().astype(np.uint32), ids[ref_tok])


@pytest.mark.parametrize("has_min", [False, True])
@pytest.mark.parametrize("m", [1, 2])
@pytest.mark.parametrize("n,k", [(296, 1024), (9472, 384), (19000, 2048), (148 * 64 * 3 + 40, 2048),
                                 (12344, 2560), (10008, 4096), (4840, 8192)])
def test_lmhead_stream_shapes(cuda, n, k, m, has_min):
    """The streaming lm_head (group 128, per-token, one or two tokens, n a multiple
    of 8) over each split of a row between lanes (8, 16 or 32 lanes of one or two
    groups, idle lanes past the row's end), ragged last stages and CTAs of a single
    8-row block; k=8192 with two tokens is past its cover and takes the other
    kernel.  Logits bit-exact, the argmax with a planted tie."""
    q, s, _ = make_weight(n, k, 128, has_min, seed=k + n)
    xq, xs = orc.quant(make_x(m, k, seed=k), act=1)
    logits = orc.gemv(q, s, k, 128, has_min, xq, xs, act=1)
    best = int(orc.argmax(logits)[0])
    lo = best // 3  # a copy of the best row at a lower index wins the tie
    q[lo], s[lo] = q[best], s[best]
    logits = orc.gemv(q, s, k, 128, has_min, xq, xs, act=1)
    ref = orc.argmax(logits)
    assert ref[0] == min(lo, best)
    w = dev_weight(q, s, n, k, 128, has_min, cuda)
    lg = torch.empty((m, n), dtype=torch.float32, device=cuda)
    ws = ops.lmhead_workspace(w, m, cuda)
    for _ in range(2):
        key, tok = ops.lmhead_argmax(w, to_dev(xq, cuda), to_dev(xs, cuda), act=1, logits=lg, workspace=ws)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(bits(lg.cpu().numpy()), bits(logits))
        np.testing.assert_array_equal(tok.cpu().numpy().astype(np.uint32), ref)
    assert ops.device_error() == 0


@pytest.mark.parametrize("shards", [2, 4, 8])
def test_lmhead_sharded_merge(cuda, shards):
    """Column split with row_offset: the max of the shard keys is the full key."""
    n, k, m = 8 * 520, 512, 2
    q, s, xq, xs = lmhead_case(n, k, m, seed=shards)
    w = dev_weight(q, s, n, k, 128, False, cuda)
    dxq, dxs = to_dev(xq, cuda), to_dev(xs, cuda)
    full, tok = ops.lmhead_argmax(w, dxq, dxs, act=1)
    per = n // shards
    keys = []
    for r in range(shards):
        ws = dev_weight(q[r * per:(r + 1) * per], s[r * per:(r + 1) * per], per, k, 128, False, cuda)
        kk, _ = ops.lmhead_argmax(ws, dxq, dxs, act=1, row_offset=r * per)
        keys.append(kk.cpu().numpy().view(np.uint64))
    torch.cuda.synchronize()
    merged = np.max(np.stack(keys), axis=0)
    np.testing.assert_array_equal(merged, full.cpu().numpy().view(np.uint64))
    ref = orc.argmax(orc.gemv(q, s, k, 128, False, xq, xs, act=1))
    np.testing.assert_array_equal(tok.cpu().numpy().astype(np.uint32), ref)


def test_lmhead_c3_full_vocab(cuda):
    """K=2048, N=248320 vocab, group 128 symmetric, per-token."""
    n, k = 248320, 2048
    q, s, xq, xs = lmhead_case(n, k, 1, seed=3)
    logits = orc.gemv(q, s, k, 128, False, xq, xs, act=1)
    ref = orc.argmax(logits)
    w = dev_weight(q, s, n, k, 128, False, cuda)
    lg = torch.empty((1, n), dtype=torch.float32, device=cuda)
    key, tok = ops.lmhead_argmax(w, to_dev(xq, cuda), to_dev(xs, cuda), act=1, logits=lg)
    torch.cuda.synchronize()
    assert int(tok.cpu()[0]) == int(ref[0])
    np.testing.assert_array_equal(bits(lg.cpu().numpy()), bits(logits))


def test_lmhead_group32_matches_unfused(cuda):
    """f32 path: the fused argmax equals the standalone argmax of the logits it wrote."""
    n, k, m = 3000, 2048, 2
    q, s, _ = make_weight(n, k, 32, True, seed=8)
    xq, xs = orc.quant(make_x(m, k, seed=9), act=0)
    w = dev_weight(q, s, n, k, 32, True, cuda)
    lg = torch.empty((m, n), dtype=torch.float32, device=cuda)
    _, tok = ops.lmhead_argmax(w, to_dev(xq, cuda), to_dev(xs, cuda), act=0, logits=lg)
    tok2 = ops.argmax(lg)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(tok.cpu().numpy(), tok2.cpu().numpy())
    np.testing.assert_array_equal(tok.cpu().numpy().astype(np.uint32), orc.argmax(lg.cpu().numpy()))
    assert_rel_close(lg.cpu().numpy(), orc.gemv(q, s, k, 32, True, xq, xs, act=0), 1e-3)


def test_argmax_standalone(cuda):
    v = 1000
    lg = np.zeros((6, v), np.float32)
    lg[0, 17] = 5.0
    lg[0, 900] = 5.0
    lg[1, :] = -np.inf
    lg[2, :] = np.nan
    lg[2, 123] = 1.0
    lg[3, :] = -1.0
    lg[3, 10] = -0.0
    lg[3, 5] = 0.0
    lg[4, :] = -3.0e38
    lg[4, 999] = -2.9e38
    lg[5, :] = -5.0
    lg[5, 300] = -4.0
    big = make_x(3, 248320, seed=2)
    big[1, 1000] = big[1, 200000] = 50.0
    ids = (np.arange(248320, dtype=np.uint32) * 5 + 2)
    for a, i in ((lg, None), (big, None), (big, ids)):
        out = ops.argmax(to_dev(a, cuda), None if i is None else to_dev(i, cuda))
        torch.cuda.synchronize()
        np.testing.assert_array_equal(out.cpu().numpy().astype(np.uint32), orc.argmax(a, i))


def test_device_pointer_errors(cuda):
    q, s, _ = make_weight(16, 256, 128, False)
    w = dev_weight(q, s, 16, 256, 128, False, cuda)
    xq = torch.zeros(257, dtype=torch.int8, device=cuda)
    xs = torch.ones(1, dtype=torch.float32, device=cuda)
    with pytest.raises(W4A8Error, match="aligned"):
        ops.gemv(w, xq[1:].view(1, 256), xs, act=1)


@pytest.mark.parametrize("has_min", [False, True])
@pytest.mark.parametrize("m", [1, 2, 3, 5, 8, 13, 16])
@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("nk", [(200, 2048), (64, 6144), (48, 1024), (24, 256)])
def test_tensor_core_and_dp4a_kernels_agree(cuda, has_min, m, mode, nk):
    """Group-128 per-token GEMVs run on the tensor-core kernel by default; the dp4a
    kernel computes the same exact sums, so both must agree bit for bit."""
    n, k = nk
    q, s, _ = make_weight(n, k, 128, has_min, seed=n + m + mode)
    xq, xs = orc.quant(make_x(m, k, seed=m), act=1)
    w = dev_weight(q, s, n, k, 128, has_min, cuda)
    base = make_x(m, n // 2 if mode == 2 else n, seed=7)
    outs = []
    for tc in (True, False):
        ops.set_gemv_kernel(tc)
        y = to_dev(base, cuda) if mode == 1 else None
        outs.append(ops.gemv(w, to_dev(xq, cuda), to_dev(xs, cuda), act=1, mode=mode, y=y).cpu().numpy())
    ops.set_gemv_kernel(True)
    np.testing.assert_array_equal(bits(outs[0]), bits(outs[1]))
    assert ops.device_error() == 0


@pytest.mark.parametrize("has_min", [False, True])
@pytest.mark.parametrize("nk", [(96, 2048), (64, 6144), (40, 128)])
@pytest.mark.parametrize("m", [1, 2, 3, 8, 9, 16])
@pytest.mark.parametrize("mode", [0, 1, 2])
def test_gemv_fused_quant_bit_exact(cuda, has_min, nk, m, mode):
    """w4a8_gemv_x (per-token quant inside the GEMV) equals w4a8_quant + w4a8_gemv and
    the oracle bit for bit, zero rows included."""
    n, k = nk
    q, s, _ = make_weight(n, k, 128, has_min, seed=n + k + m)
    x = make_x(m, k, seed=m + 17)
    if m > 2:
        x[1] = 0.0  # a zero row: dx = 0, all codes 0
    xq, xs = orc.quant(x, act=1)
    n_out = n // 2 if mode == 2 else n
    y0 = make_x(m, n_out, seed=5) if mode == 1 else None
    ref = orc.gemv(q, s, k, 128, has_min, xq, xs, act=1, mode=mode, y=None if y0 is None else y0.copy())
    w = dev_weight(q, s, n, k, 128, has_min, cuda)
    y = ops.gemv_x(w, to_dev(x, cuda), mode=mode, y=None if y0 is None else to_dev(y0, cuda))
    xq_d, xs_d = ops.quant(to_dev(x, cuda), act=1)
    y2 = ops.gemv(w, xq_d, xs_d, act=1, mode=mode, y=None if y0 is None else to_dev(y0, cuda))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(bits(y.cpu().numpy()), bits(y2.cpu().numpy()))
    if mode == 2:
        assert_rel_close(y.cpu().numpy(), ref, 1e-3)
    else:
        np.testing.assert_array_equal(bits(y.cpu().numpy()), bits(ref))


@pytest.mark.parametrize("fq", [False, True])
@pytest.mark.parametrize("has_min", [False, True])
@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("m", [1, 2])
@pytest.mark.parametrize("n,k", [(6144, 2048), (2048, 6144), (2048, 4096), (512, 2048), (14000, 2048),
                                 (3000, 1024), (600, 384), (1500, 2560), (4096, 6144), (20000, 2048)])
def test_gemv_decode_shapes(cuda, n, k, m, mode, has_min, fq):
    """The decode GEMV (one or two tokens into y) over each split of a row between
    lanes (8, 16 or 32 lanes of one or two groups, idle lanes past the row's end),
    one to four row passes per CTA, a zero activation row, both CTA configurations
    (three per SM where the rows fit, else two: (14000, 2048) and (4096, 6144) at one
    token), and (20000, 2048), which exceeds its shared-memory plan and takes the
    tensor-core GEMV.  Bit-exact with
    the oracle (SWIGLU within 1e-3: expf) and with the dp4a GEMV, fused quant or not."""
    q, s, _ = make_weight(n, k, 128, has_min, seed=n + k + m + mode)
    x = make_x(m, k, seed=k + m)
    if m == 2 and has_min:
        x[1] = 0.0  # dx = 0, all codes 0
    xq, xs = orc.quant(x, act=1)
    n_out = n // 2 if mode == 2 else n
    y0 = make_x(m, n_out, seed=6) if mode == 1 else None
    ref = orc.gemv(q, s, k, 128, has_min, xq, xs, act=1, mode=mode, y=None if y0 is None else y0.copy())
    w = dev_weight(q, s, n, k, 128, has_min, cuda)
    base = lambda: None if y0 is None else to_dev(y0, cuda)  # noqa: E731
    if fq:
        y = ops.gemv_x(w, to_dev(x, cuda), mode=mode, y=base())
    else:
        y = ops.gemv(w, to_dev(xq, cuda), to_dev(xs, cuda), act=1, mode=mode, y=base())
    ops.set_gemv_kernel(False)
    try:
        y_dp4a = ops.gemv(w, to_dev(xq, cuda), to_dev(xs, cuda), act=1, mode=mode, y=base())
    finally:
        ops.set_gemv_kernel(True)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(bits(y.cpu().numpy()), bits(y_dp4a.cpu().numpy()))
    if mode == 2:
        assert_rel_close(y.cpu().numpy(), ref, 1e-3)
    else:
        np.testing.assert_array_equal(bits(y.cpu().numpy()), bits(ref))
    assert ops.device_error() == 0


@pytest.mark.parametrize("has_min", [False, True])
@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("m", [1, 2])
@pytest.mark.parametrize("n,k", [(6144, 2048), (2048, 6144), (2048, 4096), (600, 384), (1500, 2560), (2960, 8192)])
def test_gemv_norm_quant_fused(cuda, n, k, m, mode, has_min):
    """w4a8_gemv_xn (RMSNorm + per-token quant + GEMV in one launch) equals
    w4a8_quant(norm) followed by w4a8_gemv bit for bit, and the oracle (bit-exact;
    SWIGLU within 1e-3), a zero row included; more than two tokens, and two tokens
    with more than 32 groups a row, are refused."""
    q, s, _ = make_weight(n, k, 128, has_min, seed=n + k + 3 * m + mode)
    x = make_x(m, k, seed=k + m + 7)
    if m == 2 and has_min:
        x[1] = 0.0
    nw = (1 + 0.3 * make_x(1, k, seed=9)[0]).astype(np.float32)
    eps = 1e-6
    xq, xs = orc.quant(x, nw, eps, act=1)
    n_out = n // 2 if mode == 2 else n
    y0 = make_x(m, n_out, seed=8) if mode == 1 else None
    ref = orc.gemv(q, s, k, 128, has_min, xq, xs, act=1, mode=mode, y=None if y0 is None else y0.copy())
    w = dev_weight(q, s, n, k, 128, has_min, cuda)
    base = lambda: None if y0 is None else to_dev(y0, cuda)  # noqa: E731
    if m == 2 and k > 4096:  # two tokens: at most 32 groups a row (the decode kernel's cover)
        with pytest.raises(W4A8Error):
            ops.gemv_xn(w, to_dev(x, cuda), to_dev(nw, cuda), eps, mode=mode, y=base())
        return
    y = ops.gemv_xn(w, to_dev(x, cuda), to_dev(nw, cuda), eps, mode=mode, y=base())
    xq_d, xs_d = ops.quant(to_dev(x, cuda), to_dev(nw, cuda), eps, act=1)
    y2 = ops.gemv(w, xq_d, xs_d, act=1, mode=mode, y=base())
    torch.cuda.synchronize()
    np.testing.assert_array_equal(bits(y.cpu().numpy()), bits(y2.cpu().numpy()))
    if mode == 2:
        assert_rel_close(y.cpu().numpy(), ref, 1e-3)
    else:
        np.testing.assert_array_equal(bits(y.cpu().numpy()), bits(ref))
    if m == 1 and mode == 0:
        with pytest.raises(W4A8Error):
            ops.gemv_xn(w, to_dev(make_x(4, k), cuda), to_dev(nw, cuda), eps)


@pytest.mark.parametrize("group,has_min", [(32, True), (128, False)])
def test_gather_rows_and_draft_argmax(cuda, group, has_min):
    """MTP draft head: rows mtp.head_ids of the (tied) embedding gathered on the GPU
    equal the oracle's, and the lm_head argmax over them with the ids mapping gives
    the vocabulary token of the oracle's argmax over those rows."""
    from oracle import spec

    v, k, rows = 3000, 1024, 517
    q, s, _ = make_weight(v, k, group, has_min, seed=31)
    ids = np.random.default_rng(3).choice(v, size=rows, replace=False).astype(np.uint32)
    w = dev_weight(q, s, v, k, group, has_min, cuda)
    dids = torch.from_numpy(ids.view(np.int32)).to(cuda)
    dw = ops.gather_rows(w, dids)
    gq, gs = spec.gather_rows(q, s, ids)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(dw.q.cpu().numpy().view(np.uint32), gq.view(np.uint32))
    np.testing.assert_array_equal(dw.s.cpu().numpy().view(gs.dtype), gs)
    if group == 128:
        m = 2
        xq, xs = orc.quant(make_x(m, k, seed=32), act=1)
        logits = orc.gemv(gq, gs, k, 128, has_min, xq, xs, act=1)
        want = ids[orc.argmax(logits)]
        _, tok = ops.lmhead_argmax(dw, to_dev(xq, cuda), to_dev(xs, cuda), act=1, ids=dids)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(tok.cpu().numpy().astype(np.uint32), want)


def test_spec_accept_chain(cuda):
    """Two speculative steps on the GPU (accepted, then rejected), the second reading
    the first's ctl as its params, against the oracle."""
    from oracle import spec

    def i32(a):
        return torch.tensor(np.asarray(a, dtype=np.uint32).view(np.int32), device=cuda)

    tok, params = [5, 9], (100, 102, 2, 1)
    steps = [([9, 11], [21, 22]), ([3, 4], [7, 8])]  # y[0] == d accepts; then tok[1] = 22 != 3 rejects
    dtok, dctl, dout = i32(tok), i32(params), i32([0] * 5)
    for y, e in steps:
        want_tok, want_ctl, want_out = spec.spec_accept(tok, y, e, params)
        ops.spec_accept(dtok, i32(y), i32(e), dctl, dctl, dout)  # params alias ctl
        torch.cuda.synchronize()
        assert dtok.cpu().numpy().view(np.uint32).tolist() == want_tok.tolist()
        assert dctl.cpu().numpy().view(np.uint32).tolist() == want_ctl.tolist()
        assert dout.cpu().numpy().view(np.uint32).tolist() == want_out.tolist()
        tok, params = want_tok.tolist(), tuple(want_ctl.tolist())


def test_gemv_fused_quant_rejects_group32(cuda):
    q, s, _ = make_weight(32, 256, 32, True, seed=1)
    w = dev_weight(q, s, 32, 256, 32, True, cuda)
    with pytest.raises(W4A8Error):
        ops.gemv_x(w, to_dev(make_x(1, 256), cuda))
