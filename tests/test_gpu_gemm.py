"""GPU parity of the tcgen05 prefill GEMM (w4a8_gemm for group-128 symmetric
weights with per-token activations), through the C ABI, against the CPU oracle.

Bars: the int32 group dots read back from tensor memory are bit-exact; y, whose
scale step is f32 (sum_g f32(s) * f32(I), then * dx), is within 1e-5 relative of
the oracle's exact per-token output (1e-3 for SWIGLU, which goes through expf)."""

import numpy as np
import pytest
import torch

from oracle import c as orc
from webyiq_b200 import ops

from helpers import assert_rel_close, make_weight, make_x
from test_gpu_parity import dev_weight, to_dev

pytestmark = pytest.mark.gpu


def case(n, k, m, seed):
    q, s, _ = make_weight(n, k, 128, False, seed=seed)
    xq, xs = orc.quant(make_x(m, k, seed=seed + 1), act=1)
    return q, s, xq, xs


# (n, k, m): one tile, row and token tails, several groups, tiles > SMs, k = 6144.
DOT_SHAPES = [(128, 128, 1), (128, 256, 128), (200, 384, 130), (96, 2048, 17), (256, 1024, 257),
              (384, 6144, 40), (6144, 256, 129)]


@pytest.mark.parametrize("n,k,m", DOT_SHAPES)
def test_gemm_tc_group_dots_exact(cuda, n, k, m):
    q, s, xq, _ = case(n, k, m, seed=n + k + m)
    ref = orc.group_dots(q, k, 128, False, xq)
    w = dev_weight(q, s, n, k, 128, False, cuda)
    out = ops.gemm_group_dots(w, to_dev(xq, cuda))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), ref)


Y_SHAPES = [(128, 128, 1), (256, 2048, 130), (96, 512, 300), (200, 1024, 64), (640, 4096, 129), (128, 6144, 256)]


@pytest.mark.parametrize("n,k,m", Y_SHAPES)
@pytest.mark.parametrize("mode", [0, 1, 2])
def test_gemm_tc_outputs(cuda, n, k, m, mode):
    q, s, xq, xs = case(n, k, m, seed=3 * n + k + m + mode)
    n_out = n // 2 if mode == 2 else n
    y0 = make_x(m, n_out, seed=9) if mode == 1 else None
    ref = orc.gemv(q, s, k, 128, False, xq, xs, act=1, mode=mode, y=None if y0 is None else y0.copy())
    w = dev_weight(q, s, n, k, 128, False, cuda)
    y = None if y0 is None else to_dev(y0, cuda)
    out = ops.gemm(w, to_dev(xq, cuda), to_dev(xs, cuda), act=1, mode=mode, y=y)
    torch.cuda.synchronize()
    assert_rel_close(out.cpu().numpy(), ref, 1e-3 if mode == 2 else 1e-5)


def test_gemm_tc_matches_token_block_path(cuda):
    """The tcgen05 kernel and the GEMV-over-token-blocks path agree to f32 rounding."""
    n, k, m = 512, 2048, 200
    q, s, xq, xs = case(n, k, m, seed=77)
    w = dev_weight(q, s, n, k, 128, False, cuda)
    xq_d, xs_d = to_dev(xq, cuda), to_dev(xs, cuda)
    y_tc = ops.gemm(w, xq_d, xs_d, act=1)
    ops.set_gemm_kernel(False)
    try:
        y_blk = ops.gemm(w, xq_d, xs_d, act=1)
    finally:
        ops.set_gemm_kernel(True)
    torch.cuda.synchronize()
    assert_rel_close(y_tc.cpu().numpy(), y_blk.cpu().numpy(), 1e-5)
    code = ops.device_error()
    assert code == 0


@pytest.mark.parametrize("k,n", [(2048, 6144), (6144, 2048)])
def test_gemm_tc_c4_full_size(cuda, k, n):
    """BASELINE C4 (M=1024 prefill): every one of the 1024 x N outputs against the
    oracle's exact per-token output, within the 1e-5 bar."""
    m = 1024
    q, s, xq, xs = case(n, k, m, seed=k + n)
    w = dev_weight(q, s, n, k, 128, False, cuda)
    out = ops.gemm(w, to_dev(xq, cuda), to_dev(xs, cuda), act=1)
    torch.cuda.synchronize()
    ref = orc.gemv(q, s, k, 128, False, xq, xs, act=1)
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    assert_rel_close(got, ref, 1e-5)
    assert ops.device_error() == 0


@pytest.mark.parametrize("k,n", [(6144, 2048), (2048, 6144)])
def test_gemm_tc_c4_group_dots_exact(cuda, k, n):
    """BASELINE C4 shapes: every int32 group dot of the tcgen05 GEMM (read back from
    tensor memory), all 1024 tokens x N rows x K/128 groups, bit-exact."""
    m = 1024
    q, s, xq, _ = case(n, k, m, seed=2 * k + n)
    w = dev_weight(q, s, n, k, 128, False, cuda)
    out = ops.gemm_group_dots(w, to_dev(xq, cuda))
    torch.cuda.synchronize()
    ref = orc.group_dots(q, k, 128, False, xq)
    np.testing.assert_array_equal(out.cpu().numpy(), ref)
    assert ops.device_error() == 0
