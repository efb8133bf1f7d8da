"""Failure detection on the GPU without a fault: every device-side wait of the
library is bounded, records a code in the device error word when it gives up and
returns, so the context stays usable.  The self-test kernel waits on a barrier that
nothing arrives on; the host then reads ETIMEOUT with that code, the word is
cleared, and ordinary kernels keep working on the same context."""

import numpy as np
import pytest
import torch

from oracle import c as orc
from webyiq_b200 import ops
from webyiq_b200._lib import W4A8Error

from helpers import make_weight, make_x
from test_gpu_parity import dev_weight, to_dev

pytestmark = pytest.mark.gpu

ETIMEOUT = 4  # W4A8_ETIMEOUT


def test_bounded_wait_reports_timeout_and_context_survives(cuda):
    assert ops.device_error() == 0
    ops.selftest_wait_timeout()
    with pytest.raises(W4A8Error) as e:
        ops.device_error()
    assert e.value.status == ETIMEOUT
    assert "0x4" in str(e.value)
    assert ops.device_error() == 0  # read and cleared
    # the same context still runs the tensor-core GEMV and GEMM correctly
    q, s, _ = make_weight(256, 2048, 128, False, seed=3)
    xq, xs = orc.quant(make_x(130, 2048, seed=4), act=1)
    ref = orc.gemv(q, s, 2048, 128, False, xq, xs, act=1)
    w = dev_weight(q, s, 256, 2048, 128, False, cuda)
    y1 = ops.gemv(w, to_dev(xq[:1], cuda), to_dev(xs[:1], cuda), act=1)
    y2 = ops.gemm(w, to_dev(xq, cuda), to_dev(xs, cuda), act=1)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(y1.cpu().numpy().view(np.uint32), ref[:1].view(np.uint32))
    err = np.abs(y2.cpu().numpy() - ref).max() / np.abs(ref).max()
    assert err < 1e-5
    assert ops.device_error() == 0
