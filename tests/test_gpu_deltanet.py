"""The Gated DeltaNet token mixer (deltanet.wgsl) on the GPU against
oracle/deltanet.py (float64 restatement; parity unpinned: the reference holds no
golden vectors for this op): the outputs and the updated state and conv windows
within 1e-4 of their scale, over decode (one token, in place) and draft verification
(two and three tokens, the per-token state slots), and several steps in a row
carrying the state."""

import numpy as np
import pytest
import torch

from oracle import deltanet as odn
from webyiq_b200 import ops

pytestmark = pytest.mark.gpu
KD = VD = 128


def _setup(nh, m, seed):
    rng = np.random.default_rng(seed)
    C = nh * (2 * KD + VD)
    proj = rng.standard_normal((m, C + nh * VD + 2 * nh)).astype(np.float32)
    conv_w = (0.5 * rng.standard_normal((C, 4))).astype(np.float32)
    conv_state = rng.standard_normal((3, C, 3)).astype(np.float32)
    state = (0.1 * rng.standard_normal((3, nh, KD, VD))).astype(np.float32)
    neg_a = (-np.exp(0.5 * rng.standard_normal(nh))).astype(np.float32)
    dt_bias = rng.standard_normal(nh).astype(np.float32)
    gate_norm = (1 + 0.1 * rng.standard_normal(VD)).astype(np.float32)
    return proj, conv_w, conv_state, state, neg_a, dt_bias, gate_norm


def _close(got, ref, tol=1e-4):
    got = np.asarray(got, np.float64)
    err = np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30)
    assert err < tol, err


@pytest.mark.parametrize("nh", [1, 4, 16])
@pytest.mark.parametrize("m,spec", [(1, False), (2, True), (3, True), (2, False)])
@pytest.mark.parametrize("slot", [0, 2])
def test_deltanet(cuda, nh, m, spec, slot):
    proj, conv_w, cs, st, neg_a, dtb, gn = _setup(nh, m, seed=nh * 10 + m + slot)
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    dcs, dst = d(cs), d(st)
    params = torch.tensor([7, 8, m, slot], dtype=torch.int32, device=cuda)
    out = ops.deltanet(d(proj), d(conv_w), dcs, dst, d(neg_a), d(dtb), d(gn), params, nh, m, spec=spec)
    torch.cuda.synchronize()
    ref, rcs, rst = odn.deltanet(proj, conv_w, cs, st, neg_a, dtb, gn, nh, m, slot, spec=spec)
    _close(out.cpu().numpy(), ref)
    _close(dcs.cpu().numpy(), rcs)
    _close(dst.cpu().numpy(), rst)
    assert ops.device_error() == 0


def test_deltanet_steps_carry_state(cuda):
    """Eight decode steps in a row: each step reads the state the previous one wrote."""
    nh = 4
    proj, conv_w, cs, st, neg_a, dtb, gn = _setup(nh, 8, seed=3)
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    dcs, dst = d(cs), d(st)
    params = torch.tensor([0, 1, 1, 1], dtype=torch.int32, device=cuda)
    outs = [ops.deltanet(d(proj[t:t + 1]), d(conv_w), dcs, dst, d(neg_a), d(dtb), d(gn), params, nh, 1)
            for t in range(8)]
    torch.cuda.synchronize()
    rcs, rst = cs, st
    for t in range(8):
        ref, rcs, rst = odn.deltanet(proj[t:t + 1], conv_w, rcs, rst, neg_a, dtb, gn, nh, 1, 1)
        _close(outs[t].cpu().numpy(), ref)
    _close(dst.cpu().numpy(), rst)
