"""CPU: the oracle pinned against the reference's own outputs (tests/golden, made by
running the reference's convert.py / reference.py), and its internal consistency."""

import os

import numpy as np
import pytest
import torch

from oracle import c as orc
from oracle import fakequant, layout
from webyiq_b200 import fmt

from helpers import assert_rel_close, make_weight, make_x

GOLD = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def conv():
    return np.load(os.path.join(GOLD, "convert_q4.npz"))


@pytest.fixture(scope="module")
def fq():
    return np.load(os.path.join(GOLD, "fakequant.npz"))


@pytest.mark.parametrize("name,group,search", [("g32", 32, False), ("g32s", 32, True), ("g128", 128, False)])
def test_quantize_q4_matches_reference(conv, name, group, search):
    p, s, d = layout.quantize_q4(conv["w"], group, search)
    np.testing.assert_array_equal(p, conv[f"{name}_packed"])
    np.testing.assert_array_equal(s, conv[f"{name}_scales"])
    np.testing.assert_array_equal(d, conv[f"{name}_deq"])


def test_symmetric_packing_matches_reference(conv):
    codes, sc = conv["sym_codes"], conv["sym_scale"]
    p, s = layout.pack_q4((codes + 8).astype(np.uint32), sc, (-8 * sc.astype(np.float32)).astype(np.float16))
    np.testing.assert_array_equal(p, conv["sym_packed"])
    np.testing.assert_array_equal(s, conv["sym_scales_u32"])
    # the product's packer writes the same words
    q2, s2 = fmt.pack_symmetric(codes, sc)
    np.testing.assert_array_equal(q2, conv["sym_packed"])
    np.testing.assert_array_equal(s2.view(np.uint16).astype(np.uint32), conv["sym_scales_u32"] & 0xFFFF)


def test_unpack_roundtrip(conv):
    k = conv["w"].shape[1]
    codes = layout.unpack_q4(conv["g32_packed"], k)
    np.testing.assert_array_equal(layout.pack_q4(codes, np.zeros((codes.shape[0], 1)), np.zeros((codes.shape[0], 1)))[0],
                                  conv["g32_packed"])
    np.testing.assert_array_equal(fmt.unpack_nibbles(conv["g32_packed"], k), codes)
    np.testing.assert_array_equal(fmt.pack_nibbles(codes), conv["g32_packed"])
    # the C oracle unpacks the same nibbles
    out = np.empty_like(codes)
    orc.lib().orc_unpack(orc._p(np.ascontiguousarray(conv["g32_packed"])), codes.shape[0], k, orc._p(out))
    np.testing.assert_array_equal(out, codes)


def test_dequant_matches_reference(conv):
    k = conv["w"].shape[1]
    d = layout.dequant(conv["g32_packed"], conv["g32_scales"], k, 32, True)
    np.testing.assert_array_equal(d, conv["g32_deq"])


def test_act_fakequant_restatement_matches_reference(fq):
    """oracle/fakequant.py's fq_group32 == the reference's fq_input hook."""
    out = fakequant.fq_group32(torch.from_numpy(fq["x"])).numpy()
    np.testing.assert_array_equal(out, fq["x_fq"])


def test_quant_vs_reference_fakequant(fq):
    """quant.wgsl multiplies by 1/dx where reference.py divides by dx: the int8 codes
    agree except, rarely, one step at a rounding tie."""
    x = fq["x"]
    xq, xs = orc.quant(x, act=0)
    deq = xq.astype(np.float32).reshape(x.shape[0], -1, 32) * xs[..., :1]
    deq = deq.reshape(x.shape)
    diff = np.abs(deq - fq["x_fq"])
    dx = np.repeat(xs[..., 0], 32, axis=1)
    assert (diff <= dx * 1.0001 + 1e-12).all()
    assert (diff > 0).mean() < 0.01
    # dx*sum side data is consistent with the codes
    sums = xq.astype(np.int64).reshape(x.shape[0], -1, 32).sum(-1)
    np.testing.assert_array_equal(xs[..., 1], (xs[..., 0] * sums.astype(np.float32)).astype(np.float32))


def test_gemv_group32_vs_reference_fakequant_linear(fq):
    """The drop-in path (group 32, (scale, min), per-32 activations) against the
    reference's own fake-quant linear, within 1e-3 relative."""
    k = fq["x"].shape[1]
    xq, xs = orc.quant(fq["x"], act=0)
    y = orc.gemv(fq["packed"], fq["scales"], k, 32, True, xq, xs, act=0)
    assert_rel_close(y, fq["y"], 1e-3)


@pytest.mark.parametrize("group,has_min", [(32, True), (32, False), (128, True), (128, False)])
def test_group_dots_exact(group, has_min):
    n, k, m = 24, 512, 3
    q, s, codes = make_weight(n, k, group, has_min, seed=group + has_min)
    xq, _ = orc.quant(make_x(m, k), act=1)
    dots = orc.group_dots(q, k, group, has_min, xq)
    w = codes.astype(np.int64) - (0 if has_min else 8)
    ref = np.einsum("nkg,mkg->mnk", w.reshape(n, k // group, group),
                    xq.astype(np.int64).reshape(m, k // group, group))
    np.testing.assert_array_equal(dots, ref)


@pytest.mark.parametrize("group,has_min", [(32, True), (128, False), (128, True)])
def test_gemv_token_exact_vs_float64(group, has_min):
    """The per-token path equals the exactly rounded result up to its two roundings."""
    n, k, m = 40, 1024, 2
    q, s, _ = make_weight(n, k, group, has_min, seed=7)
    xq, xs = orc.quant(make_x(m, k, seed=3), act=1)
    y = orc.gemv(q, s, k, group, has_min, xq, xs, act=1)
    w = layout.dequant(q, s.astype(np.uint32), k, group, has_min).astype(np.float64)
    ref = (xq.astype(np.float64) @ w.T) * xs[:, None].astype(np.float64)
    assert np.abs(y - ref).max() <= 3e-7 * np.abs(ref).max()


def test_gemv_modes():
    n, k, m = 32, 256, 2
    q, s, _ = make_weight(n, k, 128, False, seed=5)
    xq, xs = orc.quant(make_x(m, k), act=1)
    y0 = orc.gemv(q, s, k, 128, False, xq, xs, act=1, mode=0)
    base = make_x(m, n, seed=9)
    y1 = orc.gemv(q, s, k, 128, False, xq, xs, act=1, mode=1, y=base)
    np.testing.assert_array_equal(y1, (base + y0).astype(np.float32))
    y2 = orc.gemv(q, s, k, 128, False, xq, xs, act=1, mode=2)
    a, u = y0[:, : n // 2].astype(np.float64), y0[:, n // 2:].astype(np.float64)
    np.testing.assert_allclose(y2, a / (1 + np.exp(-a)) * u, rtol=1e-5, atol=1e-7)


def test_quant_norm_deterministic():
    """RMSNorm'ed quant: the fixed-order sum differs from numpy's only by rounding."""
    x = make_x(3, 2048, seed=11)
    nw = (1 + 0.1 * make_x(1, 2048, seed=12)[0]).astype(np.float32)
    xq, xs = orc.quant(x, nw, 1e-6, act=0)
    xq2, xs2 = orc.quant(x, nw, 1e-6, act=0)
    np.testing.assert_array_equal(xq, xq2)
    v = x.astype(np.float64) / np.sqrt((x.astype(np.float64) ** 2).mean(1, keepdims=True) + 1e-6) * nw
    deq = xq.astype(np.float64).reshape(3, -1, 32) * xs[..., :1]
    assert np.abs(deq.reshape(3, -1) - v).max() <= 0.51 * xs[..., 0].max() + 1e-6


def test_argmax_semantics():
    v = 1000
    lg = np.zeros((6, v), np.float32)
    lg[0, 17] = 5.0
    lg[0, 900] = 5.0                      # tie -> lowest index
    lg[1, :] = -np.inf                    # nothing above -3e38 -> 0
    lg[2, :] = np.nan
    lg[2, 123] = 1.0                      # NaN never wins
    lg[3, :] = -1.0
    lg[3, 10] = -0.0
    lg[3, 5] = 0.0                        # -0 == +0 -> lowest index among them
    lg[4, :] = -3.0e38
    lg[4, 999] = -2.9e38                  # -3e38 itself never wins
    lg[5, :] = -5.0
    lg[5, 300] = -4.0
    ids = (np.arange(v, dtype=np.uint32) * 7 + 3)
    np.testing.assert_array_equal(orc.argmax(lg), [17, 0, 123, 5, 999, 300])
    np.testing.assert_array_equal(orc.argmax(lg, ids), ids[[17, 0, 123, 5, 999, 300]])
