"""Decode attention (attn.wgsl) and the merge of its chunks into the o projection's
int8 input (attn_combine.wgsl) on the GPU, against oracle/attn.py: the head outputs
within 2e-5 relative of the float64 restatement (f32 accumulation, expf), their
per-32 quantization bit-exact with the oracle's quantization of the same outputs,
over GQA ratios, head sizes, positions on and off the 32-position chunk boundaries,
two tokens (speculative verify), the sigmoid gate, and a graph replayed at several
positions held on the device.  The oracle restates the shaders; no golden vectors of
the reference exist for this op, so its parity is unpinned."""

import numpy as np
import pytest
import torch

from oracle import attn as oattn
from webyiq_b200 import ops

pytestmark = pytest.mark.gpu


def _case(H, KVH, D, maxctx, m, seed):
    rng = np.random.default_rng(seed)
    qkv = rng.standard_normal((m, (H + 2 * KVH) * D)).astype(np.float32)
    kc = rng.standard_normal((KVH, maxctx, D)).astype(np.float16)
    vc = rng.standard_normal((KVH, maxctx, D)).astype(np.float16)
    gsrc = rng.standard_normal((m, 2 * (H + KVH) * D)).astype(np.float32)
    return qkv, kc, vc, gsrc


def _dev(a, cuda):
    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


def _check(o_gpu, xq, xs, ref):
    o_gpu = o_gpu.cpu().numpy()
    err = np.abs(o_gpu.astype(np.float64) - ref).max() / np.abs(ref).max()
    assert err < 2e-5, err
    rq, rs = oattn.quant_heads(o_gpu)
    np.testing.assert_array_equal(xq.cpu().numpy(), rq)
    np.testing.assert_array_equal(xs.cpu().numpy().view(np.uint32), rs.view(np.uint32))


@pytest.mark.parametrize("H,KVH,D", [(8, 2, 128), (16, 1, 64), (4, 4, 256), (32, 2, 64), (2, 1, 1024)])
@pytest.mark.parametrize("m", [1, 2])
@pytest.mark.parametrize("pos", [0, 30, 31, 32, 95, 777])
def test_attention_decode(cuda, H, KVH, D, m, pos):
    maxctx = 1024
    qkv, kc, vc, gsrc = _case(H, KVH, D, maxctx, m, seed=H + D + m + pos)
    gated = (pos % 2) == 1
    params = torch.tensor([pos, pos + m, m, 0], dtype=torch.int32, device=cuda)
    part = ops.attn_decode(_dev(qkv, cuda), _dev(kc, cuda), _dev(vc, cuda), H, KVH, D, params, m)
    xq, xs, o = ops.attn_combine(part, H, KVH, D, maxctx, params, m, gsrc=_dev(gsrc, cuda) if gated else None,
                                 want_o=True)
    torch.cuda.synchronize()
    ref = oattn.attention(qkv, kc, vc, H, KVH, D, pos, m, gsrc=gsrc if gated else None)
    _check(o, xq, xs, ref)
    assert ops.device_error() == 0


def test_attention_graph_replay_positions(cuda):
    """Captured once, replayed with the position advanced on the device (as a decode
    loop advances it): every replay attends to the new prefix."""
    H, KVH, D, maxctx, m = 8, 2, 128, 512, 1
    qkv, kc, vc, _ = _case(H, KVH, D, maxctx, m, seed=5)
    dq, dk, dv = _dev(qkv, cuda), _dev(kc, cuda), _dev(vc, cuda)
    params = torch.tensor([3, 4, 1, 0], dtype=torch.int32, device=cuda)
    part = torch.empty((m, H, maxctx // 32, D + 2), dtype=torch.float32, device=cuda)
    ops.attn_decode(dq, dk, dv, H, KVH, D, params, m, part=part)  # first call outside capture
    out = {}
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g):
            ops.attn_decode(dq, dk, dv, H, KVH, D, params, m, part=part)
            out["xq"], out["xs"], out["o"] = ops.attn_combine(part, H, KVH, D, maxctx, params, m, want_o=True)
    for pos in (3, 31, 64, 300, 511):
        params[0] = pos
        g.replay()
        torch.cuda.synchronize()
        _check(out["o"], out["xq"], out["xs"], oattn.attention(qkv, kc, vc, H, KVH, D, pos, m))
    del g
    assert ops.device_error() == 0


def test_attention_feeds_the_o_projection(cuda):
    """The combine's (xq, xs) is the W4A8_ACT_GROUP32 input of the o projection
    (graph.rs:286-290): the GEMV on it equals the GEMV on the same activations
    quantized by w4a8_quant from the head outputs."""
    from helpers import assert_rel_close, make_weight
    from oracle import c as orc

    H, KVH, D, maxctx, m, pos = 8, 2, 128, 256, 1, 100
    qkv, kc, vc, _ = _case(H, KVH, D, maxctx, m, seed=11)
    params = torch.tensor([pos, pos + 1, 1, 0], dtype=torch.int32, device=cuda)
    part = ops.attn_decode(_dev(qkv, cuda), _dev(kc, cuda), _dev(vc, cuda), H, KVH, D, params, m)
    xq, xs, o = ops.attn_combine(part, H, KVH, D, maxctx, params, m, want_o=True)
    q, s, _ = make_weight(512, H * D, 32, True, seed=3)
    w = ops.QWeight(_dev(q.view(np.int32), cuda), _dev(s.view(np.int32), cuda), 512, H * D, 32, True)
    y = ops.gemv(w, xq, xs.reshape(m, -1), act=ops.ACT_GROUP32)
    torch.cuda.synchronize()
    oq, os_ = orc.quant(o.cpu().numpy().reshape(m, H * D), act=0)
    np.testing.assert_array_equal(xq.cpu().numpy(), oq)
    np.testing.assert_array_equal(xs.cpu().numpy().reshape(os_.shape).view(np.uint32), os_.view(np.uint32))
    ref = orc.gemv(q, s, H * D, 32, True, oq, os_, act=0)
    assert_rel_close(y.cpu().numpy(), ref, 1e-3)  # the per-group-32 f32 path's bar
