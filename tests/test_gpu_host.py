"""The C++ host on the GPU: webyiq_cli loads a converted model directory
(manifest.json + shard, convert.py layout) into device buffers, runs quant +
matmul / the fused lm_head argmax through its Builder, and checks them against
reference outputs made here by the CPU oracle (--ref mode); --bench runs."""

import json
import os
import subprocess

import numpy as np
import pytest

from oracle import c as orc
from webyiq_b200 import build, fmt

from helpers import make_weight, make_x

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cli():
    return build.build_host()


def _write_case(prefix, op, weight, m, act, mode, x, y=None, y0=None, tok=None):
    json.dump({"op": op, "weight": weight, "m": m, "act": "token" if act == 1 else "group32", "mode": mode,
               "eps": 1e-6}, open(prefix + ".json", "w"))
    x.astype(np.float32).tofile(prefix + ".x.f32")
    if y is not None:
        y.astype(np.float32).tofile(prefix + ".y.f32")
    if y0 is not None:
        y0.astype(np.float32).tofile(prefix + ".y0.f32")
    if tok is not None:
        tok.astype(np.uint32).tofile(prefix + ".tok.u32")


def _run(cli, d, *args):
    r = subprocess.run([cli, d, *args], capture_output=True, text=True, timeout=300)
    return r.returncode, r.stdout + r.stderr


@pytest.mark.parametrize("group,has_min,act", [(32, True, 0), (128, False, 1)])
def test_cli_ref_matmul(cuda, cli, tmp_path, group, has_min, act):
    n, k = 256, 1024
    q, s, _ = make_weight(n, k, group, has_min, seed=group)
    sdt = "q4s" if has_min else "f16"
    d = str(tmp_path / "model")
    fmt.write_model(d, {"blk.0.up.q": (q, "q4", (n, k)), "blk.0.up.s": (s, sdt, s.shape)}, group=group,
                    scheme="asym-rtn" if has_min else "sym-rtn")
    for m in (1, 3, 130):
        for mode in (0, 1, 2):
            x = make_x(m, k, seed=m + mode)
            xq, xs = orc.quant(x, None, 1e-6, act=act)
            n_out = n // 2 if mode == 2 else n
            y0 = make_x(m, n_out, seed=99) if mode == 1 else None
            y = orc.gemv(q, s, k, group, has_min, xq, xs, act=act, mode=mode, y=None if y0 is None else y0.copy())
            prefix = str(tmp_path / f"case_m{m}_mode{mode}")
            _write_case(prefix, "matmul", "blk.0.up", m, act, mode, x, y=y, y0=y0)
            rc, out = _run(cli, d, "--ref", prefix)
            assert rc == 0, out
            assert " 0 of " in out, out


@pytest.mark.parametrize("norm", [False, True])
def test_cli_ref_quant_gemv(cuda, cli, tmp_path, norm):
    """Builder::quant_gemv: the norm_quant prologue and the projection in one launch,
    through the C++ host, against the oracle's quant(norm) + gemv."""
    n, k = 512, 2048
    q, s, _ = make_weight(n, k, 128, False, seed=21)
    d = str(tmp_path / "model")
    fmt.write_model(d, {"blk.0.q.q": (q, "q4", (n, k)), "blk.0.q.s": (s, "f16", s.shape)}, group=128,
                    scheme="sym-rtn")
    nw = (1 + 0.2 * make_x(1, k, seed=4)[0]).astype(np.float32) if norm else None
    for m in (1, 2):
        for mode in (0, 1):
            x = make_x(m, k, seed=m + 5 * mode)
            xq, xs = orc.quant(x, nw, 1e-6, act=1)
            y0 = make_x(m, n, seed=98) if mode == 1 else None
            y = orc.gemv(q, s, k, 128, False, xq, xs, act=1, mode=mode, y=None if y0 is None else y0.copy())
            prefix = str(tmp_path / f"qg_m{m}_mode{mode}")
            _write_case(prefix, "quant_gemv", "blk.0.q", m, 1, mode, x, y=y, y0=y0)
            if nw is not None:
                nw.tofile(prefix + ".nw.f32")
            rc, out = _run(cli, d, "--ref", prefix)
            assert rc == 0, out
            assert " 0 of " in out and "one launch" in out, out


def test_cli_ref_lmhead_and_bench(cuda, cli, tmp_path):
    v, k = 4096, 512
    q, s, _ = make_weight(v, k, 128, False, seed=5)
    d = str(tmp_path / "model")
    fmt.write_model(d, {"lm_head.q": (q, "q4", (v, k)), "lm_head.s": (s, "f16", s.shape)}, group=128,
                    scheme="sym-rtn")
    m = 2
    x = make_x(m, k, seed=3)
    xq, xs = orc.quant(x, None, 1e-6, act=1)
    tok = orc.argmax(orc.gemv(q, s, k, 128, False, xq, xs, act=1))
    prefix = str(tmp_path / "head")
    _write_case(prefix, "lm_head", "lm_head", m, 1, 0, x, tok=tok)
    rc, out = _run(cli, d, "--ref", prefix)
    assert rc == 0 and f"{m}/{m} greedy tokens match" in out, out
    rc, out = _run(cli, d, "--bench", "3")
    assert rc == 0 and "decode step" in out, out


def test_cli_reports_truncated_shard(cuda, cli, tmp_path):
    q, s, _ = make_weight(64, 256, 128, False, seed=1)
    d = str(tmp_path / "model")
    fmt.write_model(d, {"w.q": (q, "q4", (64, 256)), "w.s": (s, "f16", s.shape)}, group=128)
    shard = os.path.join(d, "shard-000.bin")
    data = open(shard, "rb").read()
    open(shard, "wb").write(data[:-8])
    rc, out = _run(cli, d, "--bench", "1")
    assert rc == 2 and "past the end" in out, out
