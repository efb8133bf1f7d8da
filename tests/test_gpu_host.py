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


def _model_oracle(layers, x, norm, ffn_norms, gate_ups, downs, head, hd, ffn, eps):
    """The decode step's W4A8 path on the CPU oracle: per layer x += down(quant(
    silu(g) * u)) with (g, u) = gate_up(quant(rmsnorm(x))), then the head."""
    x = x.copy()
    for l in range(layers):
        xq, xs = orc.quant(x, ffn_norms[l], eps, act=1)
        q, s = gate_ups[l]
        h = orc.gemv(q, s, hd, 128, False, xq, xs, act=1, mode=2)
        hq, hs = orc.quant(h, None, eps, act=1)
        q, s = downs[l]
        x = orc.gemv(q, s, ffn, 128, False, hq, hs, act=1, mode=1, y=x.copy())
    xq, xs = orc.quant(x, norm, eps, act=1)
    q, s = head
    logits = orc.gemv(q, s, hd, 128, False, xq, xs, act=1)
    return logits, orc.argmax(logits)


def test_cli_ref_model(cuda, cli, tmp_path):
    """Model-level --ref (the reference CLI's check of a whole model, main.rs:274-318)
    on a synthetic converted model: every layer's norm + quant + SWIGLU gate_up and
    quant + residual down, the final norm and the fused lm_head argmax, through the
    C++ Builder and one captured graph per step, against the oracle chain: greedy
    tokens of every step, last-step logits by cosine, max |diff| and top-10 overlap."""
    layers, hd, ffn, vocab, steps, eps = 4, 1024, 3072, 32000, 3, 1e-6
    tensors, ffn_norms, gate_ups, downs = {}, [], [], []
    for l in range(layers):
        nw = (1 + 0.1 * make_x(1, hd, seed=100 + l)[0]).astype(np.float32)
        ffn_norms.append(nw)
        tensors[f"l{l}.ffn_norm"] = (nw, "f32", (hd,))
        q, s, _ = make_weight(2 * ffn, hd, 128, False, seed=200 + l)
        gate_ups.append((q, s))
        tensors[f"l{l}.gate_up.q"] = (q, "q4", (2 * ffn, hd))
        tensors[f"l{l}.gate_up.s"] = (s, "f16", s.shape)
        q, s, _ = make_weight(hd, ffn, 128, False, seed=300 + l)
        downs.append((q, s))
        tensors[f"l{l}.down.q"] = (q, "q4", (hd, ffn))
        tensors[f"l{l}.down.s"] = (s, "f16", s.shape)
    norm = (1 + 0.1 * make_x(1, hd, seed=7)[0]).astype(np.float32)
    tensors["norm"] = (norm, "f32", (hd,))
    q, s, _ = make_weight(vocab, hd, 128, False, seed=8)
    head = (q, s)
    tensors["lm_head.q"] = (q, "q4", (vocab, hd))
    tensors["lm_head.s"] = (s, "f16", s.shape)
    cfg = {"hidden_size": hd, "intermediate_size": ffn, "num_layers": layers, "num_heads": 8, "num_kv_heads": 8,
           "head_dim": 128, "vocab_size": vocab, "rms_norm_eps": eps}
    d = str(tmp_path / "model")
    fmt.write_model(d, tensors, config=cfg, group=128, scheme="sym-rtn")

    x = make_x(steps, hd, seed=9)
    toks = []
    for t in range(steps):
        logits, tok = _model_oracle(layers, x[t:t + 1], norm, ffn_norms, gate_ups, downs, head, hd, ffn, eps)
        toks.append(int(tok[0]))
    prefix = str(tmp_path / "model_ref")
    json.dump({"op": "model", "steps": steps}, open(prefix + ".json", "w"))
    x.tofile(prefix + ".x.f32")
    logits[0].astype(np.float32).tofile(prefix + ".logits.f32")
    np.array(toks, dtype=np.uint32).tofile(prefix + ".tok.u32")
    rc, out = _run(cli, d, "--ref", prefix)
    assert rc == 0, out
    assert f"greedy: {steps}/{steps} tokens match" in out, out
    assert "top-10 overlap 10/10" in out, out
