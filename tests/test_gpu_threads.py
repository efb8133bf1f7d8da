"""GPU: the library's launch state is per device and thread-safe.  Host threads
make their first calls at the same moment (each raises a kernel's shared-memory
limit on first use), on two streams of one GPU and, when the box has two or more
GPUs, on cuda:0 and cuda:1 from the one process.  Every result must be the
oracle's: the decode GEMV and the streaming lm_head bit for bit, the tcgen05 GEMM
within its 1e-5 bar."""

import threading

import numpy as np
import pytest
import torch

from oracle import c as orc
from webyiq_b200 import ops

from helpers import assert_rel_close, make_weight, make_x

pytestmark = pytest.mark.gpu

K = 2048
N_GEMV, N_HEAD, N_GEMM, M_GEMM = 6144, 16384, 512, 256


def _data():
    out = {}
    for name, n, m, seed in (("gemv", N_GEMV, 1, 1), ("head", N_HEAD, 1, 2), ("gemm", N_GEMM, M_GEMM, 3)):
        q, s, _ = make_weight(n, K, 128, False, seed=seed)
        xq, xs = orc.quant(make_x(m, K, seed=seed + 10), act=1)
        out[name] = (n, q, s, xq, xs, orc.gemv(q, s, K, 128, False, xq, xs, act=1))
    return out


def _worker(dev, data, start, results, idx, reps=3):
    try:
        torch.cuda.set_device(dev)
        stream = torch.cuda.Stream(device=dev)
        with torch.cuda.device(dev), torch.cuda.stream(stream):
            ins = {}
            for name, (n, q, s, xq, xs, _) in data.items():
                w = ops.QWeight(torch.from_numpy(q.view(np.int32)).to(dev), torch.from_numpy(s.view(np.int16)).to(dev),
                                n, K, 128, False)
                ins[name] = (w, torch.from_numpy(xq).to(dev), torch.from_numpy(xs).to(dev))
            torch.cuda.synchronize(dev)
            start.wait()  # every thread's first library calls at once
            got = []
            for _ in range(reps):
                w, xq, xs = ins["gemv"]
                y = ops.gemv(w, xq, xs, act=ops.ACT_TOKEN)
                w, xq, xs = ins["head"]
                _, tok = ops.lmhead_argmax(w, xq, xs, act=ops.ACT_TOKEN)
                w, xq, xs = ins["gemm"]
                yg = ops.gemm(w, xq, xs, act=ops.ACT_TOKEN)
                got.append((y, tok, yg))
            stream.synchronize()
            results[idx] = [(y.cpu().numpy(), int(tok.cpu()[0]), yg.cpu().numpy()) for y, tok, yg in got]
    except Exception as exc:  # reported by the main thread
        results[idx] = exc


def _check(data, res):
    assert not isinstance(res, Exception), res
    for y, tok, yg in res:
        np.testing.assert_array_equal(y.view(np.uint32), data["gemv"][5].view(np.uint32))
        assert tok == int(orc.argmax(data["head"][5])[0])
        assert_rel_close(yg, data["gemm"][5], 1e-5)


def _run(devs):
    data = _data()
    start = threading.Barrier(len(devs))
    results = [None] * len(devs)
    ts = [threading.Thread(target=_worker, args=(d, data, start, results, i)) for i, d in enumerate(devs)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(timeout=300)
    for res in results:
        _check(data, res)


def test_two_threads_one_gpu(cuda):
    _run([cuda, cuda])


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpus_one_process(cuda):
    _run([torch.device("cuda", 0), torch.device("cuda", 1)])
