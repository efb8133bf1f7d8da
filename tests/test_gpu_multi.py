"""The column-split lm_head on every GPU of the box (2 to 8, one rank per GPU): each
rank holds a contiguous shard of the vocabulary rows (the vocabulary is not a
multiple of the world size, so shards differ in size) and the keys are exchanged (a) through torch.distributed NCCL
(ops.lmhead_argmax_sharded), (b) inside the library (w4a8_lmhead_argmax_allreduce
over its own NCCL communicator) and (c) over peer memory (w4a8_lmhead_argmax_xchg:
three calls, so both halves of the double-buffered key slots are used, then two
replays of a captured CUDA graph).  All must give the one-device argmax of the
oracle bit for bit, on every rank.  The same for shards in whole 8-row blocks with
one and two tokens, where the streaming lm_head's last CTA runs the exchange.  Then
rank 0 makes calls rank 1 never joins (through the merge kernel, then inside the
streaming lm_head): each bounded wait must give up with ETIMEOUT and its own key,
and the context must stay usable.  Skipped with fewer than 2 GPUs."""

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import c as orc

from helpers import make_weight, make_x, shard_key, to_i64

pytestmark = pytest.mark.gpu

V, K, M = 8192 + 8 * 3 + 5, 2048, 3  # not a multiple of any world size 2..8
WORLD = min(torch.cuda.device_count(), 8)
# the streaming lm_head's cover (whole 8-row blocks, one or two tokens): its last CTA
# runs the exchange itself; shards of 1037 blocks split as evenly as blocks allow
NB8, M8 = 1037, 2


def _shard(rank, world):
    """Rows [lo, hi) of rank's vocabulary shard (contiguous, sizes differ by <= 1)."""
    return rank * V // world, (rank + 1) * V // world


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _data():
    q, s, _ = make_weight(V, K, 128, False, seed=11)
    xq, xs = orc.quant(make_x(M, K, seed=12), act=1)
    return q, s, xq, xs


def _shard8(rank, world):
    """Rows [lo, hi) of rank's shard of the 8-row-block vocabulary (sizes differ by <= 8)."""
    return rank * NB8 // world * 8, (rank + 1) * NB8 // world * 8


def _data8():
    q, s, _ = make_weight(8 * NB8, K, 128, False, seed=13)
    xq, xs = orc.quant(make_x(M8, K, seed=14), act=1)
    return q, s, xq, xs


def _rank(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    from webyiq_b200 import ops
    from webyiq_b200._lib import ETIMEOUT, W4A8Error

    q, s, xq, xs = _data()
    lo, hi = _shard(rank, world)
    per = hi - lo
    qt = torch.from_numpy(np.ascontiguousarray(q[lo:hi]).view(np.int32)).to(dev)
    st = torch.from_numpy(np.ascontiguousarray(s[lo:hi]).view(np.int16)).to(dev)
    w = ops.QWeight(qt, st, per, K, 128, False)
    xq_d, xs_d = torch.from_numpy(xq).to(dev), torch.from_numpy(xs).to(dev)
    key1, tok1 = ops.lmhead_argmax_sharded(w, xq_d, xs_d, lo, act=ops.ACT_TOKEN)
    store = dist.distributed_c10d._get_default_store()
    if rank == 0:
        store.set("w4a8_nccl_uid", ops.nccl_unique_id())
    uid = store.get("w4a8_nccl_uid")
    comm = ops.NcclComm(world, uid, rank)
    key2, tok2 = ops.lmhead_argmax_allreduce(w, xq_d, xs_d, comm, act=ops.ACT_TOKEN, row_offset=lo)
    torch.cuda.synchronize()
    comm.close()
    xchg = ops.PeerExchange()
    ws = ops.lmhead_workspace(w, M, dev)
    key3 = torch.empty(M, dtype=torch.int64, device=dev)
    tok3 = torch.empty(M, dtype=torch.int32, device=dev)
    got3 = []
    for _ in range(3):
        key3.zero_()
        tok3.zero_()
        ops.lmhead_argmax_xchg(w, xq_d, xs_d, xchg, act=ops.ACT_TOKEN, row_offset=lo, workspace=ws, best_key=key3,
                               tok=tok3)
        torch.cuda.synchronize()
        got3.append((key3.tolist(), tok3.tolist()))
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            ops.lmhead_argmax_xchg(w, xq_d, xs_d, xchg, act=ops.ACT_TOKEN, row_offset=lo, workspace=ws,
                                   best_key=key3, tok=tok3)
    for _ in range(2):
        key3.zero_()
        tok3.zero_()
        g.replay()
        torch.cuda.synchronize()
        got3.append((key3.tolist(), tok3.tolist()))
    del g
    # the fused exchange: shards in whole 8-row blocks, one and two tokens, so the
    # streaming lm_head's last CTA merges the keys (two eager calls, one replay)
    q8, s8, xq8, xs8 = _data8()
    lo8, hi8 = _shard8(rank, world)
    w8 = ops.QWeight(torch.from_numpy(np.ascontiguousarray(q8[lo8:hi8]).view(np.int32)).to(dev),
                     torch.from_numpy(np.ascontiguousarray(s8[lo8:hi8]).view(np.int16)).to(dev),
                     hi8 - lo8, K, 128, False)
    got8 = []
    for m8 in (1, 2):
        xq8_d, xs8_d = torch.from_numpy(xq8[:m8]).to(dev), torch.from_numpy(xs8[:m8]).to(dev)
        ws8 = ops.lmhead_workspace(w8, m8, dev)
        key8 = torch.empty(m8, dtype=torch.int64, device=dev)
        tok8 = torch.empty(m8, dtype=torch.int32, device=dev)
        for _ in range(2):
            key8.zero_()
            tok8.zero_()
            ops.lmhead_argmax_xchg(w8, xq8_d, xs8_d, xchg, act=ops.ACT_TOKEN, row_offset=lo8, workspace=ws8,
                                   best_key=key8, tok=tok8)
            torch.cuda.synchronize()
            got8.append((key8.tolist(), tok8.tolist()))
        g8 = torch.cuda.CUDAGraph()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(g8, stream=s):
                ops.lmhead_argmax_xchg(w8, xq8_d, xs8_d, xchg, act=ops.ACT_TOKEN, row_offset=lo8, workspace=ws8,
                                       best_key=key8, tok=tok8)
        key8.zero_()
        tok8.zero_()
        g8.replay()
        torch.cuda.synchronize()
        got8.append((key8.tolist(), tok8.tolist()))
        del g8
    err = ops.device_error()
    dist.barrier()
    # failure detection: rank 0 makes one more call that no other rank joins; its
    # bounded flag wait gives up, it keeps its own shard's key and the context
    # stays usable
    timeout_seen = None
    if rank == 0:
        key3.zero_()
        ops.lmhead_argmax_xchg(w, xq_d, xs_d, xchg, act=ops.ACT_TOKEN, row_offset=lo, workspace=ws, best_key=key3,
                               tok=tok3)
        try:
            ops.device_error()
            timeout_seen = False
        except W4A8Error as exc:
            timeout_seen = exc.status == ETIMEOUT
        own = ops.lmhead_argmax(w, xq_d, xs_d, act=ops.ACT_TOKEN, row_offset=lo, workspace=ws)[0]
        torch.cuda.synchronize()
        timeout_seen = timeout_seen and key3.tolist() == own.tolist()
        # the same inside the streaming lm_head's last CTA (one token)
        xq8_d, xs8_d = torch.from_numpy(xq8[:1]).to(dev), torch.from_numpy(xs8[:1]).to(dev)
        ws8 = ops.lmhead_workspace(w8, 1, dev)
        key8 = torch.zeros(1, dtype=torch.int64, device=dev)
        ops.lmhead_argmax_xchg(w8, xq8_d, xs8_d, xchg, act=ops.ACT_TOKEN, row_offset=lo8, workspace=ws8,
                               best_key=key8, tok=torch.empty(1, dtype=torch.int32, device=dev))
        try:
            ops.device_error()
            fused_timeout = False
        except W4A8Error as exc:
            fused_timeout = exc.status == ETIMEOUT
        own8 = ops.lmhead_argmax(w8, xq8_d, xs8_d, act=ops.ACT_TOKEN, row_offset=lo8, workspace=ws8)[0]
        torch.cuda.synchronize()
        timeout_seen = timeout_seen and fused_timeout and key8.tolist() == own8.tolist()
    dist.barrier()  # no rank closes its buffer while a peer may still store into it
    xchg.close()
    results[rank] = (key1.tolist(), tok1.tolist(), key2.tolist(), tok2.tolist(), got3, err, timeout_seen, got8)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(WORLD < 2, reason="needs 2 GPUs")
def test_lmhead_split_all_gpus(cuda):
    world = WORLD
    port = _free_port()
    with mp.get_context("spawn").Manager() as mgr:
        results = mgr.dict()
        mp.spawn(_rank, args=(world, port, results), nprocs=world, join=True)
        got = dict(results)
    q, s, xq, xs = _data()
    logits = orc.gemv(q, s, K, 128, False, xq, xs, act=1)
    ref_tok = orc.argmax(logits).astype(np.int64).tolist()
    ref_key = [to_i64(shard_key(row, 0)) for row in logits]
    q8, s8, xq8, xs8 = _data8()
    logits8 = orc.gemv(q8, s8, K, 128, False, xq8, xs8, act=1)
    ref8 = [([to_i64(shard_key(row, 0)) for row in logits8[:m8]], orc.argmax(logits8[:m8]).astype(np.int64).tolist())
            for m8 in (1, 2)]
    for r in range(world):
        key1, tok1, key2, tok2, got3, err, timeout_seen, got8 = got[r]
        assert key1 == ref_key and key2 == ref_key, r
        assert tok1 == ref_tok and tok2 == ref_tok, r
        assert err == 0, r
        for i, (key3, tok3) in enumerate(got3):
            assert key3 == ref_key and tok3 == ref_tok, (r, i)
        for i, (key8, tok8) in enumerate(got8):  # three calls with one token, then three with two
            assert (key8, tok8) == ref8[i // 3], (r, i)
    assert got[0][6] is True  # the unmatched call timed out, kept its own key, context usable
