"""The column-split lm_head's exchange step on CPU: world_size-2 gloo ranks, each
holding half of the vocabulary, merge their packed argmax keys with
ops.merge_shard_keys; the result must be the one-device argmax (oracle) bit for
bit, with ties across shards going to the lowest global index."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import c as orc

from helpers import shard_key, to_i64


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _cases():
    rng = np.random.default_rng(7)
    v = 1000
    cases = []
    a = rng.standard_normal((3, v)).astype(np.float32)
    cases.append(("random", a))
    b = rng.standard_normal((2, v)).astype(np.float32)
    b[0, 100] = b[0, 700] = 9.0  # tie across the two shards: index 100 wins
    b[1, 600] = b[1, 999] = 7.5  # tie inside shard 1
    cases.append(("ties", b))
    c = rng.standard_normal((2, v)).astype(np.float32)
    c[0, 500:] = -np.inf  # shard 1 has no valid value
    c[1, :500] = np.nan  # NaN never wins
    cases.append(("inf_nan", c))
    d = np.full((1, v), np.nan, np.float32)  # no valid value anywhere: token 0
    cases.append(("all_nan", d))
    return cases


def _rank(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from webyiq_b200 import ops

    out = {}
    for name, logits in _cases():
        v = logits.shape[1]
        per = v // world
        lo = rank * per
        keys = torch.tensor([to_i64(shard_key(row[lo:lo + per], lo)) for row in logits], dtype=torch.int64)
        ops.merge_shard_keys(keys)
        out[name] = (keys.tolist(), ops.keys_to_tokens(keys).tolist())
    results[rank] = out
    dist.barrier()
    dist.destroy_process_group()


def test_sharded_argmax_merge_gloo():
    world = 2
    port = _free_port()
    with mp.Manager() as mgr:
        results = mgr.dict()
        mp.spawn(_rank, args=(world, port, results), nprocs=world, join=True)
        got = dict(results)
    for name, logits in _cases():
        ref_tok = orc.argmax(logits)
        ref_key = [to_i64(shard_key(row, 0)) for row in logits]
        for r in range(world):
            keys, toks = got[r][name]
            assert keys == ref_key, (name, r)
            np.testing.assert_array_equal(np.array(toks, np.int64), ref_tok.astype(np.int64), err_msg=name)
