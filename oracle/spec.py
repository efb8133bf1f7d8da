"""TEST INFRASTRUCTURE ONLY (see oracle/__init__.py): CPU restatements of the two
small kernels of the MTP speculative step around the hot path.

gather_rows: crates/engine/src/shaders/gather_rows.wgsl:1-24 -- the one-time gather
of the draft lm_head: destination row r is source row ids[r], packed weights and
scales alike (graph.rs:471-516 builds it from the tied embedding and mtp.head_ids).

spec_accept: crates/engine/src/shaders/spec_accept.wgsl:1-38 -- the end of a
speculative step that ran the model on tok = [x, d]: the draft d is accepted when it
equals the greedy token after x (y[0]); the step emits y[0] (and y[1] if accepted),
the next step runs on [y[a], e[a]] at pos + 1 + a, and the DeltaNet state slot
advances to (slot + 1 + a) % 3.
"""

import numpy as np


def gather_rows(q, s, ids):
    """Rows ids of a packed weight (q u32 [n, k/8]) and its scales ([n, k/group])."""
    ids = np.asarray(ids, dtype=np.int64)
    return np.ascontiguousarray(q[ids]), np.ascontiguousarray(s[ids])


def spec_accept(tok, y, e, params):
    """tok [x, d], y [2], e [2], params (pos, seq_len, m, slot) ->
    (new tok [2], ctl (pos, seq_len, m, slot), out [count, y0, y1, pos, slot])."""
    pos, _seq_len, _m, slot = (int(v) for v in params)
    a = 1 if int(tok[1]) == int(y[0]) else 0
    npos = pos + 1 + a
    nslot = (slot + 1 + a) % 3
    new_tok = np.array([y[a], e[a]], dtype=np.uint32)
    ctl = np.array([npos, npos + 2, 2, nslot], dtype=np.uint32)
    out = np.array([1 + a, y[0], y[1], npos, nslot], dtype=np.uint32)
    return new_tok, ctl, out
