"""CPU restatement of the reference's decode attention (test infrastructure only;
parity unpinned: the reference holds no golden vectors for this op and its WGSL cannot
run here, so the restatement follows the shaders' text).

Follows crates/engine/src/shaders/attn.wgsl:41-115 (flash-decoding partials per
chunk of CH = 32 positions) and attn_combine.wgsl:31-83 (the merge of the chunks per
query head, the optional sigmoid gate, and the per-32 int8 quantization of the head
output in the quant.wgsl format).  The partials are computed in float64, so the
GPU's f32 results are compared within a tolerance; the quantization of given head
outputs is restated exactly (f32 arithmetic, rint), so it can be checked bit for bit.

Layouts (per token m of a step):
  qkv  f32 [M, (H + 2 KVH) * D]  q heads first (H rows of D), then k, then v
  kc, vc  f16 [KVH, MAXCTX, D]   the caches
  token m sits at position pos + m and attends to positions 0 ..= pos + m
  gsrc f32 [M, 2 (H + KVH) D]    with GATED, head h's gate is at h * 2D + D
"""

import numpy as np

CH = 32


def attention(qkv, kc, vc, H, KVH, D, pos, m, gsrc=None):
    """Head outputs o f64 [m, H, D]: softmax(q k^T / sqrt(D)) v over positions
    0 ..= pos + t for token t, heads grouped H / KVH per kv head; times
    sigmoid(gate) when gsrc is given (attn_combine.wgsl:57-60)."""
    gq = H // KVH
    q = np.asarray(qkv, np.float64).reshape(m, -1)[:, : H * D].reshape(m, H, D)
    k = np.asarray(kc, np.float32).astype(np.float64)
    v = np.asarray(vc, np.float32).astype(np.float64)
    out = np.zeros((m, H, D))
    for t in range(m):
        n = pos + t + 1
        for h in range(H):
            kh = h // gq
            s = k[kh, :n] @ q[t, h] / np.sqrt(D)
            w = np.exp(s - s.max())
            out[t, h] = (w / w.sum()) @ v[kh, :n]
            if gsrc is not None:
                g = np.asarray(gsrc, np.float64).reshape(m, -1)[t, h * 2 * D + D: h * 2 * D + 2 * D]
                out[t, h] /= 1.0 + np.exp(-g)
    return out


def quant_heads(o):
    """The per-32 int8 quantization of head outputs o f32 [m, H, D]
    (attn_combine.wgsl:64-82, the format of quant.wgsl): per group of 32 within a
    head dx = amax / 127, xq = rint(o * (1 / dx)) (0 when dx = 0), xs = (dx, dx * sum xq).
    Returns xq int8 [m, H * D], xs f32 [m, H * D / 32, 2]."""
    o = np.ascontiguousarray(o, np.float32)
    m, H, D = o.shape
    g = o.reshape(m, H * D // 32, 32)
    amax = np.abs(g).max(axis=2).astype(np.float32)
    dx = (amax / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(dx > 0, np.float32(1.0) / np.where(dx > 0, dx, np.float32(1.0)), np.float32(0.0)).astype(np.float32)
    q = np.rint((g * inv[:, :, None]).astype(np.float32)).astype(np.int32)
    xs = np.stack([dx, (dx * q.sum(axis=2).astype(np.float32)).astype(np.float32)], axis=2).astype(np.float32)
    return q.reshape(m, H * D).astype(np.int8), xs
