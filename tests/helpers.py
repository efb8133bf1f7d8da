"""Seeded synthetic inputs shared by the tests (numpy, host side)."""

import numpy as np

from oracle import layout


def make_weight(n, k, group, has_min, seed=0, scale=0.01):
    """Random int4 codes with f16 scales |N(0,1)|*scale (and mins for has_min).
    Returns (q u32 [n, k/8], s (u32 | u16) [n, k/group], codes uint8 [n, k])."""
    rng = np.random.default_rng(seed)
    codes = rng.integers(0, 16, size=(n, k), dtype=np.uint32)
    sc = (np.abs(rng.standard_normal((n, k // group))) * scale).astype(np.float16)
    if has_min:
        mn = (-(0.5 + rng.random((n, k // group))) * 7.5 * sc.astype(np.float32)).astype(np.float16)
        q, s = layout.pack_q4(codes, sc, mn)
    else:
        q, _ = layout.pack_q4(codes, sc, np.zeros_like(sc))
        s = layout.pack_scales_sym(sc)
    return q, s, codes.astype(np.uint8)


def make_x(m, k, seed=1):
    return np.random.default_rng(seed).standard_normal((m, k)).astype(np.float32)


def assert_rel_close(y, ref, rtol=1e-3):
    """fp parity bar: max|y-ref| <= rtol*max|ref| and, element-wise,
    |y-ref| <= rtol*|ref| + rtol*rms(ref)."""
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    assert y.shape == ref.shape, (y.shape, ref.shape)
    err = np.abs(y - ref)
    scale = max(np.abs(ref).max(), 1e-30)
    rms = np.sqrt(np.mean(ref ** 2)) if ref.size else 0.0
    assert err.max() <= rtol * scale, f"normwise rel err {err.max() / scale:.3g} > {rtol}"
    bad = err > rtol * np.abs(ref) + rtol * rms
    assert not bad.any(), f"{bad.sum()} elements out of tolerance, worst {err[bad].max():.3g}"


def pack_key(v, idx):
    """Packed argmax key of value v at global index idx, as u64 (argmax.wgsl:17-39
    order: larger value first, then lower index; NaN and values <= -3e38 give 0)."""
    v = np.float32(v)
    if not (v > np.float32(-3e38)):
        return 0
    if v == 0:
        v = np.float32(0.0)
    b = int(np.array([v], np.float32).view(np.uint32)[0])
    b = (~b & 0xFFFFFFFF) if b & 0x80000000 else (b | 0x80000000)
    return (b << 32) | (~int(idx) & 0xFFFFFFFF)


def shard_key(logits_row, offset):
    """Best packed key of one row of a vocabulary shard whose first row is `offset`."""
    best = 0
    for j, v in enumerate(logits_row):
        best = max(best, pack_key(v, offset + j))
    return best


def to_i64(u):
    """u64 bits as a signed int64 value (for torch int64 tensors)."""
    return u - (1 << 64) if u >= (1 << 63) else u
