"""TEST INFRASTRUCTURE ONLY: numpy restatement of the reference's int4 weight format
and round-to-nearest quantizer (rtx527896828/webyIQ tools/convert.py).

  pack_q4      convert.py:68-75   u32 word i of a row holds weights 8i..8i+7,
                                  byte b = w[8i+b] | w[8i+4+b] << 4;
                                  scales u32 = f16 scale | f16 min << 16
  q4_grid      convert.py:55-57   scale = (hi - lo)/15, min = lo, both rounded to f16
  q4_round     convert.py:60-65   q = clip(rint((g - min)/scale), 0, 15), scale 0 -> 1
  quantize_q4  convert.py:78-106  per-group RTN, optional shrink search 1.0 .. 0.7 (16 steps)

Pinned against the reference's own functions by tests/golden/make_golden.py.
"""

import numpy as np

# byte b of word i: low nibble = weight 8i+b, high nibble = weight 8i+4+b
_SHIFT = np.array([0, 8, 16, 24, 4, 12, 20, 28], dtype=np.uint32)


def pack_q4(q, scale, mn):
    """q uint [n, k] in 0..15; scale/mn f16 [n, k/group] -> (u32 [n, k/8], u32 [n, k/group])."""
    n, k = q.shape
    assert k % 8 == 0
    words = (q.astype(np.uint32).reshape(n, k // 8, 8) << _SHIFT).sum(axis=2, dtype=np.uint64)
    packed = words.astype(np.uint32)
    sc = scale.astype(np.float16).view(np.uint16).astype(np.uint32)
    sc |= mn.astype(np.float16).view(np.uint16).astype(np.uint32) << np.uint32(16)
    return packed, sc


def unpack_q4(packed, k):
    """u32 [n, k/8] -> uint8 [n, k] nibbles."""
    n = packed.shape[0]
    w = packed.reshape(n, k // 8, 1) >> _SHIFT
    return (w & np.uint32(15)).astype(np.uint8).reshape(n, k)


def pack_scales_sym(scale):
    """f16 scale [n, k/group] -> the u16 array of the symmetric format."""
    return scale.astype(np.float16).view(np.uint16)


def q4_grid(lo, hi):
    return ((hi - lo) / np.float32(15.0)).astype(np.float16), lo.astype(np.float16)


def q4_round(g, scale, mn):
    s = scale.astype(np.float32)[..., None]
    m = mn.astype(np.float32)[..., None]
    q = np.clip(np.rint((g - m) / np.where(s == 0, np.float32(1.0), s)), 0, 15)
    return q.astype(np.uint32), q.astype(np.float32) * s + m


def quantize_q4(w, group, search=False):
    """Asymmetric RTN int4 of w f32 [n, k] -> (packed u32, scales u32, dequant f32)."""
    n, k = w.shape
    assert k % group == 0 and group % 8 == 0
    g = w.reshape(n, k // group, group)
    lo, hi = g.min(axis=2), g.max(axis=2)
    best_s, best_m = q4_grid(lo, hi)
    if search:
        best_err = np.full(lo.shape, np.inf, np.float32)
        for f in np.linspace(1.0, 0.7, 16):
            s_, m_ = q4_grid(lo * f, hi * f)
            err = ((q4_round(g, s_, m_)[1] - g) ** 2).sum(axis=2)
            better = err < best_err
            best_err = np.where(better, err, best_err)
            best_s = np.where(better, s_, best_s)
            best_m = np.where(better, m_, best_m)
    q, d = q4_round(g, best_s, best_m)
    packed, sc = pack_q4(q.reshape(n, k), best_s, best_m)
    return packed, sc, d.reshape(n, k)


def dequant(packed, scales, k, group, has_min):
    """f32 [n, k] weights of either format."""
    q = unpack_q4(packed, k).astype(np.float32)
    n = packed.shape[0]
    if has_min:
        s = (scales & 0xFFFF).astype(np.uint16).view(np.float16).astype(np.float32)
        m = (scales >> 16).astype(np.uint16).view(np.float16).astype(np.float32)
    else:
        s = scales.astype(np.uint16).view(np.float16).astype(np.float32)
        m = -8.0 * s
    s = np.repeat(s, group, axis=1).reshape(n, k)
    m = np.repeat(m, group, axis=1).reshape(n, k)
    return q * s + m
