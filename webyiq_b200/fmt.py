"""The reference's weight format on the host side: int4 packing, scale words,
manifest.json + shard loading (rtx527896828/webyIQ tools/convert.py and
crates/engine/src/manifest.rs), and seeded synthetic weights.

  q  u32[n, k/8]       word i holds weights 8i..8i+7: byte b = w[8i+b] | w[8i+4+b] << 4
  s  u32[n, k/group]   f16 scale | f16 min << 16        (w = q*scale + min; convert.py)
     f16[n, k/group]   scale only                        (w = (q-8)*scale; symmetric)
"""

import json
import os

import numpy as np

FORMAT = "webyiq-v2"
ALIGN = 256
_SHIFTS = np.array([0, 8, 16, 24, 4, 12, 20, 28], dtype=np.uint32)


def pack_nibbles(q):
    """uint [n, k] in 0..15 -> u32 [n, k/8] in the engine's nibble order."""
    n, k = q.shape
    if k % 8:
        raise ValueError("k must be a multiple of 8")
    q = np.asarray(q, dtype=np.uint32).reshape(n, k // 8, 8)
    out = np.zeros((n, k // 8), np.uint32)
    for j in range(8):
        out |= q[:, :, j] << _SHIFTS[j]
    return out


def unpack_nibbles(packed, k):
    """u32 [n, k/8] -> uint8 [n, k]."""
    n = packed.shape[0]
    return ((packed.reshape(n, k // 8, 1) >> _SHIFTS) & 15).astype(np.uint8).reshape(n, k)


def scale_words(scale, mn):
    """f16 scale, f16 min [n, g] -> u32 words (scale low, min high)."""
    return (np.asarray(scale, np.float16).view(np.uint16).astype(np.uint32)
            | (np.asarray(mn, np.float16).view(np.uint16).astype(np.uint32) << 16))


def pack_symmetric(codes, scale):
    """signed codes int [n, k] in -8..7 and f16 scale [n, k/group] -> (q u32, s f16)."""
    codes = np.asarray(codes)
    if codes.min() < -8 or codes.max() > 7:
        raise ValueError("symmetric int4 codes must be in [-8, 7]")
    return pack_nibbles(codes + 8), np.asarray(scale, np.float16)


# ---------------------------------------------------------------------------
class Manifest:
    """manifest.json of a converted model (manifest.rs:6-95)."""

    def __init__(self, path):
        self.dir = os.path.dirname(os.path.abspath(path))
        with open(path) as f:
            m = json.load(f)
        # Manifest::parse (manifest.rs:77-86)
        if m.get("format") != FORMAT or m.get("arch") not in ("llama", "qwen3_5"):
            raise ValueError(f"unsupported model: {m.get('format')} / {m.get('arch')}")
        q = m.get("quant", {})
        if q.get("bits") != 4 or q.get("group") not in (32, 128):
            raise ValueError(f"unsupported quant: {q}")
        self.raw = m
        self.config = m["config"]
        self.group = q["group"]
        self.shards = m["shards"]
        self.tensors = m["tensors"]

    def shard_bytes(self):
        sizes = [0] * len(self.shards)
        for t in self.tensors.values():
            sizes[t["shard"]] = max(sizes[t["shard"]], t["offset"] + t["bytes"])
        return sizes

    def read(self, name):
        """Raw bytes of one tensor as a numpy array of its dtype."""
        t = self.tensors[name]
        path = os.path.join(self.dir, self.shards[t["shard"]])
        size = os.path.getsize(path)
        if t["offset"] + t["bytes"] > size:
            raise ValueError(f"tensor {name} past the end of {path} ({t['offset']}+{t['bytes']} > {size})")
        raw = np.fromfile(path, dtype=np.uint8, count=t["bytes"], offset=t["offset"])
        dt = {"q4": np.uint32, "q4s": np.uint32, "f32": np.float32, "u32": np.uint32, "f16": np.float16}[t["dtype"]]
        return raw.view(dt)

    def q4(self, name):
        """(q u32 [n, k/8], s, n, k, group) of a quantized weight `name`; s is u32
        [n, k/group] (f16 scale | f16 min << 16, convert.py) or, for symmetric
        weights, u16 [n, k/group] (f16 scale bits)."""
        tq, ts = self.tensors[name + ".q"], self.tensors[name + ".s"]
        n, k = tq["shape"]
        kg = k // self.group if self.group else 0
        if k % self.group or tq["bytes"] != n * k // 2 or ts["bytes"] not in (n * kg * 4, n * kg * 2):
            raise ValueError(f"tensor {name}: sizes do not match shape {n}x{k} group {self.group}")
        s = self.read(name + ".s")
        s = s.view(np.uint32 if ts["bytes"] == n * kg * 4 else np.uint16).reshape(n, kg)
        return self.read(name + ".q").reshape(n, k // 8), s, n, k, self.group


def write_model(out_dir, tensors, config=None, arch="llama", group=32, scheme="asym-rtn"):
    """Write manifest.json + one shard of `tensors` ({name: (array, dtype, shape)}),
    256-byte aligned like ShardWriter.add (convert.py:138-153)."""
    os.makedirs(out_dir, exist_ok=True)
    table = {}
    pos = 0
    with open(os.path.join(out_dir, "shard-000.bin"), "wb") as f:
        for name, (arr, dtype, shape) in tensors.items():
            data = np.ascontiguousarray(arr).tobytes()
            pad = (-pos) % ALIGN
            f.write(b"\0" * pad)
            pos += pad
            table[name] = {"shard": 0, "offset": pos, "bytes": len(data), "dtype": dtype, "shape": list(shape)}
            f.write(data)
            pos += len(data)
    manifest = {"format": FORMAT, "arch": arch, "config": config or {},
                "quant": {"bits": 4, "group": group, "scheme": scheme}, "shards": ["shard-000.bin"],
                "tensors": table}
    with open(os.path.join(out_dir, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1)
    return os.path.join(out_dir, "manifest.json")
