"""The C++ host (webyiq_b200/host: Manifest, Engine, Builder, webyiq_cli) on CPU:
it builds, reads manifests written by webyiq_b200.fmt (the convert.py layout) and
rejects what Manifest::parse rejects (manifest.rs:77-86).  No GPU is touched
(--list only parses the manifest)."""

import json
import subprocess

import numpy as np
import pytest

from webyiq_b200 import build, fmt


@pytest.fixture(scope="module")
def cli():
    return build.build_host()


def _model(tmp_path, name="m", group=32):
    codes = np.random.default_rng(0).integers(0, 16, (64, 256), dtype=np.uint32)
    q = fmt.pack_nibbles(codes)
    kg = 256 // group
    s = fmt.scale_words(np.full((64, kg), 0.01, np.float16), np.full((64, kg), -0.08, np.float16))
    return fmt.write_model(str(tmp_path / name), {"blk.0.up.q": (q, "q4", (64, 256)),
                                                  "blk.0.up.s": (s, "q4s", (64, kg)),
                                                  "norm": (np.ones(256, np.float32), "f32", (256,))}, group=group)


def test_cli_lists_manifest(cli, tmp_path):
    path = _model(tmp_path)
    r = subprocess.run([cli, str(tmp_path / "m"), "--list"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr
    assert "blk.0.up.q" in r.stdout and "64x256" in r.stdout and "group 32" in r.stdout
    m = fmt.Manifest(path)
    for name, t in m.tensors.items():
        assert f"{t['bytes']} bytes" in r.stdout.split(name, 1)[1].splitlines()[0]


@pytest.mark.parametrize("patch,msg", [({"format": "webyiq-v1"}, "unsupported model"),
                                       ({"arch": "gpt2"}, "unsupported model"),
                                       ({"quant": {"bits": 4, "group": 64, "scheme": "x"}}, "unsupported quant"),
                                       ({"quant": {"bits": 8, "group": 32, "scheme": "x"}}, "unsupported quant")])
def test_cli_rejects_bad_manifest(cli, tmp_path, patch, msg):
    path = _model(tmp_path)
    raw = json.load(open(path))
    raw.update(patch)
    json.dump(raw, open(path, "w"))
    r = subprocess.run([cli, str(tmp_path / "m"), "--list"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 2 and msg in r.stderr, (r.returncode, r.stderr)


def test_cli_rejects_broken_json_and_missing_dir(cli, tmp_path):
    path = _model(tmp_path)
    open(path, "w").write('{"format": "webyiq-v2", "arch": ')
    r = subprocess.run([cli, str(tmp_path / "m"), "--list"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 2 and "manifest.json" in r.stderr
    r = subprocess.run([cli, str(tmp_path / "nope"), "--list"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 2 and "cannot read" in r.stderr


def test_symmetric_scales_roundtrip(tmp_path):
    """f16-scale (symmetric, group 128) weights in the manifest layout."""
    codes = np.random.default_rng(1).integers(0, 16, (8, 256), dtype=np.uint32)
    q = fmt.pack_nibbles(codes)
    sc = np.full((8, 2), 0.02, np.float16)
    path = fmt.write_model(str(tmp_path / "s"), {"w.q": (q, "q4", (8, 256)), "w.s": (sc.view(np.uint16), "f16", (8, 2))},
                           group=128, scheme="sym-rtn")
    q2, s2, n, k, g = fmt.Manifest(path).q4("w")
    np.testing.assert_array_equal(q2, q)
    assert s2.dtype == np.uint16 and (s2 == sc.view(np.uint16)).all() and (n, k, g) == (8, 256, 128)
