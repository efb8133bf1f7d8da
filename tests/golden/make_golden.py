"""Generate the golden fixtures in this directory from the reference's own Python.

Run where the reference checkout is present, with its root in the REFERENCE
environment variable; the GPU box and the test suite only read the .npz files.

  convert_q4.npz     tools/convert.py quantize_q4 (group 32, with and without the
                     clip search; group 128) and pack_q4 on the symmetric signed
                     format (codes q+8, min = -8*scale)
  fakequant.npz      tools/reference.py's activation fake-quant (the `fq_input`
                     hook, executed from the reference source) and its fake-quant
                     linear: F.linear(fq_input(x), quantize_q4(W, 32)[2]) in fp32

    REFERENCE=<reference checkout> python tests/golden/make_golden.py
"""

import ast
import os
import sys

import numpy as np
import torch

REF = os.environ.get("REFERENCE", "")
HERE = os.path.dirname(os.path.abspath(__file__))


def reference_fq_input():
    """The `fq_input` forward pre-hook of tools/reference.py (defined inside main()),
    compiled from the reference source as written."""
    path = os.path.join(REF, "tools", "reference.py")
    tree = ast.parse(open(path).read(), path)
    for node in ast.walk(tree):
        if isinstance(node, ast.FunctionDef) and node.name == "fq_input":
            mod = ast.Module(body=[node], type_ignores=[])
            ns = {"torch": torch}
            exec(compile(mod, path, "exec"), ns)
            return ns["fq_input"]
    raise RuntimeError("fq_input not found in reference.py")


def main():
    if not REF or not os.path.isfile(os.path.join(REF, "tools", "convert.py")):
        sys.exit("set REFERENCE to the reference checkout (the directory holding tools/convert.py)")
    sys.path.insert(0, os.path.join(REF, "tools"))
    import convert  # the reference's converter

    rng = np.random.default_rng(20261201)
    out = {}
    # weights with outliers and a constant group (scale 0 path of q4_round)
    w = (rng.standard_normal((24, 256)) * 0.02).astype(np.float32)
    w[3, 40] = 0.5
    w[5, 64:96] = 0.01
    out["w"] = w
    for name, group, search in (("g32", 32, False), ("g32s", 32, True), ("g128", 128, False)):
        p, s, d = convert.quantize_q4(w, group, search)
        out[f"{name}_packed"], out[f"{name}_scales"], out[f"{name}_deq"] = p, s, d
    # symmetric signed int4, group 128, fp16 scale |N(0,1)|*0.01 (the BASELINE format)
    qs = rng.integers(-8, 8, size=(16, 512)).astype(np.int32)
    sc = (np.abs(rng.standard_normal((16, 4))) * 0.01).astype(np.float16)
    p, s = convert.pack_q4((qs + 8).astype(np.uint32), sc, (-8 * sc.astype(np.float32)).astype(np.float16))
    out.update(sym_codes=qs, sym_scale=sc, sym_packed=p, sym_scales_u32=s)
    np.savez_compressed(os.path.join(HERE, "convert_q4.npz"), **out)

    fq_input = reference_fq_input()
    x = rng.standard_normal((4, 256)).astype(np.float32)
    x[1, :32] = 0.0          # an all-zero group (dx = 0)
    x[2, 100] = 30.0         # an outlier
    wl = (rng.standard_normal((40, 256)) * 0.02).astype(np.float32)
    _, wl_s, wl_deq = convert.quantize_q4(wl, 32)
    wl_p = convert.quantize_q4(wl, 32)[0]
    with torch.no_grad():
        xt = torch.from_numpy(x)
        xf = fq_input(None, (xt,))[0]
        y = torch.nn.functional.linear(xf, torch.from_numpy(wl_deq))
    np.savez_compressed(os.path.join(HERE, "fakequant.npz"), x=x, x_fq=xf.numpy(), w=wl, packed=wl_p,
                        scales=wl_s, deq=wl_deq, y=y.numpy())
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    main()
