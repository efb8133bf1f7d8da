"""Build the sm_100a CUDA library in-tree: webyiq_b200/lib/libwebyiq_w4a8.so.

Every .cu file under csrc/ is compiled separately (in parallel) with
`nvcc -gencode arch=compute_100a,code=sm_100a -lineinfo -O3` and linked into one
shared library with the CUDA runtime linked statically, so the library needs
nothing at run time beyond the driver.  Objects are cached by content hash of the
sources under webyiq_b200/_build/.
"""

import concurrent.futures as cf
import hashlib
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.environ.get("W4A8_BUILD_DIR", os.path.join(HERE, "_build"))
LIBDIR = os.path.join(HERE, "lib")
LIB = os.environ.get("W4A8_LIB_OUT", os.path.join(LIBDIR, "libwebyiq_w4a8.so"))
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", f"-I{os.path.join(ROOT, 'include')}"]
FLAGS += os.environ.get("W4A8_NVCC_FLAGS", "").split()


def _headers_digest():
    h = hashlib.sha256()
    for d in (CSRC, os.path.join(ROOT, "include")):
        for fn in sorted(os.listdir(d)):
            if fn.endswith((".cuh", ".h")):
                with open(os.path.join(d, fn), "rb") as f:
                    h.update(fn.encode() + f.read())
    return h.hexdigest()


def _compile(src, digest, verbose):
    with open(src, "rb") as f:
        key = hashlib.sha256(f.read() + digest.encode() + " ".join(ARCH + FLAGS).encode()).hexdigest()[:16]
    obj = os.path.join(BUILD, f"{os.path.basename(src)}.{key}.o")
    if os.path.exists(obj):
        return obj
    cmd = [NVCC, *ARCH, *FLAGS, "-c", src, "-o", obj + ".tmp"]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
    if verbose and r.stderr:
        print(r.stderr, file=sys.stderr)
    os.replace(obj + ".tmp", obj)
    return obj


def build(verbose=False, jobs=None):
    """Compile csrc/*.cu for sm_100a and link the shared library; returns its path."""
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    digest = _headers_digest()
    srcs = sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))
    with cf.ThreadPoolExecutor(max_workers=jobs or os.cpu_count()) as ex:
        objs = list(ex.map(lambda s: _compile(s, digest, verbose), srcs))
    keep = set(objs)
    for fn in os.listdir(BUILD):  # drop objects of earlier sources
        path = os.path.join(BUILD, fn)
        if path not in keep and fn.endswith(".o"):
            os.remove(path)
    link_key = hashlib.sha256("".join(objs).encode()).hexdigest()[:16]
    stamp = LIB + ".stamp"
    if os.path.exists(LIB) and os.path.exists(stamp) and open(stamp).read() == link_key:
        return LIB
    cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", LIB + ".tmp", *objs, "-lpthread", "-ldl", "-lrt"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(LIB + ".tmp", LIB)
    with open(stamp, "w") as f:
        f.write(link_key)
    return LIB


HOST = os.path.join(HERE, "host")
CLI = os.path.join(LIBDIR, "webyiq_cli")
CXX = os.environ.get("CXX", "g++")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def build_host():
    """Compile the C++ host (host/*.cpp: manifest, engine, Builder, CLI) against the
    shared library and the CUDA runtime; returns the path of lib/webyiq_cli."""
    lib = build()
    srcs = sorted(os.path.join(HOST, f) for f in os.listdir(HOST) if f.endswith(".cpp"))
    h = hashlib.sha256()
    for p in srcs + sorted(os.path.join(HOST, f) for f in os.listdir(HOST) if f.endswith(".h")) + \
            [os.path.join(ROOT, "include", "w4a8.h")]:
        with open(p, "rb") as f:
            h.update(p.encode() + f.read())
    h.update(open(lib + ".stamp").read().encode() if os.path.exists(lib + ".stamp") else b"")
    key = h.hexdigest()[:16]
    stamp = CLI + ".stamp"
    if os.path.exists(CLI) and os.path.exists(stamp) and open(stamp).read() == key:
        return CLI
    cmd = [CXX, "-O2", "-std=c++17", "-Wall", "-Wextra", f"-I{os.path.join(ROOT, 'include')}", f"-I{HOST}",
           f"-I{CUDA_HOME}/include", *srcs, "-o", CLI + ".tmp", f"-L{LIBDIR}", "-lwebyiq_w4a8",
           f"-L{CUDA_HOME}/lib64", "-lcudart", f"-Wl,-rpath,$ORIGIN:{CUDA_HOME}/lib64"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"host build failed:\n{r.stdout}\n{r.stderr}")
    os.replace(CLI + ".tmp", CLI)
    with open(stamp, "w") as f:
        f.write(key)
    return CLI


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
    if "--host" in sys.argv:
        print(build_host())
