"""webyIQ W4A8 hot path on NVIDIA B200 (sm_100a).

The product is the CUDA library lib/libwebyiq_w4a8.so behind the C ABI in
include/w4a8.h.  This package binds it with ctypes (`_lib`), offers the engine's
operator surface on torch CUDA tensors (`ops`, mirroring Builder::{gemv, gemm,
matmul, quant} and the argmax op of crates/engine/src/graph.rs), and reads the
reference's weight format (`fmt`: convert.py packing, manifest.json + shards).
There is no CPU fallback: without the built library every op raises.
"""

from . import fmt, ops  # noqa: F401
from ._lib import W4A8Error  # noqa: F401
