"""The engine's operator surface on torch CUDA tensors, over the C ABI.

Mirrors crates/engine/src/graph.rs: Builder::gemv (:190-198), Builder::gemm
(:200-205), Builder::matmul (:207-214), Builder::quant (:216-222) and the argmax op
of head_ops (:478-486), plus the fused lm_head argmax.  Every call launches on
torch's current CUDA stream and returns without synchronizing; arguments are
checked by the library (W4A8Error with status EINVAL before any launch).
"""

import ctypes

import torch

from . import _lib
from ._lib import ACT_GROUP32, ACT_TOKEN, ADD, GEMV_MAX_M, STORE, SWIGLU  # noqa: F401


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _need_cuda(*ts):
    for t in ts:
        if t is not None and (not t.is_cuda or not t.is_contiguous()):
            raise ValueError("webyiq_b200 ops take contiguous CUDA tensors")


class QWeight:
    """A quantized linear weight in device memory, in the reference's layout.

    q: int32/uint32 tensor [n, k/8] (the u32 words of `{w}.q`);
    s: has_min -> int32/uint32 [n, k/group] (`{w}.s`: f16 scale | f16 min << 16),
       else float16/int16 [n, k/group] (scale only, w = (q-8)*scale).
    """

    def __init__(self, q, s, n, k, group, has_min):
        _need_cuda(q, s)
        self.q, self.s = q, s
        self.n, self.k, self.group, self.has_min = int(n), int(k), int(group), int(bool(has_min))
        self.c = _lib.Weight()
        _lib.check(_lib.load().w4a8_weight_view(_ptr(q), _ptr(s), self.n, self.k, self.group, self.has_min,
                                                ctypes.byref(self.c)))

    def __repr__(self):
        return f"QWeight(n={self.n}, k={self.k}, group={self.group}, has_min={self.has_min})"


def xs_shape(m, k, act):
    return (m,) if act == ACT_TOKEN else (m, k // 32, 2)


def quant(x, norm_w=None, eps=1e-6, act=ACT_GROUP32, xq=None, xs=None):
    """int8 activation quantization of the rows of x f32 [m, k], optionally
    RMSNorm'ed with norm_w (quant.wgsl).  Returns (xq int8 [m, k], xs f32)."""
    _need_cuda(x, norm_w)
    m, k = x.shape
    if xq is None:
        xq = torch.empty((m, k), dtype=torch.int8, device=x.device)
    if xs is None:
        xs = torch.empty(xs_shape(m, k, act), dtype=torch.float32, device=x.device)
    _lib.check(_lib.load().w4a8_quant(_ptr(x), _ptr(norm_w), float(eps), m, k, act, _ptr(xq), _ptr(xs), _stream()))
    return xq, xs


def _out(w, m, mode, y, device):
    n_out = w.n // 2 if mode == SWIGLU else w.n
    if y is None:
        if mode == ADD:
            raise ValueError("mode ADD needs y")
        y = torch.empty((m, n_out), dtype=torch.float32, device=device)
    return y


def gemv(w, xq, xs, act=ACT_GROUP32, mode=STORE, y=None):
    """y (+)= W x for m <= 16 tokens (gemv_q4q8.wgsl)."""
    _need_cuda(xq, xs, y)
    m = xq.shape[0]
    y = _out(w, m, mode, y, xq.device)
    _lib.check(_lib.load().w4a8_gemv(ctypes.byref(w.c), _ptr(xq), _ptr(xs), act, m, mode, _ptr(y), _stream()))
    return y


def gemv_x(w, x, mode=STORE, y=None):
    """Per-token quant of f32 x [m, k] and the GEMV in one launch (group-128 weights);
    equal to quant(act=ACT_TOKEN) followed by gemv, bit for bit."""
    _need_cuda(x, y)
    m = x.shape[0]
    y = _out(w, m, mode, y, x.device)
    _lib.check(_lib.load().w4a8_gemv_x(ctypes.byref(w.c), _ptr(x), m, mode, _ptr(y), _stream()))
    return y


def gemv_xn(w, x, norm_w, eps, mode=STORE, y=None):
    """RMSNorm (norm_w f32 [k], eps), per-token quant and the GEMV in one launch, for
    one or two tokens; equal to quant(x, norm_w, eps, act=ACT_TOKEN) followed by gemv,
    bit for bit."""
    _need_cuda(x, norm_w, y)
    m = x.shape[0]
    y = _out(w, m, mode, y, x.device)
    _lib.check(_lib.load().w4a8_gemv_xn(ctypes.byref(w.c), _ptr(x), _ptr(norm_w), float(eps), m, mode, _ptr(y),
                                        _stream()))
    return y


def gemm(w, xq, xs, act=ACT_GROUP32, mode=STORE, y=None):
    """Y (+)= X W^T for any m (gemm_q4q8.wgsl)."""
    _need_cuda(xq, xs, y)
    m = xq.shape[0]
    y = _out(w, m, mode, y, xq.device)
    _lib.check(_lib.load().w4a8_gemm(ctypes.byref(w.c), _ptr(xq), _ptr(xs), act, m, mode, _ptr(y), _stream()))
    return y


def matmul(w, xq, xs, act=ACT_GROUP32, mode=STORE, y=None):
    """GEMV for m <= 16 tokens, GEMM above (Builder::matmul)."""
    _need_cuda(xq, xs, y)
    m = xq.shape[0]
    y = _out(w, m, mode, y, xq.device)
    _lib.check(_lib.load().w4a8_matmul(ctypes.byref(w.c), _ptr(xq), _ptr(xs), act, m, mode, _ptr(y), _stream()))
    return y


def argmax(logits, ids=None, out=None):
    """Greedy token of every row of logits f32 [m, v] (argmax.wgsl)."""
    _need_cuda(logits, ids, out)
    m, v = logits.shape
    if out is None:
        out = torch.empty(m, dtype=torch.int32, device=logits.device)
    _lib.check(_lib.load().w4a8_argmax(_ptr(logits), m, v, _ptr(ids), _ptr(out), _stream()))
    return out


def group_dots(w, xq):
    """Exact int32 dot of every (token, row, group): int32 [m, n, k/group]."""
    _need_cuda(xq)
    m = xq.shape[0]
    dots = torch.empty((m, w.n, w.k // w.group), dtype=torch.int32, device=xq.device)
    _lib.check(_lib.load().w4a8_group_dots(ctypes.byref(w.c), _ptr(xq), m, _ptr(dots), _stream()))
    return dots


def gemm_group_dots(w, xq):
    """The tcgen05 GEMM's int32 group dots (read back from tensor memory): int32 [m, n, k/128]."""
    _need_cuda(xq)
    m = xq.shape[0]
    dots = torch.empty((m, w.n, w.k // w.group), dtype=torch.int32, device=xq.device)
    _lib.check(_lib.load().w4a8_gemm_group_dots(ctypes.byref(w.c), _ptr(xq), m, _ptr(dots), _stream()))
    return dots


def lmhead_workspace(w, m, device):
    nbytes = _lib.load().w4a8_lmhead_workspace_bytes(w.n, m)
    return torch.zeros(nbytes, dtype=torch.uint8, device=device)


def lmhead_argmax(w, xq, xs, act=ACT_TOKEN, row_offset=0, logits=None, ids=None, workspace=None,
                  best_key=None, tok=None):
    """lm_head GEMV with fused argmax.  Returns (best_key int64 [m] (u64 bits), tok int32 [m])."""
    _need_cuda(xq, xs, logits, ids, workspace)
    m = xq.shape[0]
    dev = xq.device
    if workspace is None:
        workspace = lmhead_workspace(w, m, dev)
    if best_key is None:
        best_key = torch.empty(m, dtype=torch.int64, device=dev)
    if tok is None:
        tok = torch.empty(m, dtype=torch.int32, device=dev)
    _lib.check(_lib.load().w4a8_lmhead_argmax(ctypes.byref(w.c), int(row_offset), _ptr(xq), _ptr(xs), act, m,
                                              _ptr(logits), _ptr(best_key), _ptr(tok), _ptr(ids), _ptr(workspace),
                                              workspace.numel(), _stream()))
    return best_key, tok


def lmhead_argmax_noalloc(w, xq, xs, act=ACT_TOKEN, row_offset=0, logits=None, ids=None, best_key=None, tok=None):
    """lm_head GEMV with fused argmax, using the library's own scratch (no workspace,
    no device allocation; m <= 16).  Returns (best_key int64 [m], tok int32 [m])."""
    _need_cuda(xq, xs, logits, ids)
    m = xq.shape[0]
    dev = xq.device
    if best_key is None:
        best_key = torch.empty(m, dtype=torch.int64, device=dev)
    if tok is None:
        tok = torch.empty(m, dtype=torch.int32, device=dev)
    _lib.check(_lib.load().w4a8_lmhead_argmax_noalloc(ctypes.byref(w.c), int(row_offset), _ptr(xq), _ptr(xs), act, m,
                                                      _ptr(logits), _ptr(best_key), _ptr(tok), _ptr(ids), _stream()))
    return best_key, tok


# ---------------------------------------------------------------------------
# Column-split lm_head over GPUs (vocabulary rows sharded; one exchange of keys).

_SIGN = -(2 ** 63)


def merge_shard_keys(keys, group=None):
    """All-reduce (max) of packed argmax keys (int64 tensor holding u64 bits) over a
    torch.distributed group, in place.  Keys compare as unsigned integers; flipping
    the top bit makes the signed max agree, so any backend (NCCL, gloo) works."""
    import torch.distributed as dist

    keys ^= _SIGN
    dist.all_reduce(keys, op=dist.ReduceOp.MAX, group=group)
    keys ^= _SIGN
    return keys


def keys_to_tokens(keys, ids=None):
    """Token of every packed key (int64 u64 bits) on the keys' device: the index
    (~low word, 0 for the key 0), mapped through ids (int32 [vocab]) if given."""
    low = keys & 0xFFFFFFFF
    idx = torch.where(keys != 0, 0xFFFFFFFF - low, torch.zeros_like(low))
    if ids is not None:
        return ids.to(torch.int64)[idx].to(torch.int32)
    return idx.to(torch.int32)


def lmhead_argmax_sharded(w, xq, xs, row_offset, act=ACT_TOKEN, group=None, ids=None, workspace=None, logits=None):
    """This rank's vocabulary shard (global rows row_offset .. + w.n) through the
    fused lm_head argmax, then the keys merged over the torch.distributed group.
    Returns (best_key int64 [m], tok int32 [m]) of the global argmax on every rank."""
    best_key, _ = lmhead_argmax(w, xq, xs, act=act, row_offset=row_offset, logits=logits, workspace=workspace)
    merge_shard_keys(best_key, group)
    return best_key, keys_to_tokens(best_key, ids)


def gather_rows(w, ids):
    """The draft lm_head of an MTP step: rows ids (int32/uint32 [rows] on the device)
    of w's packed weights and scales, as a new QWeight (gather_rows.wgsl)."""
    _need_cuda(ids)
    rows = ids.numel()
    q = torch.empty((rows, w.k // 8), dtype=torch.int32, device=ids.device)
    sdt = torch.int32 if w.has_min else torch.int16
    s = torch.empty((rows, w.k // w.group), dtype=sdt, device=ids.device)
    _lib.check(_lib.load().w4a8_gather_rows(ctypes.byref(w.c), _ptr(ids), rows, _ptr(q), _ptr(s), _stream()))
    return QWeight(q, s, rows, w.k, w.group, w.has_min)


def spec_accept(tok, y, e, params, ctl, out=None):
    """End of a speculative step (spec_accept.wgsl), all int32 device tensors: tok [2]
    (rewritten), y [2], e [2], params [4] -> ctl [4] (may be params), out [5] or None."""
    _need_cuda(tok, y, e, params, ctl, out)
    _lib.check(_lib.load().w4a8_spec_accept(_ptr(tok), _ptr(y), _ptr(e), _ptr(params), _ptr(ctl), _ptr(out),
                                            _stream()))
    return tok, ctl, out


ATTN_CHUNK = 32


def attn_decode(qkv, kc, vc, H, KVH, D, params, m, chunks=None, part=None):
    """Flash-decoding partials (attn.wgsl): qkv f32 [m, (H + 2 KVH) D], kc / vc f16
    [KVH, maxctx, D], params int32 [4] on the device (pos first).  Returns part f32
    [m, H, maxctx / 32, D + 2]; chunks defaults to all of them."""
    _need_cuda(qkv, kc, vc, params, part)
    maxctx = kc.shape[1]
    nch = maxctx // ATTN_CHUNK
    if part is None:
        part = torch.empty((m, H, nch, D + 2), dtype=torch.float32, device=qkv.device)
    _lib.check(_lib.load().w4a8_attn_decode(_ptr(qkv), _ptr(kc), _ptr(vc), H, KVH, D, maxctx, _ptr(params), m,
                                            nch if chunks is None else chunks, _ptr(part), _stream()))
    return part


def attn_combine(part, H, KVH, D, maxctx, params, m, gsrc=None, want_o=False):
    """The chunks merged per head (attn_combine.wgsl), times sigmoid(gate) with gsrc,
    quantized per 32: -> (xq int8 [m, H D], xs f32 [m, H D / 32, 2], o f32 [m, H, D] or None)."""
    _need_cuda(part, params, gsrc)
    xq = torch.empty((m, H * D), dtype=torch.int8, device=part.device)
    xs = torch.empty((m, H * D // 32, 2), dtype=torch.float32, device=part.device)
    o = torch.empty((m, H, D), dtype=torch.float32, device=part.device) if want_o else None
    _lib.check(_lib.load().w4a8_attn_combine(_ptr(part), H, KVH, D, maxctx, _ptr(params), m, _ptr(gsrc), _ptr(xq),
                                             _ptr(xs), _ptr(o), _stream()))
    return xq, xs, o


def deltanet(proj, conv_w, conv_state, state, neg_a, dt_bias, gate_norm, params, nh, m, eps=1e-6, spec=False,
             out=None):
    """Gated DeltaNet mixer (deltanet.wgsl) on device f32 tensors; conv_state and state
    (three slots each) are updated in place.  Returns out f32 [m, nh * 128]."""
    _need_cuda(proj, conv_w, conv_state, state, neg_a, dt_bias, gate_norm, params, out)
    if out is None:
        out = torch.empty((m, nh * 128), dtype=torch.float32, device=proj.device)
    _lib.check(_lib.load().w4a8_deltanet(_ptr(proj), _ptr(conv_w), _ptr(conv_state), _ptr(state), _ptr(out),
                                         _ptr(neg_a), _ptr(dt_bias), _ptr(gate_norm), _ptr(params), nh, m, eps,
                                         1 if spec else 0, _stream()))
    return out


XCHG_HANDLE_BYTES = 64


class PeerExchange:
    """Peer-memory exchange buffers for w4a8_lmhead_argmax_xchg (one process per GPU
    of one node): this rank's buffer is made on the current device and its CUDA IPC
    handle is all-gathered over the torch.distributed group, then every peer's buffer
    is opened.  Every rank of the group must construct it (collective)."""

    def __init__(self, group=None):
        import torch.distributed as dist

        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.ptr = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(XCHG_HANDLE_BYTES)
        _lib.check(_lib.load().w4a8_xchg_create(self.world, self.rank, handle, ctypes.byref(self.ptr)))
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle.raw), group=group)
        allh = ctypes.create_string_buffer(b"".join(handles), XCHG_HANDLE_BYTES * self.world)
        _lib.check(_lib.load().w4a8_xchg_open(self.ptr, allh))

    def close(self):
        if self.ptr:
            _lib.check(_lib.load().w4a8_xchg_destroy(self.ptr))
            self.ptr = ctypes.c_void_p()


def lmhead_argmax_xchg(w, xq, xs, xchg, act=ACT_TOKEN, row_offset=0, logits=None, ids=None, workspace=None,
                       best_key=None, tok=None, check=False):
    """Sharded lm_head with the key exchange over peer memory (PeerExchange) instead
    of NCCL.  Returns (best_key int64 [m], tok int32 [m]) of the global argmax.

    A peer that does not join within the exchange's bounded wait leaves this rank's
    own shard key in best_key, and only the device error word records it: with
    check=True the call synchronizes the stream and raises W4A8Error (ETIMEOUT) in
    that case; otherwise call device_error() before trusting the tokens (not inside
    a stream capture)."""
    _need_cuda(xq, xs, logits, ids, workspace)
    m = xq.shape[0]
    dev = xq.device
    if workspace is None:
        workspace = lmhead_workspace(w, m, dev)
    if best_key is None:
        best_key = torch.empty(m, dtype=torch.int64, device=dev)
    if tok is None:
        tok = torch.empty(m, dtype=torch.int32, device=dev)
    _lib.check(_lib.load().w4a8_lmhead_argmax_xchg(ctypes.byref(w.c), int(row_offset), _ptr(xq), _ptr(xs), act, m,
                                                   _ptr(logits), _ptr(best_key), _ptr(tok), _ptr(ids),
                                                   _ptr(workspace), workspace.numel(), xchg.ptr, _stream()))
    if check:
        device_error()
    return best_key, tok


def nccl_unique_id():
    """128-byte NCCL unique id (make it on one rank, give it to all)."""
    buf = ctypes.create_string_buffer(128)
    _lib.check(_lib.load().w4a8_nccl_get_unique_id(buf))
    return buf.raw


class NcclComm:
    """An NCCL communicator made by the library (for w4a8_lmhead_argmax_allreduce)."""

    def __init__(self, nranks, uid, rank):
        self.ptr = ctypes.c_void_p()
        buf = ctypes.create_string_buffer(bytes(uid), 128)
        _lib.check(_lib.load().w4a8_nccl_comm_init(int(nranks), buf, int(rank), ctypes.byref(self.ptr)))

    def close(self):
        if self.ptr:
            _lib.check(_lib.load().w4a8_nccl_comm_destroy(self.ptr))
            self.ptr = ctypes.c_void_p()


def lmhead_argmax_allreduce(w, xq, xs, comm, act=ACT_TOKEN, row_offset=0, logits=None, ids=None, workspace=None,
                            best_key=None, tok=None):
    """Sharded lm_head with the key exchange inside the library (NCCL all-reduce of
    the u64 keys over `comm`).  Returns (best_key int64 [m], tok int32 [m])."""
    _need_cuda(xq, xs, logits, ids, workspace)
    m = xq.shape[0]
    dev = xq.device
    if workspace is None:
        workspace = lmhead_workspace(w, m, dev)
    if best_key is None:
        best_key = torch.empty(m, dtype=torch.int64, device=dev)
    if tok is None:
        tok = torch.empty(m, dtype=torch.int32, device=dev)
    _lib.check(_lib.load().w4a8_lmhead_argmax_allreduce(ctypes.byref(w.c), int(row_offset), _ptr(xq), _ptr(xs), act, m,
                                                        _ptr(logits), _ptr(best_key), _ptr(tok), _ptr(ids),
                                                        _ptr(workspace), workspace.numel(), comm.ptr, _stream()))
    return best_key, tok


def key_index(key):
    """Index carried by a packed argmax key (python int, u64 bits)."""
    key &= (1 << 64) - 1
    return (~key) & 0xFFFFFFFF if key else 0


def set_pdl(enable):
    _lib.load().w4a8_set_pdl(1 if enable else 0)


def device_error():
    """Synchronize the current stream and raise W4A8Error(ETIMEOUT) if a kernel's
    bounded wait gave up since the last check."""
    code = ctypes.c_uint32(0)
    _lib.check(_lib.load().w4a8_device_error(ctypes.byref(code), _stream()))
    return code.value


def selftest_wait_timeout():
    """Launch the library's wait-timeout self test (see w4a8.h); read the result
    with device_error()."""
    _lib.check(_lib.load().w4a8_selftest_wait_timeout(_stream()))


def set_gemv_kernel(tensor_core):
    """Group-128 per-token GEMVs on the tensor-core kernel (True) or dp4a (False)."""
    _lib.load().w4a8_set_gemv_kernel(1 if tensor_core else 0)


def set_gemm_kernel(tensor_core):
    """GEMMs the tcgen05 kernel covers on it (True) or on GEMV token blocks (False)."""
    _lib.load().w4a8_set_gemm_kernel(1 if tensor_core else 0)
