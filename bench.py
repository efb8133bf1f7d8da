"""Benchmark of the W4A8 hot path on B200 (the driver's contract: one JSON line).

Headline workload ("decode projection sweep"): M=1 W4A8 GEMV
over (K, N) = (2048,2048) (2048,4096) (2048,6144) (6144,2048) (4096,2048) (2048,512),
24 distinct layers (144 weight tensors, 586 MB of packed int4 + fp16 scales, far
larger than the 126 MB L2), run back to back as one decode step's matvec sequence.
Weights: signed int4 uniform in [-8, 7] (uniform random nibbles), group 128, fp16
scales |N(0,1)|*0.01; activations fp32 N(0,1) quantized per token to int8.

  value   algorithmic GB/s of the step (packed weights + scales + activations +
          outputs per projection), inputs resident in HBM, the 144 GEMV launches
          replayed as one CUDA graph with programmatic dependent launch between
          them;
  e2e     the same metric through the public API with host buffers: per step the
          pinned-host -> device copies of the 144 fp32 input vectors, 144 launches
          of the GEMV with the per-token quant fused in (w4a8_gemv_x), and the
          device -> host copies of all outputs; the copies of later layers' inputs
          and earlier layers' outputs overlap the chain on a side stream;
  extra   secondary BASELINE metrics from the same run: config 1 (single GEMV),
          config 3 (lm_head + fused argmax, tok/s), config 4 (prefill GEMM, TOPS),
          config 5 (batched GEMV, M = 2..16).

--impl reference times the reference's CPU path (tools/reference.py: int4 weights
dequantized once, int8 activation fake-quant + fp32 F.linear per projection) on
the host cores, for the same metric and config; its `extra` holds config 3 (the
lm_head over the 248,320-token vocabulary plus argmax) through the same path.

Multi-GPU (torchrun, one rank per GPU): the decode sweep runs as independent
replicas (weak scaling, no collective); value = all ranks' bytes / max-over-ranks
time.  The column-split lm_head with an all-reduce of packed (logit, index) keys is
measured as an extra.
"""

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

SWEEP = [(2048, 2048), (2048, 4096), (2048, 6144), (6144, 2048), (4096, 2048), (2048, 512)]
LAYERS = 24
GROUP = 128


def gemv_bytes(k, n, m=1, group=GROUP):
    """Algorithmic bytes of one W4A8 GEMV, per-token activations, fp16 scales:
    packed weights + scales + int8 activations + per-token scale + fp32 output."""
    return n * k // 2 + n * (k // group) * 2 + m * k + m * 4 + m * n * 4


def step_bytes():
    return LAYERS * sum(gemv_bytes(k, n) for k, n in SWEEP)


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p.get("bf16_tflops", 1590.0)), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


# ---------------------------------------------------------------------------
class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons during a timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", str(self.idx)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        rows = []
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                rows.append((float(f[1]), float(f[2]), f[5:9]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i, v in enumerate(r[2]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------
def rand_weight(n, k, group, gen, dev, torch, ops):
    """Uniform random nibbles (= signed int4 uniform in [-8, 7]) and fp16 scales
    |N(0,1)|*0.01, generated on the device."""
    q = torch.randint(-2 ** 31, 2 ** 31 - 1, (n, k // 8), dtype=torch.int32, device=dev, generator=gen)
    s = (torch.randn((n, k // group), device=dev, generator=gen).abs() * 0.01).half()
    return ops.QWeight(q, s, n, k, group, False)


def time_graph(torch, fn, steps, warmup, sync_all=None):
    """Capture fn() in a CUDA graph, replay W times untimed then K times between
    events; returns (ms per step, graph)."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()  # eager once (also warms the library)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    for _ in range(warmup):
        g.replay()
    torch.cuda.synchronize()
    if sync_all:
        sync_all()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    if sync_all:
        sync_all()
    return e0.elapsed_time(e1) / steps, g


C3_CALLS = 4  # lm_head calls per captured graph in the C3 timing


class Sweep:
    """The decode-projection sweep: 24 layers x 6 shapes of distinct weights."""

    def __init__(self, torch, ops, dev, seed):
        self.torch, self.ops, self.dev = torch, ops, dev
        gen = torch.Generator(device=dev)
        gen.manual_seed(seed)
        self.w = [[rand_weight(n, k, GROUP, gen, dev, torch, ops) for k, n in SWEEP] for _ in range(LAYERS)]
        ks = sorted({k for k, _ in SWEEP})
        self.x = {k: torch.randn((1, k), device=dev, generator=gen) for k in ks}
        self.act = {k: ops.quant(self.x[k], act=ops.ACT_TOKEN) for k in ks}
        self.y = {(k, n): torch.empty((1, n), device=dev) for k, n in SWEEP}
        # e2e: host inputs for every projection, and device staging
        self.nin = LAYERS * sum(k for k, _ in SWEEP)
        self.nout = LAYERS * sum(n for _, n in SWEEP)
        self.h_in = torch.randn(self.nin, generator=torch.Generator().manual_seed(seed)).pin_memory()
        self.h_out = torch.empty(self.nout).pin_memory()
        self.d_in = torch.empty(self.nin, device=dev)
        self.d_out = torch.empty(self.nout, device=dev)
        self.side = torch.cuda.Stream(device=dev)  # e2e: copies that overlap the GEMV chain

    def step(self):
        ops = self.ops
        for layer in self.w:
            for (k, n), w in zip(SWEEP, layer):
                xq, xs = self.act[k]
                ops.gemv(w, xq, xs, act=ops.ACT_TOKEN, y=self.y[(k, n)])

    def step_e2e(self):
        """One step from pinned host buffers: every input goes up and every output comes
        down inside the step.  The inputs of layers 0-1 are copied first; the other
        layers' inputs go up on a side stream while those two run, and the outputs of
        all but the last two layers come down on the side stream while those two run.
        The GEMV chain waits for the side stream once: a kernel that waits on another
        stream starts only when its predecessor has finished (no early launch), which
        costs about 6 us per wait."""
        torch, ops = self.torch, self.ops
        main, side = torch.cuda.current_stream(), self.side
        fin, fout = sum(k for k, _ in SWEEP), sum(n for _, n in SWEEP)  # floats per layer
        self.d_in[:2 * fin].copy_(self.h_in[:2 * fin], non_blocking=True)
        side.wait_stream(main)
        with torch.cuda.stream(side):
            self.d_in[2 * fin:].copy_(self.h_in[2 * fin:], non_blocking=True)
            up_rest = torch.cuda.Event()
            up_rest.record(side)
        tail = LAYERS - 2  # first layer whose outputs the main stream copies down
        i = o = 0
        for li, layer in enumerate(self.w):
            if li == 2:
                main.wait_event(up_rest)
            elif li == tail:
                side.wait_stream(main)
                with torch.cuda.stream(side):
                    self.h_out[:tail * fout].copy_(self.d_out[:tail * fout], non_blocking=True)
            for (k, n), w in zip(SWEEP, layer):
                x = self.d_in[i:i + k].view(1, k)
                # per-token quant fused into the GEMV launch (w4a8_gemv_x)
                ops.gemv_x(w, x, y=self.d_out[o:o + n].view(1, n))
                i, o = i + k, o + n
        self.h_out[tail * fout:].copy_(self.d_out[tail * fout:], non_blocking=True)
        main.wait_stream(side)

    launches_per_step = LAYERS * len(SWEEP)


def measure_int8_peak(torch, dev, size=8192, reps=5):
    """Dense int8 tensor-core throughput of the library GEMM (cuBLAS via
    torch._int_mm) on this GPU, TOPS; None if unavailable."""
    try:
        a = torch.randint(-128, 127, (size, size), dtype=torch.int8, device=dev)
        b = torch.randint(-128, 127, (size, size), dtype=torch.int8, device=dev).t()
        for _ in range(2):
            torch._int_mm(a, b)
        torch.cuda.synchronize()
        best = None
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch._int_mm(a, b)
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1)
            best = ms if best is None else min(best, ms)
        del a, b
        return 2 * size ** 3 / (best * 1e-3) / 1e12
    except Exception:
        return None


# ---------------------------------------------------------------------------
def run_extras(torch, ops, dev, steps, warmup, world, rank, dist):
    """Secondary BASELINE configs, timed with CUDA graphs on this GPU."""
    out = {}
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234)
    hbm, _, _ = peaks()
    # config 1: one GEMV; rotate over 32 copies (208 MB) so every launch reads HBM
    k, n = 2048, 6144
    ws = [rand_weight(n, k, GROUP, gen, dev, torch, ops) for _ in range(32)]
    xq, xs = ops.quant(torch.randn((1, k), device=dev, generator=gen), act=ops.ACT_TOKEN)
    y = torch.empty((1, n), device=dev)

    def c1():
        for w in ws:
            ops.gemv(w, xq, xs, act=ops.ACT_TOKEN, y=y)

    ms, g = time_graph(torch, c1, steps, warmup)
    del g
    per = ms / len(ws)
    out["c1_gemv"] = {"us": round(per * 1e3, 3), "gbs": round(gemv_bytes(k, n) / (per * 1e-3) / 1e9, 1),
                      "frac_hbm": round(gemv_bytes(k, n) / (per * 1e-3) / 1e9 / hbm, 3)}
    del ws
    def max_ms(ms):
        if world == 1:
            return ms
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    sync_all = (lambda: dist.barrier()) if world > 1 else None
    # config 5: batched decode / verify, M in {2, 4, 8, 16}, rotating weights; at
    # N > 1 every rank runs its own replica (no collective) and the aggregate is all
    # ranks' bytes over the max-over-ranks time
    c5 = {}
    for k, n in ((2048, 6144), (6144, 2048)):
        ws = [rand_weight(n, k, GROUP, gen, dev, torch, ops) for _ in range(16)]
        for m in (2, 4, 8, 16):
            xq, xs = ops.quant(torch.randn((m, k), device=dev, generator=gen), act=ops.ACT_TOKEN)
            y = torch.empty((m, n), device=dev)

            def c5f():
                for w in ws:
                    ops.gemv(w, xq, xs, act=ops.ACT_TOKEN, y=y)

            ms, g = time_graph(torch, c5f, max(steps // 2, 3), warmup, sync_all)
            del g
            per = max_ms(ms) / len(ws)
            gbs = gemv_bytes(k, n, m) / (per * 1e-3) / 1e9
            c5[f"{k}x{n}_m{m}"] = {"us": round(per * 1e3, 3), "gbs_per_gpu": round(gbs, 1),
                                   "gbs_all_gpus": round(world * gbs, 1),
                                   "tokens_s_all_gpus": round(world * m / (per * 1e-3), 1)}
        del ws
    c5["replicas"] = world
    c5["timing"] = "per GPU: max over ranks of the CUDA-event time; all GPUs: world x bytes (or tokens) / that time"
    out["c5_batched_gemv"] = c5
    # config 3: lm_head + fused argmax, vocab column-split over the ranks
    k, vocab = 2048, 248320
    per_rank = vocab // world
    w = rand_weight(per_rank, k, GROUP, gen, dev, torch, ops)
    xq, xs = ops.quant(torch.randn((1, k), device=dev, generator=gen), act=ops.ACT_TOKEN)
    wsp = ops.lmhead_workspace(w, 1, dev)
    key = torch.empty(1, dtype=torch.int64, device=dev)
    tok = torch.empty(1, dtype=torch.int32, device=dev)

    comm = xchg = None
    if world > 1:
        # the library's own NCCL communicator (w4a8_lmhead_argmax_allreduce), and the
        # peer-memory exchange buffers (w4a8_lmhead_argmax_xchg)
        store = dist.distributed_c10d._get_default_store()
        if rank == 0:
            store.set("w4a8_nccl_uid", ops.nccl_unique_id())
        comm = ops.NcclComm(world, store.get("w4a8_nccl_uid"), rank)
        xchg = ops.PeerExchange()

    def c3():
        if xchg is None:
            ops.lmhead_argmax(w, xq, xs, act=ops.ACT_TOKEN, row_offset=0, workspace=wsp, best_key=key, tok=tok)
        else:
            ops.lmhead_argmax_xchg(w, xq, xs, xchg, act=ops.ACT_TOKEN, row_offset=rank * per_rank,
                                   workspace=wsp, best_key=key, tok=tok)

    def c3_nccl():
        ops.lmhead_argmax_allreduce(w, xq, xs, comm, act=ops.ACT_TOKEN, row_offset=rank * per_rank,
                                    workspace=wsp, best_key=key, tok=tok)

    # every rank replays its own graph (C3_CALLS tokens' lm_head calls, chained by
    # programmatic dependent launch as in a captured decode loop); the exchange
    # kernel meets the other ranks once per call
    ms, g = time_graph(torch, lambda: [c3() for _ in range(C3_CALLS)], steps, warmup, sync_all)
    del g
    # a peer that missed an exchange leaves only the device error word set: raise
    ops.device_error()
    ms = max_ms(ms) / C3_CALLS
    ms_nccl = None
    if comm is not None:
        # NCCL collectives stay eager (no graph capture across ranks here)
        for _ in range(warmup):
            c3_nccl()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            c3_nccl()
        e1.record()
        torch.cuda.synchronize()
        ms_nccl = max_ms(e0.elapsed_time(e1) / steps)
    c3_parity = None
    if world > 1:
        c3_parity = c3_sharded_parity(torch, ops, dist, w, xq, xs, wsp, key, tok, rank, world, per_rank, c3,
                                      c3_nccl)
    lm_bytes = gemv_bytes(k, vocab)
    out["c3_lmhead_argmax"] = {"gpus": world, "c3_parity": c3_parity, "us_per_token": round(ms * 1e3, 2), "tok_s": round(1e3 / ms, 1),
                               "gbs_total": round(lm_bytes / (ms * 1e-3) / 1e9, 1),
                               "frac_hbm_per_gpu": round(lm_bytes / world / (ms * 1e-3) / 1e9 / hbm, 3),
                               "collective": "w4a8_lmhead_argmax_xchg: packed keys tagged with the call, stored "
                                             "into every peer's buffer over NVLink by the lm_head kernel's last CTA"
                                             if world > 1 else None,
                               "us_per_token_nccl_allreduce": round(ms_nccl * 1e3, 2) if ms_nccl else None,
                               "timing": f"CUDA graph of {C3_CALLS} calls (one token each), PDL between them"}
    if xchg is not None:
        dist.barrier()  # no rank frees its buffer while a peer may still store into it
        xchg.close()
    if comm is not None:
        comm.close()
    del w
    # config 4: prefill GEMM, M = 1024 (rotating over 4 weight copies), against the
    # int8 tensor-core peak measured here with cuBLAS (torch._int_mm)
    int8_peak = measure_int8_peak(torch, dev)
    c4 = {}
    for k, n in ((2048, 6144), (6144, 2048)):
        ws = [rand_weight(n, k, GROUP, gen, dev, torch, ops) for _ in range(4)]
        xq, xs = ops.quant(torch.randn((1024, k), device=dev, generator=gen), act=ops.ACT_TOKEN)
        y = torch.empty((1024, n), device=dev)

        def c4f():
            for w in ws:
                ops.gemm(w, xq, xs, act=ops.ACT_TOKEN, y=y)

        ms, g = time_graph(torch, c4f, max(steps // 4, 3), min(warmup, 3))
        del g
        per = ms / len(ws)
        tops = 2 * 1024 * k * n / (per * 1e-3) / 1e12
        c4[f"{k}x{n}"] = {"us": round(per * 1e3, 2), "tops": round(tops, 1),
                          "frac_int8_peak": round(tops / int8_peak, 3) if int8_peak else None}
        del ws
    c4["kernel"] = "gemm_tc_kernel: tcgen05.mma.cta_group::2.kind::i8, TMEM accumulators"
    c4["int8_peak_tops"] = round(int8_peak, 1) if int8_peak else None
    c4["int8_peak_kind"] = "measured here: cuBLAS int8 GEMM (torch._int_mm) 8192^3, best of 5"
    out["c4_prefill_gemm"] = c4
    return out


def c3_sharded_parity(torch, ops, dist, w, xq, xs, wsp, key, tok, rank, world, per_rank, c3, c3_nccl):
    """The sharded lm_head's result on every rank against the max of the per-shard
    keys: each rank's own shard key (plain fused argmax, no exchange) is gathered
    over torch.distributed and the max taken on the host; the peer-memory exchange
    (c3) and the NCCL all-reduce variant (c3_nccl) must both return that key and its
    token on every rank.  Returns True only if they do on all ranks."""
    own, _ = ops.lmhead_argmax(w, xq, xs, act=ops.ACT_TOKEN, row_offset=rank * per_rank, workspace=wsp)
    gathered = [torch.empty_like(own) for _ in range(world)]
    dist.all_gather(gathered, own)
    mask = (1 << 64) - 1
    ref_key = max(int(g.item()) & mask for g in gathered)
    ref_tok = (~ref_key) & 0xFFFFFFFF if ref_key else 0
    ok = True
    for fn in (c3, c3_nccl):
        key.zero_()
        tok.fill_(-1)
        fn()
        torch.cuda.synchronize()
        ops.device_error()
        ok = ok and (int(key.item()) & mask) == ref_key and int(tok.item()) == ref_tok
    flag = torch.tensor([1 if ok else 0], device=key.device)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    return bool(flag.item())


# ---------------------------------------------------------------------------
def reference_arm(args, rank, world):
    """The reference's CPU path (tools/reference.py fake-quant linear, fp32 torch)
    on the decode sweep; rank 0 only."""
    if rank != 0:
        return None
    import torch

    from oracle import fakequant

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    g = torch.Generator().manual_seed(0)
    # one layer's 6 projections, weights dequantized once (outside the timed loop)
    layer = []
    for k, n in SWEEP:
        codes = torch.randint(-8, 8, (n, k), generator=g, dtype=torch.int8).float()
        sc = (torch.randn((n, k // GROUP), generator=g).abs() * 0.01).half().float()
        layer.append((k, n, codes * sc.repeat_interleave(GROUP, dim=1)))
    xs = {k: torch.randn((1, k), generator=g) for k in {k for k, _ in SWEEP}}

    def one_layer():
        for k, n, wd in layer:
            fakequant.fake_quant_linear(xs[k], wd, per_token=True)

    for _ in range(max(args.warmup, 3)):
        one_layer()
    # each step = a bounded sample of the sweep: all 6 shapes of one layer, R times
    t0 = time.perf_counter()
    one_layer()
    per_layer = time.perf_counter() - t0
    reps = max(1, int(min(2.0, 20.0 / max(args.steps, 1)) / max(per_layer, 1e-6)))
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        for _ in range(reps):
            one_layer()
        times.append((time.perf_counter() - t0) / reps)
    per = statistics.median(times)
    layer_bytes = sum(gemv_bytes(k, n) for k, n in SWEEP)
    gbs = layer_bytes / per / 1e9
    return {
        "metric": "W4A8 GEMV HBM GB/s (decode projection sweep, M=1)", "value": round(gbs, 3), "unit": "GB/s",
        "impl": "reference", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(per * LAYERS * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "decode_sweep_c2", "shapes_kn": SWEEP, "layers": LAYERS, "group": GROUP,
                   "m": 1, "act": "per-token int8"},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": f"one layer (6 projections) x {reps} per step, median of {args.steps} steps; "
                                   "tools/reference.py fake-quant F.linear fp32, weights dequantized once"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "extra": {"c3_lmhead_argmax": cpu_lmhead_argmax(torch, fakequant, cores)},
    }


C3_K, C3_VOCAB = 2048, 248320  # config 3: the lm_head of the 248,320-token vocabulary


def cpu_lmhead_argmax(torch, fakequant, cores, tokens=3):
    """Config 3 on the host cores through the reference's CPU path: activation
    fake-quant, fp32 F.linear against the dequantized vocabulary (dequantized once,
    in row blocks, outside the timed region), then argmax (lowest index among
    equal maxima, as the reference's argmax).  Per-token latency, median of
    `tokens` tokens after one warm-up."""
    g = torch.Generator().manual_seed(3)
    k, vocab = C3_K, C3_VOCAB
    wd = torch.empty((vocab, k))
    for r0 in range(0, vocab, 16384):
        r1 = min(vocab, r0 + 16384)
        codes = torch.randint(-8, 8, (r1 - r0, k), generator=g, dtype=torch.int8).float()
        sc = (torch.randn((r1 - r0, k // GROUP), generator=g).abs() * 0.01).half().float()
        wd[r0:r1] = codes * sc.repeat_interleave(GROUP, dim=1)
    x = torch.randn((1, k), generator=g)

    def one():
        return int(torch.argmax(fakequant.fake_quant_linear(x, wd, per_token=True)))

    one()
    times = []
    for _ in range(tokens):
        t0 = time.perf_counter()
        one()
        times.append(time.perf_counter() - t0)
    per = statistics.median(times)
    del wd
    return {"us_per_token": round(per * 1e6, 1), "tok_s": round(1.0 / per, 2),
            "gbs_total": round(gemv_bytes(k, vocab) / per / 1e9, 3), "cores": cores,
            "sample": f"{tokens} tokens after one warm-up, median; fp32 weights dequantized once"}


def cpu_baseline_sample(seconds=10.0):
    """The same reference CPU path as the reference arm, bounded to ~`seconds`."""
    import torch

    from oracle import fakequant

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    g = torch.Generator().manual_seed(0)
    layer = []
    for k, n in SWEEP:
        codes = torch.randint(-8, 8, (n, k), generator=g, dtype=torch.int8).float()
        sc = (torch.randn((n, k // GROUP), generator=g).abs() * 0.01).half().float()
        layer.append((k, n, codes * sc.repeat_interleave(GROUP, dim=1)))
    xs = {k: torch.randn((1, k), generator=g) for k in {k for k, _ in SWEEP}}
    for _ in range(3):
        for k, n, wd in layer:
            fakequant.fake_quant_linear(xs[k], wd, per_token=True)
    t0 = time.perf_counter()
    reps = 0
    while time.perf_counter() - t0 < seconds:
        for k, n, wd in layer:
            fakequant.fake_quant_linear(xs[k], wd, per_token=True)
        reps += 1
    per = (time.perf_counter() - t0) / reps
    gbs = sum(gemv_bytes(k, n) for k, n in SWEEP) / per / 1e9
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"{reps} x one sweep layer (6 projections) in {seconds:.0f}s; tools/reference.py "
                      "fake-quant F.linear fp32 on the host cores, weights dequantized once"}


# ---------------------------------------------------------------------------
def run_case(case, iters, torch, ops, dev):
    """A small, fixed workload for profiling one kernel (4 rotating weight copies)."""
    kind, *dims = case.split(":")
    gen = torch.Generator(device=dev)
    gen.manual_seed(0)
    k, n = int(dims[0]), int(dims[1])
    m = int(dims[2]) if len(dims) > 2 else 1
    ws = [rand_weight(n, k, GROUP, gen, dev, torch, ops) for _ in range(4)]
    xq, xs = ops.quant(torch.randn((m, k), device=dev, generator=gen), act=ops.ACT_TOKEN)
    if kind == "gemv":
        y = torch.empty((m, n), device=dev)
        for i in range(iters):
            ops.gemv(ws[i % 4], xq, xs, act=ops.ACT_TOKEN, y=y)
    elif kind == "lmhead":
        wsp = ops.lmhead_workspace(ws[0], m, dev)
        for i in range(iters):
            ops.lmhead_argmax(ws[i % 4], xq, xs, act=ops.ACT_TOKEN, workspace=wsp)
    elif kind == "gemm":
        y = torch.empty((m, n), device=dev)
        for i in range(iters):
            ops.gemm(ws[i % 4], xq, xs, act=ops.ACT_TOKEN, y=y)
    else:
        raise SystemExit(f"unknown case {case}")
    torch.cuda.synchronize()
    ops.device_error()
    print(f"case {case}: {iters} calls ok")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-extras", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--case", default=None,
                    help="profiling case instead of the benchmark: 'gemv:K:N[:M]' or 'lmhead:K:N' runs that "
                         "call `--steps` times on rotating weights (small, for ncu)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))

    if args.impl == "reference":
        line = reference_arm(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return

    import torch

    from webyiq_b200 import _lib, ops

    _lib.load()
    if local >= torch.cuda.device_count():
        # one GPU per rank: the sharded lm_head's exchange kernels wait on each other,
        # which ranks sharing a GPU must never do
        raise SystemExit(f"rank {rank}: local rank {local} but only {torch.cuda.device_count()} GPU(s) visible")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if args.case:
        run_case(args.case, args.steps, torch, ops, dev)
        return
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    def sync_all():
        if dist is not None:
            dist.barrier()

    sweep = Sweep(torch, ops, dev, seed=1000 + rank)
    hbm, _, peak_kind = peaks()

    # value: device-resident inputs, CUDA graph of the 144 GEMVs
    gpu_idx = os.environ.get("CUDA_VISIBLE_DEVICES", str(local)).split(",")[local] if world > 1 else \
        os.environ.get("CUDA_VISIBLE_DEVICES", "0").split(",")[0]
    with Clocks(gpu_idx) as clk:
        ms, graph = time_graph(torch, sweep.step, args.steps, args.warmup, sync_all)
    if dist is not None:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    del graph
    sb = step_bytes()
    value = world * sb / (ms * 1e-3) / 1e9
    achieved = sb / (ms * 1e-3) / 1e9  # per GPU = per-launch bytes / average launch time

    # e2e: host buffers, copies inside the timed region
    try:
        ms_e2e, g2 = time_graph(torch, sweep.step_e2e, args.steps, args.warmup, sync_all)
        del g2
        e2e_mode = ("cuda graph: H2D copies of all inputs + fused quant/GEMV (w4a8_gemv_x) + D2H copies of all "
                    "outputs, the copies of layers 2-23 (up) and 0-21 (down) overlapping the chain on a side stream")
    except Exception as exc:  # capture of the host copies unsupported: time eagerly
        e2e_mode = f"eager ({type(exc).__name__})"
        for _ in range(args.warmup):
            sweep.step_e2e()
        torch.cuda.synchronize()
        sync_all()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            sweep.step_e2e()
        e1.record()
        torch.cuda.synchronize()
        ms_e2e = e0.elapsed_time(e1) / args.steps
    torch.cuda.synchronize()
    if not (torch.equal(sweep.d_in.cpu(), sweep.h_in) and torch.equal(sweep.d_out.cpu(), sweep.h_out)):
        raise RuntimeError("e2e: the host and device copies of the step's inputs or outputs differ")
    if dist is not None:
        t = torch.tensor([ms_e2e], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_e2e = float(t.item())
    e2e = world * sb / (ms_e2e * 1e-3) / 1e9

    extras = None if args.no_extras else run_extras(torch, ops, dev, args.steps, args.warmup, world, rank, dist)

    cpu = None
    if rank == 0 and world == 1:
        cpu = cpu_baseline_sample(args.cpu_seconds)

    # DRAM bytes per launch of the sweep's GEMV, from the committed ncu capture of
    # the same workload (bytes per step / launches per step).
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tpath):
        try:
            per_step = json.load(open(tpath)).get("gemv_decode_sweep_bytes_per_step")
            traffic = round(per_step / Sweep.launches_per_step) if per_step else None
        except Exception:
            traffic = None

    if rank == 0:
        line = {
            "metric": "W4A8 GEMV HBM GB/s (decode projection sweep, M=1)",
            "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8xint4->int32/int64", "data": "synthetic",
            "config": {"workload": "decode_sweep_c2", "shapes_kn": SWEEP, "layers": LAYERS, "group": GROUP,
                       "m": 1, "act": "per-token int8", "weights_bytes_per_step": sb,
                       "l2": "inputs larger than L2 (586 MB per step vs 126 MB)",
                       "parallelism": f"replicas x{world}", "launch": "cuda graph, PDL between GEMVs"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(achieved / hbm, 4), "peak_kind": peak_kind, "traffic": traffic,
                         "kernel": "gemv_dec_kernel (decode GEMV, group-128 per-token)",
                         "algorithmic_bytes_per_launch": round(sb / Sweep.launches_per_step),
                         "launch_us": round(ms * 1e3 / Sweep.launches_per_step, 3)},
            "e2e": {"value": round(e2e, 1), "unit": "GB/s", "ms_per_step": round(ms_e2e, 4),
                    "h2d_bytes_per_step": sweep.nin * 4, "d2h_bytes_per_step": sweep.nout * 4, "mode": e2e_mode},
            "gpu_launches": args.steps * Sweep.launches_per_step,
            "clocks": clk.summary(),
            "cpu_baseline": cpu,
            "extra": extras,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    c3p = (extras or {}).get("c3_lmhead_argmax", {}).get("c3_parity")
    if c3p is False:
        raise SystemExit("c3_parity: the sharded lm_head's key differs from the max of the shard keys")


if __name__ == "__main__":
    main()
