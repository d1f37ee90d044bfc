#!/usr/bin/env python
"""EXL3 packed-weight GEMV benchmark on B200.

One step = one batch-1 decode pass over the linear layers of the synthetic
2B-class hybrid decoder: 28 layers x {q 2048x2048, k 2048x512, v 2048x512,
o 2048x2048, gate 2048x6144, up 2048x6144, down 6144x2048} at 4 bpw (196 EXL3
mul_mats, distinct weights per layer: 680 MB of packed trellis per step, far
above the 126 MB L2, so every step streams its weights from HBM).  Weights are
seeded synthetic (uniform random trellis words, +-1 input signs,
+-U(0.01,0.03) output scales), activations fp16 N(0,1).

Launch patterns (every one computes the same 196 products):
  decoder   per layer: {q,k,v} | {o} | {gate,up} | {down} -- the launches a
            decoder layer can issue, since o and down wait for attention and the
            activation function; 112 grouped launches per step (the headline)
  matrix    one exl3cu_mul_mat launch per matrix, 196 per step
  layer     one grouped launch per layer (7 problems), 28 per step
Each pattern's step is captured once in a CUDA graph and replayed; launches
chain with programmatic dependent launch.

  value   algorithmic bytes of K steps / device time of K replays (decoder)
  e2e     the same metric from host memory: per step every matrix's fp16 x
          copied from pinned host memory and every f32 y copied back, pipelined
          by layer on two copy streams around the decoder pattern's C-ABI calls,
          all inside the timed region
  --impl reference   the reference's own CPU operator (ggml_exl3_mul_mat from
          oracle/_ref, built from the reference's sources) on all host cores

Multi-GPU (torchrun, one rank per GPU): every rank runs its own replica of the
sweep -- batch-1 decode has no exchange step -- so scaling is weak and the
time is the max over ranks.
"""
from __future__ import annotations

import argparse
import csv
import io
import json
import os
import statistics
import subprocess
import sys
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "xiaomi-hexagon-exl3_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "EXL3 4bpw GEMV HBM GB/s; 2B decode tok/s at 1 and 8 ragged reqs, 1-8 GPU"
LAYERS = 28
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
DECODER_GROUPS = (("q", "k", "v"), ("o",), ("gate", "up"), ("down",))


def parse_args(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--bits", type=int, default=4)
    ap.add_argument("--layers", type=int, default=LAYERS)
    ap.add_argument("--no-sweep", action="store_true", help="skip the 2/3/5/6-bit side measurements")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--e2e-steps", type=int, default=30)
    ap.add_argument("--config", choices=("sweep", "large", "ragged", "model"), default="sweep",
                    help="sweep: configs[1] decode GEMV sweep (default); large: configs[4] column-split matrix; "
                         "ragged: configs[2] packed continuous-admission batches on the tensor-core GEMM")
    ap.add_argument("--no-ragged", action="store_true", help="skip the configs[2] summary in the default run")
    ap.add_argument("--no-model", action="store_true", help="skip the configs[3] hybrid decoder summary")
    ap.add_argument("--no-large", action="store_true",
                    help="skip the configs[4] column-split summary (14336x4096, batch 1/8/512)")
    return ap.parse_args(argv)


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return PEAKS_FALLBACK, "fallback"


def shapes():
    from exl3_b200.synthetic import LAYER_SHAPES

    return list(LAYER_SHAPES.items())


def algo_bytes(bits, rows=1):
    from exl3_b200.synthetic import algorithmic_bytes

    return sum(algorithmic_bytes(k, n, bits, rows) for _, (k, n) in shapes())


class ClockSampler:
    """nvidia-smi clocks and throttle reasons, sampled every 50 ms around the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.text = ""

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
        time.sleep(0.15)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.1)
            self.proc.terminate()
            try:
                self.text, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.text, _ = self.proc.communicate()
        return False

    def summary(self):
        rows = [r for r in csv.reader(io.StringIO(self.text)) if len(r) >= 9]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "samples": 0}

        def num(v):
            try:
                return float(v)
            except ValueError:
                return None

        sm = [x for x in (num(r[1]) for r in rows) if x is not None]
        mx = [x for x in (num(r[2]) for r in rows) if x is not None]
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip().lower() == "active"})
        loaded = sorted(sm)[len(sm) // 2:] if sm else []
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------------------------
# workload

class Stack(list):
    """Layers of {name: matrix} dicts; every matrix's x [1, k] and y [1, n] are views into the packed
    device buffers x_all (fp16) and y_all (fp32), so a step's inputs and outputs move in one copy each."""

    x_all = None
    y_all = None


def build_stack(torch, ops, bits, layers, device, seed, keep_host_layer0=False):
    """Seeded synthetic weights generated on the device, uploaded through the C ABI."""
    dev = f"cuda:{device}"
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    stack = Stack()
    kx = sum(k for _, (k, _) in shapes()) * layers
    ny = sum(n for _, (_, n) in shapes()) * layers
    stack.x_all = torch.randn((kx,), generator=g, device=dev).to(torch.float16)
    stack.y_all = torch.empty((ny,), dtype=torch.float32, device=dev)
    ox = oy = 0
    for layer in range(layers):
        mats = {}
        for name, (k, n) in shapes():
            trellis = torch.randint(0, 65536, (k // 16, n // 16, 16 * bits), generator=g, device=dev,
                                    dtype=torch.int32).to(torch.int16)
            suh = (torch.randint(0, 2, (k,), generator=g, device=dev) * 2 - 1).to(torch.float16)
            sign = (torch.randint(0, 2, (n,), generator=g, device=dev) * 2 - 1).float()
            svh = (sign * (0.01 + 0.02 * torch.rand(n, generator=g, device=dev))).to(torch.float16)
            w = ops.Exl3Weight.from_trellis(trellis, suh.view(torch.int16), svh.view(torch.int16), device=device)
            x = stack.x_all[ox:ox + k].view(1, k)
            y = stack.y_all[oy:oy + n].view(1, n)
            ox += k
            oy += n
            host = None
            if keep_host_layer0 and layer == 0:
                host = (trellis.cpu().numpy().view("uint16"), suh.cpu().numpy().view("uint16"),
                        svh.cpu().numpy().view("uint16"))
            mats[name] = {"k": k, "n": n, "w": w, "x": x, "y": y, "host": host}
            del trellis
        stack.append(mats)
    torch.cuda.synchronize(device)
    return stack


def step_launcher(ops, stack, pattern, stream):
    """A callable issuing one step of `pattern` on `stream` (and its launch count)."""
    if pattern == "matrix":
        calls = [(m["w"], m["x"], m["y"]) for mats in stack for m in mats.values()]

        def run():
            for w, x, y in calls:
                w.mul_mat(x, out=y, stream=stream)
        return run, len(calls)
    if pattern == "layer":
        groups = [list(mats.values()) for mats in stack]
    else:
        groups = [[mats[name] for name in grp] for mats in stack for grp in DECODER_GROUPS]
    packed = [([m["w"] for m in grp], [m["x"] for m in grp], [m["y"] for m in grp]) for grp in groups]

    def run():
        for ws, xs, ys in packed:
            ops.mul_mat_batch(ws, xs, ys, stream=stream)
    return run, len(packed)


def time_pattern(torch, dist, ops, stack, pattern, steps, warmup, world):
    stream = torch.cuda.Stream()
    run, launches = step_launcher(ops, stack, pattern, stream)
    with torch.cuda.stream(stream):
        for _ in range(3):
            run()
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream, capture_error_mode="relaxed"):
        run()
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            graph.replay()
    stream.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(steps):
            graph.replay()
        end.record(stream)
    end.synchronize()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = start.elapsed_time(end)
    del graph
    return ms, launches


def time_e2e(torch, ops, stack, steps):
    """End to end from host memory, per step: every matrix's fp16 x copied from pinned host memory, the
    decoder pattern's 112 C-ABI launches, every f32 y copied back into pinned memory, and a stream
    synchronisation.  The copies are pipelined by layer: a copy stream moves layer l's x while earlier
    layers compute, layer l's launches wait only for their own x, and a second copy stream returns
    layer l's y while later layers compute.  The whole step (copies, launches, the streams' events)
    is one CUDA graph, replayed.  Returns (ms for `steps` steps, H2D bytes and D2H bytes per step)."""
    stream, cin, cout = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
    x_host = stack.x_all.cpu().pin_memory()
    y_host = torch.empty(stack.y_all.shape, dtype=torch.float32).pin_memory()
    layers = []
    for mats in stack:  # each layer's x and y are contiguous ranges of x_all / y_all
        xs = [m["x"] for m in mats.values()]
        ys = [m["y"] for m in mats.values()]
        x0 = min(x.storage_offset() for x in xs)
        x1 = max(x.storage_offset() + x.numel() for x in xs)
        y0 = min(y.storage_offset() for y in ys)
        y1 = max(y.storage_offset() + y.numel() for y in ys)
        groups = [[mats[name] for name in grp] for grp in DECODER_GROUPS]
        packed = [([m["w"] for m in g], [m["x"] for m in g], [m["y"] for m in g]) for g in groups]
        layers.append((x0, x1, y0, y1, packed))
    ev_in = [torch.cuda.Event() for _ in layers]
    ev_out = [torch.cuda.Event() for _ in layers]

    def body():
        cin.wait_stream(stream)
        cout.wait_stream(stream)
        with torch.cuda.stream(cin):
            for li, (x0, x1, _, _, _) in enumerate(layers):
                stack.x_all[x0:x1].copy_(x_host[x0:x1], non_blocking=True)
                ev_in[li].record(cin)
        with torch.cuda.stream(stream):
            for li, (_, _, _, _, packed) in enumerate(layers):
                stream.wait_event(ev_in[li])
                for ws, xs, ys in packed:
                    ops.mul_mat_batch(ws, xs, ys, stream=stream)
                ev_out[li].record(stream)
        with torch.cuda.stream(cout):
            for li, (_, _, y0, y1, _) in enumerate(layers):
                cout.wait_event(ev_out[li])
                y_host[y0:y1].copy_(stack.y_all[y0:y1], non_blocking=True)
        stream.wait_stream(cin)
        stream.wait_stream(cout)

    with torch.cuda.stream(stream):
        for _ in range(3):
            body()
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream, capture_error_mode="relaxed"):
        body()

    def step():
        with torch.cuda.stream(stream):
            graph.replay()
        stream.synchronize()

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    start.record(stream)
    for _ in range(steps):
        step()
    end.record(stream)
    end.synchronize()
    wall_ms = (time.perf_counter() - t0) * 1e3
    del graph
    h2d = stack.x_all.numel() * stack.x_all.element_size()
    d2h = stack.y_all.numel() * stack.y_all.element_size()
    return max(start.elapsed_time(end), wall_ms), h2d, d2h


def time_ggml_e2e(bits, layers, steps, seed=4242):
    """The reference-facing plugin call, per matrix, from host memory: ggml_exl3_mul_mat (the
    libexl3cu_ggml.so drop-in) called as ggml's CPU backend calls the reference's operator -- one
    GGML_OP_MUL_MAT node per matrix, ggml tensors over host buffers (packed records, f32 x [1, k],
    f32 y [1, n]), every call copying its x in and its y out and returning when y is in host memory.
    The records (seeded, same shapes and distribution as the device stack) are uploaded once, on the
    first step, by the adapter's weight cache; timed: `steps` steps of 7 * layers calls, host wall
    clock (each call is synchronous).  Returns (ms per step, h2d and d2h bytes per step, calls per step)."""
    import ctypes

    import numpy as np

    from exl3_b200 import _lib
    from exl3_b200.format import BITS_GGML_TYPE, pack_records

    class T(ctypes.Structure):
        _fields_ = [("type", ctypes.c_int), ("ne", ctypes.c_int64 * 4), ("nb", ctypes.c_size_t * 4),
                    ("src", ctypes.c_void_p * 10), ("data", ctypes.c_void_p)]

    class P(ctypes.Structure):
        _fields_ = [("ith", ctypes.c_int), ("nth", ctypes.c_int), ("wsize", ctypes.c_size_t),
                    ("wdata", ctypes.c_void_p)]

    def tensor(typ, ne, nb, data):
        t = T()
        t.type = typ
        for i in range(4):
            t.ne[i], t.nb[i] = ne[i], nb[i]
        t.data = data
        return t

    gl = ctypes.CDLL(str(_lib.GGML_LIB_PATH))
    fn = gl.ggml_exl3_mul_mat
    fn.argtypes = [ctypes.POINTER(P), ctypes.POINTER(T)]
    fn.restype = None
    rng = np.random.Generator(np.random.PCG64(seed))
    keep, nodes = [], []
    h2d = d2h = 0
    for _ in range(layers):
        for _, (k, n) in shapes():
            tr = rng.integers(0, 65536, size=(k // 16, n // 16, 16 * bits), dtype=np.uint16)
            suh = rng.choice(np.array([-1.0, 1.0], np.float16), size=k).view(np.uint16)
            svh = (rng.choice(np.array([-1.0, 1.0]), size=n) * rng.uniform(0.01, 0.03, size=n)).astype(
                np.float16).view(np.uint16)
            rec = pack_records(tr, suh, svh, bits)
            x = rng.standard_normal((1, k), dtype=np.float32)
            y = np.zeros((1, n), np.float32)
            w = tensor(BITS_GGML_TYPE[bits], (k, n, 1, 1), (1, 1, 1, 1), rec.ctypes.data)
            xi = tensor(0, (k, 1, 1, 1), (4, 4 * k, 4 * k, 4 * k), x.ctypes.data)
            dst = tensor(0, (n, 1, 1, 1), (4, 4 * n, 4 * n, 4 * n), y.ctypes.data)
            dst.src[0], dst.src[1] = ctypes.addressof(w), ctypes.addressof(xi)
            keep.append((rec, x, y, w, xi, dst))
            nodes.append(ctypes.byref(dst))
            h2d += x.nbytes
            d2h += y.nbytes
    params = ctypes.byref(P(0, 1, 0, None))
    for _ in range(2):  # the first step uploads every matrix into the adapter's cache
        for d in nodes:
            fn(params, d)
    t0 = time.perf_counter()
    for _ in range(steps):
        for d in nodes:
            fn(params, d)
    ms = (time.perf_counter() - t0) * 1e3 / steps
    gl.ggml_exl3_release_weights()
    del keep
    return ms, h2d, d2h, len(nodes)


def per_shape_us(torch, stack, reps=4):
    """Average device time of one exl3cu_mul_mat per shape, back to back over distinct layers."""
    out = {}
    stream = torch.cuda.Stream()
    for name, _ in shapes():
        ms = [layer[name] for layer in stack]
        with torch.cuda.stream(stream):
            for m in ms:
                m["w"].mul_mat(m["x"], out=m["y"], stream=stream)
            s, t = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            for _ in range(reps):
                for m in ms:
                    m["w"].mul_mat(m["x"], out=m["y"], stream=stream)
            t.record(stream)
        t.synchronize()
        out[name] = round(s.elapsed_time(t) * 1e3 / (reps * len(ms)), 2)
    return out


# ---------------------------------------------------------------------------------------------
# the synthetic 2B hybrid decoder (exl3_b200.hybrid)

def run_model_measure(torch, dist, local, rank, world, new_tokens=256, single_prompt=512, seed=2024):
    import numpy as np

    """Decode tokens/s of the 28-layer hybrid decoder on this GPU (DP replica per rank).

    single: one request, 512-token prompt prefilled, then `new_tokens` greedy steps replayed from one
            captured step with device-side token feedback (CUDA events around the replays);
    single_e2e: the same request served step by step through the engine API: per token the host fills
            the step metadata, one captured graph copies it in, runs the step and copies the token
            out (pinned buffers), and the host synchronises; events around the loop;
    ragged8: 8 requests, prompts U[32,1024] seeded, `new_tokens` greedy tokens each, continuous
            admission (decode rows of running requests + 512-row prefill chunks of the next one per
            step), host scheduler in the loop; runs of pure decode steps with nothing to admit go
            to the device as multi-step blocks; tokens/s = generated tokens / elapsed of the median of
            three identical runs."""
    from exl3_b200.hybrid import DecodeGraph, HybridConfig, HybridEngine, Request, run_requests, _StepGraph

    dev = f"cuda:{local}"
    cfg = HybridConfig()
    w = synthetic_weights_cached(cfg, seed + rank)
    eng = HybridEngine(w, device=local, slots=8, max_len=1536, max_rows=512)
    del w
    rng = np.random.Generator(np.random.PCG64(seed + 17 * rank))
    stream = torch.cuda.Stream(device=dev)
    # -- single request ---------------------------------------------------------------------------
    prompt = rng.integers(0, cfg.vocab, single_prompt).astype(np.int32)
    eng.reset_slot(0)
    n = len(prompt)
    eng.meta.fill(prompt, np.zeros(n), np.arange(n), [0, n], [0], [n - 1])
    with torch.cuda.stream(stream):
        eng.meta.upload(stream)
        eng.forward(n, 1, 1, stream)
    stream.synchronize()
    tok = int(eng.out_tokens[0].item())
    eng.meta.fill([tok], [0], [n], [0, 1], [0], [0])
    with torch.cuda.stream(stream):
        eng.meta.upload(stream)
    stream.synchronize()
    dg = DecodeGraph(eng, 1, new_tokens + 8, stream)  # its eager warm-up and capture advance nothing
    for _ in range(3):
        dg.replay()
    stream.synchronize()
    dg.reset()
    s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s_ev.record(stream)
    with torch.cuda.stream(stream):
        for _ in range(new_tokens):
            dg.replay()
    e_ev.record(stream)
    e_ev.synchronize()
    single_ms = s_ev.elapsed_time(e_ev)
    # -- single request, host in the loop ---------------------------------------------------------
    eng.reset_slot(1)
    eng.meta.fill(prompt, np.zeros(n), np.arange(n), [0, n], [1], [n - 1])
    with torch.cuda.stream(stream):
        eng.meta.upload(stream)
        eng.forward(n, 1, 1, stream)
    stream.synchronize()
    tok = int(eng.out_tokens[0].item())
    eng.meta.fill([tok], [0], [n], [0, 1], [1], [0])
    with torch.cuda.stream(stream):
        eng.meta.upload(stream)
        eng.forward(1, 1, 1, stream)  # eager step at this shape before capture
    stream.synchronize()
    sg = _StepGraph(eng, 1, stream)
    pos = n + 1
    tok = int(eng.out_tokens[0].item())
    e2e_steps = min(new_tokens, 128)
    s_ev.record(stream)
    for _ in range(e2e_steps):
        eng.meta.fill([tok], [0], [pos], [0, 1], [1], [0])
        with torch.cuda.stream(stream):
            sg.replay()  # the captured step copies the metadata in and the token out itself
        stream.synchronize()
        tok = int(sg.out_host[0])
        pos += 1
    e_ev.record(stream)
    e_ev.synchronize()
    e2e_ms = s_ev.elapsed_time(e_ev)
    del dg, sg
    # -- 8 ragged requests ------------------------------------------------------------------------
    lens = rng.integers(32, 1025, 8)
    prompts = [rng.integers(0, cfg.vocab, int(L)).astype(np.int32) for L in lens]
    graphs = {}
    # warm-up: first-time shapes and captures (eager steps, per-size step graphs, the 8-row multi-step
    # decode block), as a server does at start-up
    warm = [Request(rng.integers(0, cfg.vocab, 40).astype(np.int32), max_new=6) for _ in range(8)]
    run_requests(eng, warm, chunk=512, stream=stream, graphs=graphs)
    # three identical runs (the host scheduler is in the loop, so single runs spread by about +-10 %);
    # the median run is reported
    runs = []
    for _ in range(3):
        reqs = [Request(p.copy(), max_new=new_tokens) for p in prompts]
        torch.cuda.synchronize(dev)
        s_ev.record(stream)
        rstats = {}
        steps, rows = run_requests(eng, reqs, chunk=512, stream=stream, graphs=graphs, stats=rstats)
        e_ev.record(stream)
        e_ev.synchronize()
        runs.append((s_ev.elapsed_time(e_ev), steps, rows, rstats, sum(len(r.generated) for r in reqs)))
    runs_ms = [round(r[0], 1) for r in runs]
    ragged_ms, steps, rows, rstats, generated = sorted(runs, key=lambda r: r[0])[1]

    def over_ranks(v, op):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=op)
        return float(t.item())

    single_ms = over_ranks(single_ms, dist.ReduceOp.MAX) if world > 1 else single_ms
    e2e_ms = over_ranks(e2e_ms, dist.ReduceOp.MAX) if world > 1 else e2e_ms
    ragged_ms_max = over_ranks(ragged_ms, dist.ReduceOp.MAX) if world > 1 else ragged_ms
    gen_total = over_ranks(float(generated), dist.ReduceOp.SUM) if world > 1 else float(generated)
    from exl3_b200 import ops

    status = ops.device_status(local)
    eng.free()
    del eng
    torch.cuda.empty_cache()
    if status:
        raise RuntimeError(f"device status {status:#x} after the hybrid decoder run")
    return {
        "model": "synthetic 2B hybrid: 28 layers (21 gated delta rule + 7 GQA 16q/4kv), hidden 2048, FFN 6144, "
                 "vocab 151936 fp16 tied embed/head, EXL3 4 bpw linear layers (random trellis)",
        "single_tok_s": round(world * new_tokens / (single_ms * 1e-3), 1),
        "single_ms_per_token": round(single_ms / new_tokens, 4),
        "single_timing": "one captured decode step replayed with device-side token feedback; CUDA events",
        "single_e2e_tok_s": round(world * e2e_steps / (e2e_ms * 1e-3), 1),
        "single_e2e_api": "per token: one captured graph copies the step metadata in from pinned memory "
                          "(6.2 KB), runs the step and copies the token out; host synchronise",
        "ragged8_tok_s": round(gen_total / (ragged_ms_max * 1e-3), 1),
        "ragged8": {"requests_per_gpu": 8, "prompt_tokens": [int(x) for x in lens], "new_tokens": new_tokens,
                    "steps": steps, "rows": rows, "ms": round(ragged_ms_max, 1), "runs_ms": runs_ms,
                    "by_step_kind_host_ms": {k: (round(v, 1) if isinstance(v, float) else v) for k, v in rstats.items()},
                    "timing": "host scheduler loop with H2D metadata / D2H tokens per step; CUDA events; "
                              "median of 3 identical runs"},
        "parallelism": f"dp{world} replicas (weights replicated, requests per GPU)",
        "prompt_tokens_single": single_prompt,
    }


_WEIGHTS_CACHE = {}


def synthetic_weights_cached(cfg, seed):
    from exl3_b200.hybrid import synthetic_weights

    key = (seed, cfg.layers, cfg.vocab)
    if key not in _WEIGHTS_CACHE:
        _WEIGHTS_CACHE.clear()
        _WEIGHTS_CACHE[key] = synthetic_weights(cfg, seed)
    return _WEIGHTS_CACHE[key]


# ---------------------------------------------------------------------------------------------
# CPU legs (reference operator built from the reference's sources, or the oracle port)

def cpu_checker():
    from oracle.oracle import Oracle, Reference, have_reference, host_threads

    if have_reference():
        return Reference(), "reference", host_threads()
    return Oracle(), "port", host_threads()


def cpu_layer_pass(ref, recs, bits, nth):
    for k, n, rec, x in recs:
        ref.mul_mat(rec, bits, k, n, x, nth=nth)


def cpu_baseline(stack, bits, budget_s=8.0):
    from exl3_b200.format import pack_records

    recs = []
    for name, (k, n) in shapes():
        m = stack[0][name]
        tr, su, sv = m["host"]
        recs.append((k, n, pack_records(tr, su, sv, bits), m["x"].cpu().numpy()))
    ref, kind, nth = cpu_checker()
    cpu_layer_pass(ref, recs, bits, nth)  # warm-up: builds the codebook tables
    times = []
    t_all = time.perf_counter()
    while len(times) < 3 or (time.perf_counter() - t_all < budget_s and len(times) < 200):
        t0 = time.perf_counter()
        cpu_layer_pass(ref, recs, bits, nth)
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    who = "ggml_exl3_mul_mat (reference sources, oracle/_ref)" if kind == "reference" else "oracle port"
    return {"value": round(algo_bytes(bits) / med / 1e9, 4), "unit": "GB/s", "cores": nth, "kind": kind,
            "sample": f"one decoder layer (7 matrices, {bits} bpw, batch 1) of the same workload, {len(times)} "
                      f"timed passes, median; {who} with the ith/nth split over {nth} threads"}


def run_reference_arm(args, rank, world):
    if world > 1 and rank != 0:
        return
    from exl3_b200 import synthetic
    from exl3_b200.format import pack_records

    ref, kind, nth = cpu_checker()
    bits = args.bits
    n_layers = 4  # distinct layers rotated per step (94 MB of records, beyond the host caches)
    layers = []
    for layer in range(n_layers):
        recs = []
        for i, (_, (k, n)) in enumerate(shapes()):
            m = synthetic.matrix(k, n, bits, seed=10_000 * layer + i)
            recs.append((k, n, pack_records(m.trellis, m.suh, m.svh, bits),
                         synthetic.activations(1, k, seed=20_000 * layer + i)))
        layers.append(recs)
    for s in range(args.warmup):
        cpu_layer_pass(ref, layers[s % n_layers], bits, nth)
    t0 = time.perf_counter()
    for s in range(args.steps):
        cpu_layer_pass(ref, layers[s % n_layers], bits, nth)
    dt = time.perf_counter() - t0
    value = algo_bytes(bits) * args.steps / dt / 1e9
    who = "ggml_exl3_mul_mat (reference sources, oracle/_ref)" if kind == "reference" else "oracle port"
    line = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dt * 1e3 / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic", "impl": "reference",
        "config": {"workload": f"configs[1] per-layer GEMV sweep at {bits} bpw, batch 1; one step = one decoder "
                               f"layer (7 matrices) rotating over {n_layers} seeded layers",
                   "bits": bits, "rows": 1, "parallelism": "host threads"},
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": nth, "kind": kind,
                         "sample": f"{who}, ith/nth split over {nth} threads, one layer per step"},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------------

def large_tp_measure(torch, dist, ops, rank, world, local, bits=4, steps=50, warmup=5, rows_list=(1, 8, 512)):
    """W [k=14336, n=4096] at `bits` bpw, x [rows, 14336] fp16, column-split over the
    ranks (128-column blocks in contiguous ranges) with one NCCL all-gather of the fp32 slices.
    Per batch: the local EXL3 slice, the all-gather alone, the whole operator (slice + NCCL
    gather) and, on 2+ GPUs, the operator with the slices exchanged over NVLink peer memory;
    each timed as CUDA-graph replays of one pass over the rotated weight copies, CUDA events
    on the launching stream, max over ranks.  Batch 1 and 8 run the GEMV
    (HBM-bound: per-GPU GB/s of the slice); batch 512 runs the tcgen05 GEMM (per-GPU TFLOP/s)."""
    from exl3_b200.parallel import ColumnSplit, PeerColumnParallelExl3, gather_columns

    k, n = 14336, 4096
    split = ColumnSplit(n, world)
    first, count = split.range(rank)
    dev = f"cuda:{local}"
    g = torch.Generator(device=dev)
    g.manual_seed(4242)  # identical full matrix on every rank; each keeps its blocks
    trellis = torch.randint(0, 65536, (k // 16, n // 16, 16 * bits), generator=g, device=dev,
                            dtype=torch.int32).to(torch.int16)
    suh = (torch.randint(0, 2, (k,), generator=g, device=dev) * 2 - 1).to(torch.float16)
    svh = ((torch.randint(0, 2, (n,), generator=g, device=dev) * 2 - 1).float() *
           (0.01 + 0.02 * torch.rand(n, generator=g, device=dev))).to(torch.float16)
    # Copies of the rank's slice (same values) rotated through so that consecutive launches read
    # more than the 126 MB L2 holds: every timed launch streams its weights from HBM.
    slice_bytes = k * count * 128 * bits // 8
    ncopies = max(2, -(-300_000_000 // slice_bytes))
    copies = [ops.Exl3Weight.from_trellis(trellis, suh.view(torch.int16), svh.view(torch.int16), device=local,
                                          first_block=first, block_count=count) for _ in range(ncopies)]
    del trellis
    results = {}
    stream = torch.cuda.Stream()
    peer = None
    if world > 1:
        # the peer path runs on the same rotated copies of the slice (handed over per call)
        peer = PeerColumnParallelExl3(None, k, n, bits, max_rows=max(rows_list), device=local, weight=copies[0])

    def timed(fn):
        # one CUDA graph of one pass over the rotated copies, replayed: device time, no host gaps
        with torch.cuda.stream(stream):
            for i in range(max(warmup, 2)):
                fn(i)
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream, capture_error_mode="relaxed"):
            for i in range(ncopies):
                fn(i)
        reps = max(1, -(-steps // ncopies))
        with torch.cuda.stream(stream):
            for _ in range(2):
                graph.replay()
        stream.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            s.record(stream)
            for _ in range(reps):
                graph.replay()
            e.record(stream)
        e.synchronize()
        ms = s.elapsed_time(e) / (reps * ncopies)
        stream.synchronize()
        if world > 1:
            dist.barrier()
        del graph
        if world > 1:
            t = torch.tensor([ms], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    for rows in rows_list:
        x = torch.randn((rows, k), generator=g, device=dev).to(torch.float16)
        y_local = torch.empty((rows, count * 128), dtype=torch.float32, device=dev)
        local_bytes = k * count * 128 * bits // 8 + 2 * (k + count * 128) + 2 * k * rows + 4 * count * 128 * rows
        local_flops = 2.0 * rows * k * count * 128
        ms_local = timed(lambda i: copies[i % ncopies].mul_mat(x, out=y_local, stream=stream))
        ms_gather = timed(lambda i: gather_columns(y_local, split)) if world > 1 else 0.0

        def op(i):
            copies[i % ncopies].mul_mat(x, out=y_local, stream=stream)
            gather_columns(y_local, split)
        ms_op = timed(op)
        r = {"local_us": round(ms_local * 1e3, 2), "gather_us": round(ms_gather * 1e3, 2),
             "operator_us": round(ms_op * 1e3, 2),
             "gather_bytes_per_rank": 4 * rows * 128 * split.max_blocks * world}
        if peer is not None:
            # the same slices exchanged over NVLink peer memory instead of the NCCL all-gather
            def op_peer(i):
                peer.weight = copies[i % ncopies]
                peer.forward(x, stream=stream)
            r["operator_peer_us"] = round(timed(op_peer) * 1e3, 2)
        if rows <= 8:
            r["local_gbs_per_gpu"] = round(local_bytes / (ms_local * 1e-3) / 1e9, 1)
        else:
            r["local_tflops_per_gpu"] = round(local_flops / (ms_local * 1e-3) / 1e12, 1)
            r["operator_tflops_total"] = round(2.0 * rows * k * n / (ms_op * 1e-3) / 1e12, 1)
        results[str(rows)] = r
    if peer is not None:
        peer.free()
    for c in copies:
        c.free()
    return {"n_gpus": world, "blocks_per_rank": split.max_blocks, "copies": ncopies, "by_batch": results}


def run_large(args, torch, dist, ops, rank, world, local):
    """--config large: configs[4] alone (see large_tp_measure), one JSON line."""
    res = large_tp_measure(torch, dist, ops, rank, world, local, bits=args.bits, steps=args.steps,
                           warmup=max(3, args.warmup))
    if rank == 0:
        pk, pk_kind = peaks()
        peak = float(pk.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"]))
        b1 = res["by_batch"]["1"]
        print(json.dumps({
            "metric": "EXL3 4bpw large-matrix GEMV, column split + NCCL all-gather (configs[4])",
            "value": b1["local_gbs_per_gpu"], "unit": "GB/s per GPU", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "scaling": "strong", "dtype": "fp16",
            "data": "synthetic", "vs_baseline": None,
            "config": {"workload": "W [4096,14336] (k=14336, n=4096) 4 bpw, x fp16 N(0,1); batch 1, 8 and 512",
                       "parallelism": f"column split tp{world}", "bits": args.bits,
                       "l2": f"{res['copies']} copies of the rank's slice rotated: > 126 MB per rotation"},
            "roofline": {"bound": "hbm", "achieved": b1["local_gbs_per_gpu"], "peak": peak, "unit": "GB/s",
                         "frac": round(b1["local_gbs_per_gpu"] / peak, 4), "peak_source": f"{pk_kind} hbm_gbs"},
            "by_batch": res["by_batch"]}), flush=True)
    return 0


# ---------------------------------------------------------------------------------------------
# ragged continuous-admission batches through the mixed-bit layer stack

RAGGED_BUCKETS = (32, 64, 128, 256, 512)
RAGGED_MAX_ROWS = 512


def ragged_batches(count, seed=2024):
    """Seeded step compositions: 8..64 sequences, each a decode token, plus 0..3 prefill chunks of
    16..512 rows; decode tokens are admitted first, the packed batch is capped at 512 rows."""
    import numpy as np

    rng = np.random.Generator(np.random.PCG64(seed))
    out = []
    for _ in range(count):
        n_seq = int(rng.integers(8, 65))
        n_pre = int(rng.integers(0, 4))
        n_dec = max(n_seq - n_pre, 1)
        want = [1] * n_dec + [int(v) for v in rng.integers(16, 513, n_pre)]
        pos = [int(v) for v in rng.integers(32, 1025, len(want))]
        rows = min(sum(want), RAGGED_MAX_ROWS)
        out.append({"want": want, "pos": pos, "rows": rows,
                    "bucket": next(b for b in RAGGED_BUCKETS if b >= rows)})
    return out


def build_mixed_stack(torch, ops, layers, device, seed, frac6=0.25):
    """The 2B decoder's 196 matrices with a seeded 25% of them at 6 bpw, the rest at 4 bpw."""
    import numpy as np

    dev = f"cuda:{device}"
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    names = [name for name, _ in shapes()]
    total = layers * len(names)
    rng = np.random.Generator(np.random.PCG64(seed))
    six = set(int(i) for i in rng.choice(total, size=int(round(frac6 * total)), replace=False))
    stack, bits_bytes, weights = [], 0, 0
    for layer in range(layers):
        mats = {}
        for j, (name, (k, n)) in enumerate(shapes()):
            bits = 6 if layer * len(names) + j in six else 4
            trellis = torch.randint(0, 65536, (k // 16, n // 16, 16 * bits), generator=g, device=dev,
                                    dtype=torch.int32).to(torch.int16)
            suh = (torch.randint(0, 2, (k,), generator=g, device=dev) * 2 - 1).to(torch.float16)
            svh = ((torch.randint(0, 2, (n,), generator=g, device=dev) * 2 - 1).float() *
                   (0.01 + 0.02 * torch.rand(n, generator=g, device=dev))).to(torch.float16)
            w = ops.Exl3Weight.from_trellis(trellis, suh.view(torch.int16), svh.view(torch.int16), device=device)
            mats[name] = {"k": k, "n": n, "bits": bits, "w": w}
            bits_bytes += k * n * bits
            weights += k * n
            del trellis
        stack.append(mats)
    torch.cuda.synchronize(device)
    return stack, bits_bytes / weights


def run_ragged_measure(torch, ops, device, layers, reps, seed):
    """Per-bucket CUDA graphs of one step (GPU packer + 196 exl3cu_mul_mat_ragged calls, row count read
    on the device), replayed over seeded batch compositions; returns the summary dict."""
    dev = f"cuda:{device}"
    stack, avg_bpw = build_mixed_stack(torch, ops, layers, device, seed)
    gx = torch.Generator(device=dev)
    gx.manual_seed(seed + 1)
    xs = {k: torch.randn((RAGGED_MAX_ROWS, k), generator=gx, device=dev).to(torch.float16)
          for k in sorted({k for _, (k, _) in shapes()})}
    ys = {name: torch.empty((RAGGED_MAX_ROWS, n), dtype=torch.float32, device=dev) for name, (_, n) in shapes()}
    n_seq_max = 64
    want = torch.zeros(n_seq_max, dtype=torch.int32, device=dev)
    pos = torch.zeros(n_seq_max, dtype=torch.int32, device=dev)
    packed = (torch.empty(n_seq_max + 1, dtype=torch.int32, device=dev),
              torch.empty(RAGGED_MAX_ROWS, dtype=torch.int32, device=dev),
              torch.empty(RAGGED_MAX_ROWS, dtype=torch.int32, device=dev))
    stream = torch.cuda.Stream()

    def step(cap):
        ops.pack_ragged(want, pos, cap, stream=stream, out=packed)
        for mats in stack:
            for name, m in mats.items():
                m["w"].mul_mat_ragged(xs[m["k"]][:cap], packed[0], out=ys[name][:cap], stream=stream)

    graphs = {}
    for cap in RAGGED_BUCKETS:
        want.fill_(cap // n_seq_max + 1)
        with torch.cuda.stream(stream):
            step(cap)  # grows the scratch outside capture
        stream.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=stream, capture_error_mode="relaxed"):
            step(cap)
        graphs[cap] = gr
    batches = ragged_batches(16, seed=seed + 2)
    flop_per_row = 2 * layers * sum(k * n for _, (k, n) in shapes())
    total_ms, total_rows, per_bucket = 0.0, 0, {}
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    for b in batches:
        w = torch.zeros(n_seq_max, dtype=torch.int32)
        p = torch.zeros(n_seq_max, dtype=torch.int32)
        w[:len(b["want"])] = torch.tensor(b["want"][:n_seq_max], dtype=torch.int32)
        p[:len(b["pos"])] = torch.tensor(b["pos"][:n_seq_max], dtype=torch.int32)
        want.copy_(w)
        pos.copy_(p)
        gr = graphs[b["bucket"]]
        with torch.cuda.stream(stream):
            for _ in range(2):
                gr.replay()
            ev[0].record(stream)
            for _ in range(reps):
                gr.replay()
            ev[1].record(stream)
        ev[1].synchronize()
        ms = ev[0].elapsed_time(ev[1]) / reps
        total_ms += ms
        total_rows += b["rows"]
        e = per_bucket.setdefault(b["bucket"], {"steps": 0, "rows": 0, "ms": 0.0})
        e["steps"] += 1
        e["rows"] += b["rows"]
        e["ms"] += ms
    for e in per_bucket.values():
        e["tflops"] = round(flop_per_row * e["rows"] / (e["ms"] * 1e-3) / 1e12, 1)
        e["ms_per_step"] = round(e["ms"] / e["steps"], 3)
        del e["ms"]
    for gr in graphs.values():
        del gr
    graphs.clear()
    for mats in stack:
        for m in mats.values():
            m["w"].free()
    torch.cuda.synchronize(device)
    tflops = flop_per_row * total_rows / (total_ms * 1e-3) / 1e12
    return {"tokens_per_s": round(total_rows / (total_ms * 1e-3), 1), "tflops": round(tflops, 1),
            "ms_per_step": round(total_ms / len(batches), 3), "avg_rows": round(total_rows / len(batches), 1),
            "steps": len(batches), "avg_bpw": round(avg_bpw, 3), "by_bucket": per_bucket,
            "launches_per_step": 1 + 2 * layers * len(shapes())}


def run_ragged(args, torch, dist, ops, rank, world, local):
    """configs[2] as its own bench line (replicas on N GPUs: every rank runs its own batches)."""
    pk, pk_kind = peaks()
    peak = float(pk.get("bf16_tflops", PEAKS_FALLBACK["bf16_tflops"]))
    if world > 1:
        dist.barrier()
    with ClockSampler(local) as clk:
        r = run_ragged_measure(torch, ops, local, args.layers, max(3, args.steps // 100), seed=77 + rank)
    tps = r["tokens_per_s"]
    if world > 1:
        t = torch.tensor([r["ms_per_step"]], dtype=torch.float64, device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        tps = r["avg_rows"] / (float(t.item()) * 1e-3)
    if rank == 0:
        print(json.dumps({
            "metric": "EXL3 ragged continuous-admission batch, tokens/s through the 196-matrix stack (configs[2])",
            "value": round(tps * world, 1), "unit": "tokens/s", "n_gpus": world, "steps": r["steps"],
            "warmup": 2, "ms_per_step": r["ms_per_step"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp16", "data": "synthetic",
            "config": {"workload": "configs[2]: 8-64 sequences per step (decode tokens + 0-3 prefill chunks of "
                                   "16-512 rows), packed on the GPU to <= 512 rows; 28 layers x 7 shapes, 25% of the "
                                   "matrices at 6 bpw, 75% at 4 bpw", "avg_bpw": r["avg_bpw"],
                       "parallelism": f"dp{world} replicas", "bucket_graphs": list(RAGGED_BUCKETS)},
            "roofline": {"bound": "tensor", "achieved": r["tflops"], "peak": peak, "unit": "TFLOP/s",
                         "frac": round(r["tflops"] / peak, 4), "peak_source": f"{pk_kind} bf16_tflops",
                         "kernel": "exl3cu::k_gemm"},
            "gpu_launches": r["launches_per_step"] * r["steps"],
            "clocks": clk.summary(), "ragged": r}), flush=True)
    return 0


def main(argv=None):
    args = parse_args(argv)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return 0

    import torch
    import torch.distributed as dist

    from exl3_b200 import ops

    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=torch.device(f"cuda:{local}"))
    if args.config == "model":
        with ClockSampler(local) as clk:
            m = run_model_measure(torch, dist, local, rank, world)
        if rank == 0:
            print(json.dumps({
                "metric": "2B hybrid decode tok/s (configs[3])", "value": m["ragged8_tok_s"], "unit": "tok/s",
                "n_gpus": world, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp16",
                "data": "synthetic", "config": {"workload": "configs[3]: 8 ragged requests per GPU, 256 greedy steps",
                                                "parallelism": f"dp{world}"},
                "clocks": clk.summary(), "detail": m}), flush=True)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return 0
    if args.config in ("large", "ragged"):
        run = run_large if args.config == "large" else run_ragged
        rc = run(args, torch, dist, ops, rank, world, local)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return rc
    pk, pk_kind = peaks()
    want_cpu = rank == 0 and world == 1 and not args.no_cpu
    stack = build_stack(torch, ops, args.bits, args.layers, local, seed=1234 + 7919 * rank,
                        keep_host_layer0=want_cpu)
    step_bytes = algo_bytes(args.bits) * args.layers

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    with ClockSampler(local) as clk:
        ms, launches = time_pattern(torch, dist, ops, stack, "decoder", args.steps, args.warmup, world)
    ms = max_over_ranks(ms)
    ms_step = ms / args.steps
    value = step_bytes * world / (ms_step * 1e-3) / 1e9

    patterns = {"decoder": {"launches_per_step": launches, "ms_per_step": round(ms_step, 5),
                            "gbs_per_gpu": round(value / world, 1)}}
    side_steps = max(20, args.steps // 4)
    for pat in ("matrix", "layer"):
        pms, pl = time_pattern(torch, dist, ops, stack, pat, side_steps, 5, world)
        pms = max_over_ranks(pms) / side_steps
        patterns[pat] = {"launches_per_step": pl, "ms_per_step": round(pms, 5),
                         "gbs_per_gpu": round(step_bytes / (pms * 1e-3) / 1e9, 1)}

    e2e_ms, h2d, d2h = time_e2e(torch, ops, stack, args.e2e_steps)
    e2e_ms = max_over_ranks(e2e_ms)
    e2e_value = step_bytes * world / (e2e_ms / args.e2e_steps * 1e-3) / 1e9
    shape_us = per_shape_us(torch, stack)
    ggml_ms, ggml_h2d, ggml_d2h, ggml_calls = time_ggml_e2e(args.bits, args.layers, max(3, args.e2e_steps // 3))
    ggml_ms = max_over_ranks(ggml_ms)

    sweep = {}
    if not args.no_sweep:
        for b in (2, 3, 5, 6):
            if b == args.bits:
                continue
            st = build_stack(torch, ops, b, args.layers, local, seed=99 + b)
            sms, _ = time_pattern(torch, dist, ops, st, "decoder", side_steps, 5, world)
            sms = max_over_ranks(sms) / side_steps
            sweep[str(b)] = round(algo_bytes(b) * args.layers / (sms * 1e-3) / 1e9, 1)
            for layer in st:
                for m in layer.values():
                    m["w"].free()
            del st
            torch.cuda.empty_cache()
        sweep[str(args.bits)] = round(value / world, 1)

    cpu = cpu_baseline(stack, args.bits) if want_cpu else None
    ragged = None
    if not args.no_ragged:
        ragged = run_ragged_measure(torch, ops, local, args.layers, 3, seed=77 + rank)
    model = None
    if not args.no_model:
        model = run_model_measure(torch, dist, local, rank, world)
    large_tp = None
    if not args.no_large:
        large_tp = large_tp_measure(torch, dist, ops, rank, world, local, bits=args.bits)

    traffic = None
    tf = ROOT / "profiles" / "gemv_traffic.json"
    if tf.exists():
        try:
            ratio = float(json.loads(tf.read_text())["dram_over_algorithmic"])
            traffic = round(ratio * step_bytes / launches)  # bytes per average decoder-pattern launch
        except (ValueError, KeyError, TypeError):
            traffic = None

    peak_hbm = float(pk.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"]))
    per_gpu = value / world
    if rank == 0:
        line = {
            "metric": METRIC,
            "value": round(value, 1),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_step, 5),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "fp16",
            "data": "synthetic",
            "config": {
                "workload": f"configs[1]: batch-1 decode GEMV sweep, {args.layers} layers x "
                            "{q,k,v,o,gate,up,down} of the 2B decoder, decoder launch pattern",
                "bits": args.bits, "rows": 1, "layers": args.layers, "matrices_per_step": 7 * args.layers,
                "launches_per_step": launches,
                "weights_mb_per_step": round(step_bytes / 1e6, 1),
                "l2": "no flush: each step streams %.0f MB of distinct weights, > 126 MB L2" % (step_bytes / 1e6),
                "activations": "fp16 N(0,1)", "accumulate": "fp32", "parallelism": f"dp{world} replicas",
                "timing": "CUDA graph of the step's C-ABI calls, replayed; CUDA events on the replay stream",
            },
            "roofline": {"bound": "hbm", "achieved": round(per_gpu, 1), "peak": peak_hbm, "unit": "GB/s",
                         "frac": round(per_gpu / peak_hbm, 4), "traffic": traffic,
                         "algorithmic_bytes_per_launch": round(step_bytes / launches),
                         "peak_source": f"{pk_kind} hbm_gbs", "kernel": "exl3cu::k_gemv_mul1<4>"},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h,
                    "api": "per step: every x copied from pinned host memory and every y back, pipelined by "
                           "layer on two copy streams around the decoder pattern's exl3cu_mul_mat_batch calls "
                           "(one CUDA graph per step), stream synchronise",
                    "ms_per_step": round(e2e_ms / args.e2e_steps, 4),
                    "per_call_ggml": {
                        "value": round(step_bytes * world / (ggml_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                        "ms_per_step": round(ggml_ms, 4), "calls_per_step": ggml_calls,
                        "h2d_bytes_per_step": ggml_h2d, "d2h_bytes_per_step": ggml_d2h,
                        "api": "ggml_exl3_mul_mat per matrix as ggml's CPU backend calls it: host ggml tensors "
                               "(records, f32 x, f32 y), synchronous per call; host wall clock"}},
            "gpu_launches": launches * args.steps,
            "clocks": clk.summary(),
            "patterns": patterns,
            "per_shape_kernel_us": shape_us,
            "sweep_gbs_by_bits": sweep,
            "ragged_configs2": ragged,
            "decode_configs3": model,
            "large_tp_configs4": large_tp,
        }
        print(json.dumps(line), flush=True)
    for layer in stack:
        for m in layer.values():
            m["w"].free()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
