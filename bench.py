#!/usr/bin/env python
"""Benchmark of the INT8 group-64 GEMV path on B200.

Default workload (one "step"): the full Llama-3.2-1B per-layer GEMV set at
batch 1 -- Wq 2048x2048, Wk 512x2048, Wv 512x2048, Wo 2048x2048,
W_gate 8192x2048, W_up 8192x2048, W_down 2048x8192 -- over 16 layers with
fresh seeds (112 GEMVs, 1.04 GB of int8 weights + fp32 scales per step),
W8A32 by default (``--form w8a8`` for the fused W8A8 form).  Weights are
N(0, 0.02) quantised per row per 64-column group with the reference scheme;
activations are N(0, 1) (W8A8: 1% of channels x20).

  value  algorithmic GB/s of a step with inputs resident in HBM: the 112
         GEMVs run as one chain launch (mli_chain_run: one CTA per SM streams
         every weight stage through a shared-memory ring, no kernel boundary
         between GEMVs).  As specified, every GEMV reads its own fresh
         activation, so no GEMV waits for another.
  e2e    the same metric with host buffers: each step copies its 112
         activation vectors from pinned host memory, runs the chain and copies
         the 112 output vectors back.
  decode_chain   the same weights in decode order with decode dependencies
         (o after q/k/v, gate/up after o, down after gate/up, the next layer
         after down), gate/up as one SwiGLU pair and down adding into the
         residual stream, also one chain launch: the GEMV part of a decode
         step, as tok/s.
  percall_graph  the 112 single-GEMV calls captured into a CUDA graph
         (programmatic dependent launch between them), for comparison.

``--impl reference`` times the reference's own kernels (matmul_int8 /
quantize_activation + matmul_dp4a from src/model_cuda_v2_shared.cu, compiled
unmodified for sm_100a into oracle/_ref) on the same workload, launched the
way the reference launches them (legacy default stream, one launch per call).

Multi-GPU (torchrun, one process per GPU): independent decode streams, each
rank runs the full step on its own replica (weak scaling, no collective on
the data path); value = all ranks' bytes / the slowest rank's time.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from minillama_infra_b200 import ops, synth  # noqa: E402

GS = 64
L2_BYTES = 126 * 1024 * 1024
KERNEL_NAME = {"w8a32": "gemv_chain_kernel<W8A32>", "w8a8": "gemv_chain_kernel<W8A8 fused>"}
PROFILE_TRAFFIC = os.path.join(ROOT, "profiles", "traffic.json")


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------
def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML during the timed region."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, device_index: int, period_s: float = 0.01):
        self.period = period_s
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # NVML unavailable: report why
            self._nv = None
            self.error = str(e)

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                bits = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for b, name in self.REASONS.items():
                    if bits & b and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self._nv is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *a):
        if self._thread is not None:
            self._stop.set()
            self._thread.join()

    def summary(self):
        if self._nv is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "error": self.error}
        return {
            "sm_mhz": float(np.median(self.samples)) if self.samples else None,
            "sm_max_mhz": self.max_mhz,
            "reasons": sorted(self.reasons),
            "samples": len(self.samples),
        }


def build_workload(form: str, device, rank: int, calls=None):
    """Weights of 16 layers x 7 shapes (same on every rank: one model),
    activations per rank (independent decode streams).  The weights are
    quantised with plain torch ops (synth.weights_torch), so building them
    loads nothing of this repository's library: both arms get the same bytes.
    `calls`: reuse another workload's weights (activations are rebuilt)."""
    if calls is None:
        layers = []
        for l in range(synth.LLAMA_1B_LAYERS):
            mats = []
            for i, (name, d, n) in enumerate(synth.LLAMA_1B):
                q, s = synth.weights_torch(d, n, seed=1000 * l + i, device=device)
                mats.append((name, d, n, q, s))
            layers.append(mats)
        calls = [m for layer in layers for m in layer]
    x_sizes = [n for (_, d, n, _, _) in calls]
    y_sizes = [d for (_, d, n, _, _) in calls]
    x_off = np.concatenate([[0], np.cumsum(x_sizes)]).astype(np.int64)
    y_off = np.concatenate([[0], np.cumsum(y_sizes)]).astype(np.int64)
    rng_x = []
    for j, n in enumerate(x_sizes):
        rng_x.append(synth.activation_np(n, seed=7919 * (rank + 1) + j, outliers=(form == "w8a8")))
    x_host = torch.from_numpy(np.concatenate(rng_x)).pin_memory()
    y_host = torch.empty(int(y_off[-1]), dtype=torch.float32).pin_memory()
    x_dev = x_host.to(device)
    y_dev = torch.empty(int(y_off[-1]), dtype=torch.float32, device=device)
    bytes_per_step = sum(synth.gemv_bytes(d, n) for (_, d, n, _, _) in calls)
    return dict(calls=calls, x_off=x_off, y_off=y_off, x_host=x_host, y_host=y_host,
                x_dev=x_dev, y_dev=y_dev, bytes=bytes_per_step)


def issue_step_ours(wl, form):
    """The 112 C-ABI calls of one step on the current stream."""
    calls, xo, yo, xd, yd = wl["calls"], wl["x_off"], wl["y_off"], wl["x_dev"], wl["y_dev"]
    for j, (_, d, n, q, s) in enumerate(calls):
        x = xd[xo[j]:xo[j + 1]]
        y = yd[yo[j]:yo[j + 1]]
        if form == "w8a32":
            ops.matmul_int8(y, x, q, s, n, d, GS)
        else:
            ops.matmul_dp4a_fused(y, x, q, s, n, d, GS)


def chain_form(form):
    return "w8a32" if form == "w8a32" else "w8a8_fused"


def build_chain_independent(wl, form):
    """The step's 112 GEMVs as one chain; each reads its own activation."""
    calls, xo, yo, xd, yd = wl["calls"], wl["x_off"], wl["y_off"], wl["x_dev"], wl["y_dev"]
    chain = [dict(form=chain_form(form), n=n, d=d, wait=0, x=xd[xo[j]:xo[j + 1]], y=yd[yo[j]:yo[j + 1]],
                  w_q=q, w_s=s) for j, (_, d, n, q, s) in enumerate(calls)]
    return ops.GemvChain(chain)


def build_chain_decode(wl, form, device):
    """The same weights in decode order, as the GEMV part of a decode step of
    the reference's forward pass (src/model_cuda_v2_shared.cu:380-415) with
    its norms and residual adds fused in: q/k/v read RMSNorm(resid) (the norm
    in their prologue), o reads q's output (standing in for attention, the one
    piece of the layer outside this path) and adds into the residual stream,
    gate/up read RMSNorm(resid) as one SwiGLU pair, down reads the SwiGLU
    output and adds into the residual stream; the next layer waits for down.
    One chain launch per step; every activation is handed over inside it."""
    names = ["q", "k", "v", "o", "gate", "up", "down"]
    calls = wl["calls"]
    resid = torch.from_numpy(synth.activation_np(2048, 4242)).to(device)
    rng = np.random.default_rng(4243)
    norms = [[torch.from_numpy((1.0 + 0.1 * rng.standard_normal(2048)).astype(np.float32)).to(device)
              for _ in range(2)] for _ in range(synth.LLAMA_1B_LAYERS)]
    outs = {nm: torch.empty(d, dtype=torch.float32, device=device) for nm, (_, d, _) in zip(names, synth.LLAMA_1B)}
    chain = []
    for l in range(synth.LLAMA_1B_LAYERS):
        for i, nm in enumerate(names):
            _, d, n, q, s = calls[7 * l + i]
            op = dict(form=chain_form(form), n=n, d=d, wait=7 * l + ops.DECODE_LAYER_WAITS[i], w_q=q, w_s=s)
            if nm in ("q", "k", "v"):
                op.update(x=resid, norm_w=norms[l][0], y=outs[nm])
            elif nm == "o":
                op.update(x=outs["q"], y=resid, epilogue="add")
            elif nm == "gate":
                op.update(x=resid, norm_w=norms[l][1], y=outs["gate"], epilogue="swiglu")
            elif nm == "up":
                op.update(x=resid, norm_w=norms[l][1], y=None)
            else:
                op.update(x=outs["gate"], y=resid, epilogue="add")
            chain.append(op)
    return ops.GemvChain(chain), (resid, norms, outs)


class PipelinedSteps:
    """End-to-end steps through the public API with host buffers, double
    buffered: step k+1's host-to-device copy of its activations and step k's
    device-to-host copy of its outputs run on their own streams while step k's
    chain runs.  Every step still copies all of its inputs in and all of its
    outputs out inside the timed region."""

    def __init__(self, wl, form, device, stream):
        self.stream = stream
        self.h2d = torch.cuda.Stream(device)
        self.d2h = torch.cuda.Stream(device)
        self.x_host = wl["x_host"]
        self.sets = []
        for b in range(2):
            xd = wl["x_dev"] if b == 0 else torch.empty_like(wl["x_dev"])
            yd = wl["y_dev"] if b == 0 else torch.empty_like(wl["y_dev"])
            yh = wl["y_host"] if b == 0 else torch.empty_like(wl["y_host"]).pin_memory()
            chain = build_chain_independent(dict(wl, x_dev=xd, y_dev=yd), form)
            self.sets.append((xd, yd, yh, chain))
        self.ev = {k: [torch.cuda.Event(), torch.cuda.Event()] for k in ("in", "done", "out")}

    def _h2d(self, k):
        b = k % 2
        if k >= 2:
            self.h2d.wait_event(self.ev["done"][b])  # step k - 2 has read this buffer
        with torch.cuda.stream(self.h2d):
            self.sets[b][0].copy_(self.x_host, non_blocking=True)
        self.ev["in"][b].record(self.h2d)

    def issue(self, steps):
        """Issues `steps` pipelined steps after work already on self.stream."""
        start = torch.cuda.Event()
        start.record(self.stream)
        self.h2d.wait_event(start)
        self.d2h.wait_event(start)
        self._h2d(0)
        for k in range(steps):
            b = k % 2
            xd, yd, yh, chain = self.sets[b]
            if k + 1 < steps:
                self._h2d(k + 1)
            self.stream.wait_event(self.ev["in"][b])
            if k >= 2:
                self.stream.wait_event(self.ev["out"][b])  # step k - 2's outputs are out
            chain.run(self.stream)
            self.ev["done"][b].record(self.stream)
            self.d2h.wait_event(self.ev["done"][b])
            with torch.cuda.stream(self.d2h):
                yh.copy_(yd, non_blocking=True)
            self.ev["out"][b].record(self.d2h)
        self.stream.wait_event(self.ev["out"][(steps - 1) % 2])
        if steps > 1:
            self.stream.wait_event(self.ev["out"][(steps - 2) % 2])

    def timed(self, steps):
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        t0.record(self.stream)
        self.issue(steps)
        t1.record(self.stream)
        t1.synchronize()
        return t0.elapsed_time(t1) / steps

    def close(self):
        torch.cuda.synchronize()
        for s in self.sets:
            s[3].close()


def make_ref_issuer(wl, form, device):
    from oracle import oracle as orc

    ref = orc.ref()
    xq = torch.empty(8192, dtype=torch.int8, device=device)
    xs = torch.empty(1, dtype=torch.float32, device=device)
    calls, xo, yo = wl["calls"], wl["x_off"], wl["y_off"]
    xp, yp = wl["x_dev"].data_ptr(), wl["y_dev"].data_ptr()
    args = [(yp + 4 * int(yo[j]), xp + 4 * int(xo[j]), q.data_ptr(), s.data_ptr(), n, d)
            for j, (_, d, n, q, s) in enumerate(calls)]

    def issue():
        if form == "w8a32":
            for (y, x, q, s, n, d) in args:
                ref.ref_matmul_int8(y, x, q, s, n, d, GS)
        else:
            for (y, x, q, s, n, d) in args:
                ref.ref_quantize_activation(xq.data_ptr(), xs.data_ptr(), x, n)
                ref.ref_matmul_dp4a(y, xq.data_ptr(), xs.data_ptr(), q, s, n, d, GS)

    return issue, ref


def timed(fn, steps, stream, sampler=None):
    """CUDA-event time of `steps` calls of fn() on `stream` (ms per step)."""
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    ctx = sampler if sampler is not None else _Null()
    with ctx:
        start.record(stream)
        for _ in range(steps):
            fn()
        end.record(stream)
        end.synchronize()
    return start.elapsed_time(end) / steps


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


def max_over_ranks(v: float, world: int, device) -> float:
    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        dist.barrier()


def check_outputs(wl, form, n_calls=7):
    """Layer-0 outputs of the last step against the CPU oracle."""
    from oracle import oracle as orc

    worst = 0.0
    y_all = wl["y_dev"].cpu().numpy()
    x_all = wl["x_dev"].cpu().numpy()
    for j, (_, d, n, q, s) in enumerate(wl["calls"][:n_calls]):
        x = x_all[wl["x_off"][j]:wl["x_off"][j + 1]]
        y = y_all[wl["y_off"][j]:wl["y_off"][j + 1]]
        qn, sn = q.cpu().numpy(), s.cpu().numpy()
        if form == "w8a32":
            ref = orc.gemv_w8a32_f64(x, qn, sn)
        else:
            xq, xs = orc.quantize_activation(x)
            ref = orc.gemv_w8a8_f64(xq, xs, qn, sn)
        worst = max(worst, orc.max_abs_rel(y, ref))
    return worst


def cpu_baseline(wl, seconds: float, layers: int = 4):
    """The path on this host's CPU cores: float32 dequant-then-matvec of the
    same quantised weights (oracle/cpu_baseline.c, compiled here with -O3
    -march=native, OpenMP over rows, each group's products vectorised) over
    the first `layers` layers' GEMVs (larger than any host cache), repeated
    for about `seconds`."""
    import tempfile

    from oracle import oracle as orc

    with tempfile.TemporaryDirectory() as td:
        cl = orc.cpu_baseline_lib(td)
    mats = [(d, n, q.cpu().numpy(), s.cpu().numpy()) for (_, d, n, q, s) in wl["calls"][:7 * layers]]
    xs = [np.ascontiguousarray(synth.activation_np(n, 100 + i)) for i, (d, n, _, _) in enumerate(mats)]
    outs = [np.empty(d, np.float32) for (d, _, _, _) in mats]
    sample_bytes = sum(synth.gemv_bytes(d, n) for (d, n, _, _) in mats)
    for (d, n, q, s), x, y in zip(mats, xs, outs):  # warm-up pass (page faults, thread pool)
        cl.cpu_dequant_matvec(y, x, q, s, n, d, GS)
    reps = 0
    t0 = time.perf_counter()
    while True:
        for (d, n, q, s), x, y in zip(mats, xs, outs):
            cl.cpu_dequant_matvec(y, x, q, s, n, d, GS)
        reps += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    cpu = ""
    try:
        with open("/proc/cpuinfo") as f:
            cpu = next((ln.split(":", 1)[1].strip() for ln in f if ln.startswith("model name")), "")
    except OSError:
        pass
    return {
        "value": round(sample_bytes * reps / el / 1e9, 3), "unit": "GB/s",
        "cores": int(cl.cpu_num_threads()), "kind": "port",
        "sample": f"layers 0-{layers - 1} of the workload ({7 * layers} GEMVs, {sample_bytes / 1e6:.1f} MB) x "
                  f"{reps} repeats, {el:.1f} s: float32 dequant-then-matvec (oracle/cpu_baseline.c, "
                  f"-O3 -march=native, OpenMP over rows, vectorised groups) on {cpu or 'this host'}",
    }


def per_shape(device, form, steps):
    """Isolated back-to-back calls of each shape, rotating over >= 2x L2 of
    distinct weight copies (CUDA graph, PDL)."""
    res = {}
    stream = torch.cuda.Stream(device)
    shapes = list(synth.LLAMA_1B) + [synth.CLASSIFIER_1B]
    for name, d, n in shapes:
        q, s = synth.weights_gpu(d, n, seed=77, device=device)
        size = synth.gemv_bytes(d, n)
        copies = max(2, -(-2 * L2_BYTES // (d * n)))
        qs = [q] + [q.clone() for _ in range(copies - 1)]
        ss = [s] + [s.clone() for _ in range(copies - 1)]
        x = synth.activation_gpu(n, 5, device, outliers=(form == "w8a8"))
        y = torch.empty(d, dtype=torch.float32, device=device)

        def issue():
            for qq, sc in zip(qs, ss):
                if form == "w8a32":
                    ops.matmul_int8(y, x, qq, sc, n, d, GS)
                else:
                    ops.matmul_dp4a_fused(y, x, qq, sc, n, d, GS)

        with torch.cuda.stream(stream):
            issue()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            issue()

        def replay():
            g.replay()

        with torch.cuda.stream(stream):
            for _ in range(3):
                replay()
            ms = timed(replay, max(3, steps // 20), stream)
        us = ms * 1000 / copies
        res[name] = {"d": d, "n": n, "us": round(us, 3), "GB/s": round(size / us / 1e3, 1)}
        del g, qs, ss
        torch.cuda.empty_cache()
    return res


def profile_case(device, form, shape_name, launches):
    """A few back-to-back launches of one shape and nothing else: the command
    the ncu summaries under profiles/ are captured from."""
    shapes = {name: (d, n) for name, d, n in list(synth.LLAMA_1B) + [synth.CLASSIFIER_1B]}
    d, n = shapes[shape_name]
    q, s = synth.weights_gpu(d, n, seed=77, device=device)
    x = synth.activation_gpu(n, 5, device, outliers=(form == "w8a8"))
    y = torch.empty(d, dtype=torch.float32, device=device)
    stream = torch.cuda.Stream(device)
    with torch.cuda.stream(stream):
        for _ in range(launches):
            if form == "w8a32":
                ops.matmul_int8(y, x, q, s, n, d, GS)
            else:
                ops.matmul_dp4a_fused(y, x, q, s, n, d, GS)
    torch.cuda.synchronize()
    print(json.dumps({"profile_case": shape_name, "form": form, "d": d, "n": n,
                      "launches": launches, "device_error": ops.device_error()}))


METRIC = "int8 group-64 GEMV achieved HBM GB/s (% peak) + Llama-3.2-1B decode tok/s"


def graph_of(fn, stream):
    """fn() captured into a CUDA graph on `stream` (after one eager run)."""
    with torch.cuda.stream(stream):
        fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        fn()
    return g


def time_graph(g, steps, warmup, stream, world, device, sampler=None):
    """ms per replay, max over ranks, with a barrier on both sides."""
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            g.replay()
        torch.cuda.synchronize()
        barrier(world)
        ms = timed(g.replay, steps, stream, sampler)
        barrier(world)
    return max_over_ranks(ms, world, device)


# ---------------------------------------------------------------------------
# batched W8A8 on the Llama-3.2-3B projections (tensor cores)
# ---------------------------------------------------------------------------
def int8_peak_measure(device, iters=4096):
    """This GPU's int8 tensor-core roof: one CTA per SM issuing back-to-back
    kind::i8 MMAs (M = 128, N = 256, K = 32) on resident operands, no loads,
    no epilogue (mli_debug_int8_mma_peak), timed with CUDA events."""
    from minillama_infra_b200._lib import check, lib

    sms = torch.cuda.get_device_properties(device).multi_processor_count
    stream = torch.cuda.current_stream()
    for _ in range(3):
        check(lib().mli_debug_int8_mma_peak(256, iters, sms, stream.cuda_stream), "int8 peak")
    torch.cuda.synchronize()
    ms = timed(lambda: check(lib().mli_debug_int8_mma_peak(256, iters, sms, stream.cuda_stream), "int8 peak"),
               5, stream)
    ops_ = sms * iters * 4 * 2 * 128 * 256 * 32
    if ops.device_error() != 0:
        raise RuntimeError("the int8 peak kernel gave up on its wait")
    return {"TOPS": round(ops_ / (ms * 1e-3) / 1e12, 1), "ms": round(ms, 4), "ctas": sms,
            "mma": "tcgen05.mma.cta_group::1.kind::i8 M=128 N=256 K=32, operands in shared memory, one "
                   "issuing thread per SM, no loads, no epilogue"}


def gemm3b_measure(args, device, rank, world, m, modes=("group", "per_call", "cuda_core"), sampler=None,
                   int8_peak=None):
    """The seven Llama-3.2-3B projections at m tokens, 4 layers with fresh
    seeds rotated so that no step finds its weights in L2.  Each rank runs its
    own batch (data parallel).  Returns ms per layer per mode and the check of
    every token of layer 0 against the oracle."""
    layers = 4
    mats = []
    for l in range(layers):
        for i, (name, d, n) in enumerate(synth.LLAMA_3B):
            q, s = synth.weights_torch(d, n, seed=5000 + 100 * l + i, device=device)
            xq = torch.empty((m, n), dtype=torch.int8, device=device)
            xs = torch.empty(m, dtype=torch.float32, device=device)
            ops.quantize_activation_rows(xq, xs, synth.activation_gpu(n, 77 + i + rank, device, m=m,
                                                                      outliers=True), m, n)
            y = torch.empty((m, d), dtype=torch.float32, device=device)
            ws = torch.zeros(max(256, ops.gemm_workspace_bytes(m, n, d)), dtype=torch.uint8, device=device)
            mats.append((name, d, n, q, s, xq, xs, y, ws))
    torch.cuda.synchronize()
    bytes_layer = sum(synth.gemv_bytes(d, n, m) for (_, d, n) in synth.LLAMA_3B)
    ops_layer = sum(synth.gemv_ops(d, n, m) for (_, d, n) in synth.LLAMA_3B)
    stream = torch.cuda.Stream(device)

    def issue(mode):
        if mode == "group":  # one launch per layer for its seven projections
            for l in range(layers):
                ops.gemm_w8a8_group([(y, xq, xs, q, s, n, d) for (_, d, n, q, s, xq, xs, y, ws)
                                     in mats[7 * l:7 * l + 7]], m)
            return
        for (_, d, n, q, s, xq, xs, y, ws) in mats:
            if mode == "cuda_core":
                ops.gemm_w8a8_cuda_core(y, xq, xs, q, s, m, n, d, GS)
            else:
                ops.gemm_w8a8(y, xq, xs, q, s, m, n, d, GS, workspace=ws)

    res = {}
    for mode in modes:
        g = graph_of(lambda: issue(mode), stream)
        res[mode] = time_graph(g, args.gemm_steps, args.warmup, stream, world, device,
                               sampler if mode == "group" else None) / layers
        del g
    # every token of layer 0 (the grouped launch's results) against the oracle
    worst = 0.0
    if rank == 0:
        from oracle import oracle as orc
        issue(modes[0])
        torch.cuda.synchronize()
        for (_, d, n, q, s, xq, xs, y, ws) in mats[:7]:
            exact = orc.gemm_w8a8_f64(xq.cpu().numpy(), xs.cpu().numpy(), q.cpu().numpy(), s.cpu().numpy())
            yn = y.cpu().numpy()
            worst = max(worst, max(orc.max_abs_rel(yn[t], exact[t]) for t in range(m)))
    peak, _ = measured_peaks()
    ms = res[modes[0]]
    out = {
        "m": m, "ms_per_layer": round(ms, 5),
        "TOPS": round(world * ops_layer / (ms * 1e-3) / 1e12, 2),
        "GB/s": round(world * bytes_layer / (ms * 1e-3) / 1e9, 1),
        "frac_of_hbm_peak_per_gpu": round(bytes_layer / (ms * 1e-3) / 1e9 / peak, 4),
        "frac_of_int8_dense_datasheet_4500_TOPS": round(ops_layer / (ms * 1e-3) / 1e12 / 4500, 4),
        "frac_of_int8_measured_peak": (round(ops_layer / (ms * 1e-3) / 1e12 / int8_peak, 4)
                                       if int8_peak else None),
        "bytes_per_layer": bytes_layer, "ops_per_layer": ops_layer,
        "check": {"max_abs_rel_vs_oracle_layer0_every_token": worst, "tolerance": 1e-6},
    }
    for mode in modes[1:]:
        out[f"{mode}_ms_per_layer"] = round(res[mode], 5)
    return out


# ---------------------------------------------------------------------------
# the 128256 x 2048 classifier, row-sharded over the ranks
# ---------------------------------------------------------------------------
def classifier_measure(args, device, rank, world, form, allgather="p2p", sampler=None):
    """Row-sharded classifier step: this rank's rows of the GEMV, the
    all-gather of the fp32 logits (fused NVLink peer stores, or NCCL) and the
    device argmax.  Total work is fixed (strong scaling).  The gathered
    logits and the argmax are checked bit for bit against the whole matrix's
    GEMV on one GPU."""
    from minillama_infra_b200._lib import check, lib
    from minillama_infra_b200.shard import PeerShardedLinear, ShardedLinear, row_shard

    _, d, n = synth.CLASSIFIER_1B
    q, s = synth.weights_torch(d, n, seed=4242, device=device)  # same matrix on every rank
    sh = row_shard(d, world, rank)
    q_local = q[sh.r0:sh.r1].clone()
    s_local = s[sh.r0:sh.r1].clone()
    x_host = torch.from_numpy(synth.activation_np(n, 4343, outliers=(form == "w8a8"))).pin_memory()
    x = x_host.to(device)
    shard_bytes = q_local.numel() + s_local.numel() * 4
    copies = max(1, -(-2 * L2_BYTES // shard_bytes))  # no step finds its shard in L2
    shards = [(q_local, s_local)] + [(q_local.clone(), s_local.clone()) for _ in range(copies - 1)]
    fused = allgather == "p2p"
    if fused:
        lins = [PeerShardedLinear(qq, ss, d, n, rank, world, form=form) for qq, ss in shards]
    else:
        lins = [ShardedLinear(qq, ss, d, n, rank, world, form=form) for qq, ss in shards] if world > 1 else None
    y1 = torch.empty(d, dtype=torch.float32, device=device)  # the whole matrix on this GPU
    if form == "w8a32":
        ops.matmul_int8(y1, x, q, s, n, d, GS)
    else:
        ops.matmul_dp4a_fused(y1, x, q, s, n, d, GS)
    torch.cuda.synchronize()
    del q, s
    torch.cuda.empty_cache()
    stream = torch.cuda.Stream(device)
    idx = torch.empty((), dtype=torch.int64, device=device)
    idx_host = torch.empty((), dtype=torch.int64).pin_memory()
    y_single = torch.empty(d, dtype=torch.float32, device=device)

    def forward(c=0):
        if fused:
            lins[c].forward(x, out=idx)  # GEMV with peer stores + wait + argmax, one launch
            return None
        if lins is not None:
            logits = lins[c].forward(x)
        else:
            logits = y_single
            qq, ss = shards[c]
            if form == "w8a32":
                ops.matmul_int8(logits, x, qq, ss, n, d, GS)
            else:
                ops.matmul_dp4a_fused(logits, x, qq, ss, n, d, GS)
        check(lib().mli_argmax(logits.data_ptr(), d, idx.data_ptr(), torch.cuda.current_stream().cuda_stream),
              "mli_argmax")
        return logits

    with torch.cuda.stream(stream):
        for _ in range(3):
            logits = forward()
    torch.cuda.synchronize()
    barrier(world)  # every rank's words of the last step have landed
    if logits is None:  # fused: this rank's copy of the last step's logits (tags checked)
        last = lins[0]
        logits = torch.from_numpy(last.read_logits(last.steps - 1)).to(device)
    ok_bits = bool(torch.equal(logits.view(torch.int32), y1.view(torch.int32)))
    ref_arg = int(torch.argmax(y1).item())
    ok_arg = int(idx.item()) == ref_arg

    def all_copies():
        for c in range(copies):
            forward(c)

    g = graph_of(all_copies, stream)
    ms = time_graph(g, args.steps, args.warmup, stream, world, device, sampler) / copies

    def step_e2e():
        x.copy_(x_host, non_blocking=True)
        g.replay()
        idx_host.copy_(idx, non_blocking=True)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step_e2e()
        torch.cuda.synchronize()
        barrier(world)
        ms_e2e = timed(step_e2e, e2e_steps(args), stream) / copies
        barrier(world)
    ms_e2e = max_over_ranks(ms_e2e, world, device)
    torch.cuda.synchronize()
    del g
    # this rank's shard GEMV alone and the argmax of a full logits vector alone
    rows = sh.rows

    def gemv_only():
        for c in range(copies):
            qq, ss = shards[c]
            if form == "w8a32":
                ops.matmul_int8(y_single[:rows], x, qq, ss, n, rows, GS)
            else:
                ops.matmul_dp4a_fused(y_single[:rows], x, qq, ss, n, rows, GS)

    def argmax_only():
        for _ in range(copies):
            check(lib().mli_argmax(y_single.data_ptr(), d, idx.data_ptr(),
                                   torch.cuda.current_stream().cuda_stream), "mli_argmax")

    g_gemv, g_arg = graph_of(gemv_only, stream), graph_of(argmax_only, stream)
    with torch.cuda.stream(stream):
        for gg in (g_gemv, g_arg):
            for _ in range(3):
                gg.replay()
        ms_g = timed(g_gemv.replay, args.steps, stream) / copies
        ms_a = timed(g_arg.replay, args.steps, stream) / copies
    del g_gemv, g_arg
    if fused:
        for lin in lins:
            lin.close()
    ok = torch.tensor([1 if (ok_bits and ok_arg) else 0], device=device)
    if world > 1:
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    bytes_step = synth.gemv_bytes(d, n)
    peak, _ = measured_peaks()
    return {
        "form": form, "gpus": world,
        "gather": "fused NVLink peer stores in the GEMV, argmax from per-CTA partials" if fused
                  else "GEMV + NCCL all_gather_into_tensor + device argmax",
        "us_per_step": round(ms * 1e3, 2), "GB/s": round(bytes_step / (ms * 1e-3) / 1e9, 1),
        "per_gpu_frac_of_hbm_peak": round(bytes_step / world / (ms * 1e-3) / 1e9 / peak, 4),
        "tokens_per_s_classifier_only": round(1000.0 / ms, 1),
        "e2e_us_per_step": round(ms_e2e * 1e3, 2),
        "rows_per_gpu": sh.chunk, "bytes_per_step": bytes_step, "steps_per_replay": copies,
        "breakdown_rank0" if rank == 0 else "breakdown": {
            "shard_gemv_us": round(ms_g * 1e3, 2), "full_argmax_us": round(ms_a * 1e3, 2),
            "shard_gemv_GB/s": round(synth.gemv_bytes(rows, n) / (ms_g * 1e-3) / 1e9, 1)},
        "check": {"logits_bit_exact_vs_1gpu": ok_bits, "argmax_equal_vs_1gpu": bool(ok.item()),
                  "argmax": ref_arg},
    }


# ---------------------------------------------------------------------------
# the Llama-3.2-1B FFN blocks, row-sharded over the ranks
# ---------------------------------------------------------------------------
def ffn_chain_measure(args, device, rank, world, form, layers=16):
    """The 16 FFN blocks of a Llama-3.2-1B decode step as a stack (layer l+1
    reads layer l's output), row-sharded over the ranks in ONE chained launch
    per step on every rank: each rank's gate/up (SwiGLU, 8192/G rows) and down
    (2048/G rows) store their rows, tagged with the launch, into every rank's
    copy of hb / x' over NVLink inside the kernel (mli_chain_create_sharded);
    no NCCL call.  Total work is fixed (strong scaling).  Every layer's hb and
    the last x' are checked bit for bit against the same stack on one GPU."""
    import numpy as np

    from minillama_infra_b200.shard import ChainShardedFFN, row_shard

    dim, hidden = 2048, 8192
    hs, ds = row_shard(hidden, world, rank), row_shard(dim, world, rank)
    full, mine = [], []
    for l in range(layers):
        g = synth.weights_torch(hidden, dim, seed=2000 * l + 4, device=device)
        u = synth.weights_torch(hidden, dim, seed=2000 * l + 5, device=device)
        d = synth.weights_torch(dim, hidden, seed=2000 * l + 6, device=device)
        full.append((g[0], g[1], u[0], u[1], d[0], d[1]))
        mine.append((g[0][hs.r0:hs.r1].clone(), g[1][hs.r0:hs.r1].clone(), u[0][hs.r0:hs.r1].clone(),
                     u[1][hs.r0:hs.r1].clone(), d[0][ds.r0:ds.r1].clone(), d[1][ds.r0:ds.r1].clone()))
    x0 = synth.activation_gpu(dim, 990, device, outliers=(form == "w8a8"))
    one = ChainShardedFFN(full, x0, dim, hidden, 0, 1, form=form)
    one.run()
    torch.cuda.synchronize()
    want = [one.hidden_rows(l)[0].view(np.uint32) for l in range(layers)] + [one.output_rows()[0].view(np.uint32)]
    one.close()
    del one, full
    torch.cuda.empty_cache()

    def exchange(h):
        out = [None] * world
        dist.all_gather_object(out, h)
        return out

    sh = ChainShardedFFN(mine, x0, dim, hidden, rank, world, form=form, exchange=exchange if world > 1 else None)
    barrier(world)
    stream = torch.cuda.Stream(device)
    g = graph_of(lambda: sh.run(stream), stream)
    ms = time_graph(g, args.ffn_steps, args.warmup, stream, world, device)
    del g
    torch.cuda.synchronize()
    barrier(world)  # every rank's last run has landed everywhere
    got = [sh.hidden_rows(l) for l in range(layers)] + [sh.output_rows()]
    ok = all(t and np.array_equal(v.view(np.uint32), w) for (v, t), w in zip(got, want))
    barrier(world)
    sh.close()
    okt = torch.tensor([1 if ok else 0], device=device)
    if world > 1:
        dist.all_reduce(okt, op=dist.ReduceOp.MIN)
    bytes_step = layers * (2 * synth.gemv_bytes(hidden, dim) + synth.gemv_bytes(dim, hidden))
    peak, _ = measured_peaks()
    return {
        "form": form, "gpus": world, "layers": layers,
        "ms_per_step": round(ms, 5), "us_per_layer": round(ms * 1e3 / layers, 2),
        "GB/s": round(bytes_step / (ms * 1e-3) / 1e9, 1),
        "per_gpu_frac_of_hbm_peak": round(bytes_step / world / (ms * 1e-3) / 1e9 / peak, 4),
        "exchange": "tagged peer stores of hb and x' rows inside one chained launch per step (no NCCL)"
                    if world > 1 else "none (one GPU)",
        "dependencies": "layer l+1 reads layer l's x'; down reads every rank's hb rows",
        "bytes_per_step": bytes_step, "launches_per_step": 1,
        "check": {"every_hb_and_last_x_bit_exact_vs_1gpu_stack": bool(okt.item())},
    }


def ffn_measure(args, device, rank, world, form, layers=16, sampler=None):
    """The 16 FFN blocks of a Llama-3.2-1B decode step row-sharded over the
    ranks (gate/up: 8192/G rows with SwiGLU, NCCL all-gather of hb; down:
    2048/G rows, NCCL all-gather of xb), one layer after the other.  Total work
    is fixed (strong scaling).  Layer 0's gathered hb and xb are checked bit
    for bit against the whole block on one GPU."""
    from minillama_infra_b200.shard import ShardedFFN, row_shard

    dim, hidden = 2048, 8192
    hs, ds = row_shard(hidden, world, rank), row_shard(dim, world, rank)
    blocks, xs = [], []
    full0 = None
    for l in range(layers):
        gate = synth.weights_torch(hidden, dim, seed=1000 * l + 4, device=device)
        up = synth.weights_torch(hidden, dim, seed=1000 * l + 5, device=device)
        down = synth.weights_torch(dim, hidden, seed=1000 * l + 6, device=device)
        x = synth.activation_gpu(dim, 900 + l, device, outliers=(form == "w8a8"))
        if l == 0:
            full0 = (gate, up, down)
        blocks.append(ShardedFFN(gate[0][hs.r0:hs.r1].clone(), gate[1][hs.r0:hs.r1].clone(),
                                 up[0][hs.r0:hs.r1].clone(), up[1][hs.r0:hs.r1].clone(),
                                 down[0][ds.r0:ds.r1].clone(), down[1][ds.r0:ds.r1].clone(),
                                 dim, hidden, rank, world, form=form))
        xs.append(x)
        del gate, up, down
    one = ShardedFFN(full0[0][0], full0[0][1], full0[1][0], full0[1][1], full0[2][0], full0[2][1],
                     dim, hidden, 0, 1, form=form)
    stream = torch.cuda.Stream(device)
    with torch.cuda.stream(stream):
        xb1 = one.forward(xs[0]).clone()
        hb1 = one.hidden_vector().clone()
        xb = blocks[0].forward(xs[0])
        torch.cuda.synchronize()
        ok = bool(torch.equal(xb.view(torch.int32), xb1.view(torch.int32))) and \
            bool(torch.equal(blocks[0].hidden_vector().view(torch.int32), hb1.view(torch.int32)))
    one.close()
    del full0, one
    torch.cuda.empty_cache()

    def step():
        for blk, x in zip(blocks, xs):
            blk.forward(x)

    def local_only():  # the rank's GEMVs without the gathers
        for blk, x in zip(blocks, xs):
            blk.compute_gateup(blk.hb_local[: blk.hs.rows], x)
            blk.compute_down(blk.xb_local[: blk.ds.rows], blk.hb_full[: blk.hidden])

    g = graph_of(step, stream)
    ms = time_graph(g, args.ffn_steps, args.warmup, stream, world, device, sampler)
    del g
    g_loc = graph_of(local_only, stream)
    ms_loc = time_graph(g_loc, args.ffn_steps, args.warmup, stream, world, device)
    del g_loc
    for blk in blocks:
        blk.close()
    okt = torch.tensor([1 if ok else 0], device=device)
    if world > 1:
        dist.all_reduce(okt, op=dist.ReduceOp.MIN)
    bytes_step = layers * (2 * synth.gemv_bytes(hidden, dim) + synth.gemv_bytes(dim, hidden))
    peak, _ = measured_peaks()
    return {
        "form": form, "gpus": world, "layers": layers,
        "ms_per_step": round(ms, 5), "us_per_layer": round(ms * 1e3 / layers, 2),
        "GB/s": round(bytes_step / (ms * 1e-3) / 1e9, 1),
        "per_gpu_frac_of_hbm_peak": round(bytes_step / world / (ms * 1e-3) / 1e9 / peak, 4),
        "local_gemvs_only_ms_per_step": round(ms_loc, 5),
        "gather": "NCCL all_gather_into_tensor of hb (8192 fp32) and xb (2048 fp32) per layer"
                  if world > 1 else "none (one GPU)",
        "bytes_per_step": bytes_step,
        "l2": f"{layers} layers x {(2 * synth.gemv_bytes(hidden, dim) + synth.gemv_bytes(dim, hidden)) / 1e6:.1f} MB"
              " of weights per step, sharded: every layer's shard is read once per step",
        "check": {"hb_and_xb_bit_exact_vs_1gpu_layer0": bool(okt.item())},
    }


# ---------------------------------------------------------------------------
# Llama-3.2-1B decode end to end through the reference's unchanged forward
# ---------------------------------------------------------------------------
REF_BIN = os.path.join(ROOT, "oracle", "_ref")
DECODE_SEQ_LEN = 136  # the dp4a benchmark decodes positions up to 127 + its prompt length


def parse_reference_output(text):
    """Per-benchmark tok/s from the reference program's own report
    (src/main_cuda.cpp:121-124, the context-scaling table of :302-307, and
    :188-191): W8A32 prompts, the W8A32 context-scaling rows, W8A8 prompts."""
    import re

    w8a32, ctx, w8a8 = [], [], []
    stage6 = False
    for ln in text.splitlines():
        if "Stage 6" in ln:
            stage6 = True
        m = re.search(r"Throughput:\s*([0-9.]+)\s*tok/s", ln)
        if m:
            (w8a8 if stage6 else w8a32).append(float(m.group(1)))
            continue
        m = re.match(r"\|\s*(\d+)\s*\|\s*([0-9.]+)\s*\|\s*([0-9.]+)\s*\|\s*([0-9.]+)\s*\|", ln)
        if m and not stage6:
            ctx.append({"context": int(m.group(1)), "ttft_ms": float(m.group(2)), "tpot_ms": float(m.group(3)),
                        "tok_s": float(m.group(4))})
    vram = re.search(r"Peak VRAM:\s*([0-9.]+)\s*MB", text)
    return {"w8a32_tok_s": w8a32, "w8a8_tok_s": w8a8, "context_scaling": ctx,
            "peak_vram_mb": float(vram.group(1)) if vram else None}


def decode_e2e_measure(device, timeout_s=900):
    """The reference's own decoder (src/main_cuda.cpp + model_cuda_v2_shared.cu +
    tokenizer.cpp, unchanged) run twice on one synthetic Llama-3.2-1B weight
    file: as the reference builds it, and with its three GEMV launchers bound
    to libmli_dropin.so at dynamic link time (oracle/Makefile).  tok/s are the
    program's own decode figures (its wall clock around the decode loop, the
    logits copy and host argmax included)."""
    import statistics
    import subprocess
    import tempfile

    from minillama_infra_b200 import weights_file as wf

    stock, dropin = os.path.join(REF_BIN, "minillama_stock"), os.path.join(REF_BIN, "minillama_dropin")
    if not (os.path.exists(stock) and os.path.exists(dropin)):
        return {"unavailable": "oracle/_ref decoder builds missing (make -C oracle REF_ROOT=<reference tree>)"}
    out = {"model": "synthetic llama-3.2-1b, N(0,0.02) weights quantised int8 group-64, norms 1, "
                    "tokenizer.bin of placeholder tokens (prompts encode to their punctuation)",
           "seq_len": DECODE_SEQ_LEN}
    with tempfile.TemporaryDirectory(dir=os.environ.get("MLI_TMP")) as td:
        model = os.path.join(td, "llama3_2_1B_q8_group.bin")
        t0 = time.perf_counter()
        wf.write_synthetic_model(model, wf.LLAMA_1B, seed=1, device=device)
        wf.write_tokenizer(os.path.join(td, "tokenizer.bin"), wf.LLAMA_1B.vocab_size,
                           {13: ".", 11: ",", 30: "?", 0: "!"})
        out["file_write_s"] = round(time.perf_counter() - t0, 1)
        torch.cuda.synchronize()
        env = dict(os.environ, CUDA_VISIBLE_DEVICES=str(device.index))
        bind = subprocess.run([dropin, "/nonexistent"], env=dict(env, LD_BIND_NOW="1", LD_DEBUG="bindings"),
                              capture_output=True, text=True, timeout=60)
        bound = [ln for ln in bind.stderr.splitlines()
                 if "libmli_dropin.so" in ln.split(" to ")[-1] and "libref_model.so" in ln.split(" to ")[0]]
        out["dropin_bindings"] = sorted({ln.split("`")[-1].rstrip("'") for ln in bound})
        for name, exe in (("reference", stock), ("dropin", dropin)):
            t0 = time.perf_counter()
            r = subprocess.run([exe, model, str(DECODE_SEQ_LEN)], cwd=td, env=env, capture_output=True,
                               text=True, timeout=timeout_s)
            if r.returncode != 0:
                out[name] = {"error": f"exit {r.returncode}", "tail": r.stdout[-400:] + r.stderr[-400:]}
                continue
            p = parse_reference_output(r.stdout)
            p["wall_s"] = round(time.perf_counter() - t0, 1)
            for k in ("w8a32_tok_s", "w8a8_tok_s"):
                p[k + "_median"] = round(statistics.median(p[k]), 2) if p[k] else None
            out[name] = p
    ref, ours = out.get("reference", {}), out.get("dropin", {})
    for k in ("w8a32_tok_s_median", "w8a8_tok_s_median"):
        if ref.get(k) and ours.get(k):
            out[f"speedup_{k.split('_')[0]}"] = round(ours[k] / ref[k], 2)
    return out


# ---------------------------------------------------------------------------
# the default workload: the Llama-3.2-1B per-layer GEMV set
# ---------------------------------------------------------------------------
def roofline_of(form, bytes_step, ms, peak, peak_kind):
    achieved = bytes_step / (ms * 1e-3) / 1e9
    traffic = None
    if os.path.exists(PROFILE_TRAFFIC):
        with open(PROFILE_TRAFFIC) as f:
            t = json.load(f).get(f"llama1b_chain_{form}")
        if t:
            traffic = t["traffic_bytes_per_launch"]
    return {
        "kernel": KERNEL_NAME[form], "bound": "hbm", "achieved": round(achieved, 1),
        "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
        "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
        else "fallback 6.65 TB/s",
        "algorithmic_bytes_per_launch": bytes_step, "traffic": traffic,
    }


def e2e_steps(args):
    """Steps of an end-to-end timing: a serving loop runs continuously, so the
    pipeline's fill (the first step's input copy) and drain (the last step's
    output copy) are spread over at least 100 steps; every step still copies
    all of its inputs in and all of its outputs out inside the timed region."""
    return max(100, args.steps)


def llama1b_measure(args, wl, form, device, rank, world, sampler=None, side=True):
    """The 112 GEMVs of a step as one chain launch (value), end to end through
    the public API with host copies (e2e), and, with `side`, the
    decode-ordered chain and the per-call graph."""
    stream = torch.cuda.Stream(device)
    pipe = PipelinedSteps(wl, form, device, stream)
    chain = pipe.sets[0][3]
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            chain.run(stream)
        torch.cuda.synchronize()
        barrier(world)
        ms = timed(lambda: chain.run(stream), args.steps, stream, sampler)
        barrier(world)
        ms = max_over_ranks(ms, world, device)
        pipe.issue(args.warmup)
        torch.cuda.synchronize()
        barrier(world)
        ms_e2e = pipe.timed(e2e_steps(args))
        barrier(world)
        ms_e2e = max_over_ranks(ms_e2e, world, device)
    torch.cuda.synchronize()
    err = check_outputs(wl, form) if rank == 0 else None
    out = {"ms": ms, "ms_e2e": ms_e2e, "err": err}
    if side:
        dchain, _resid = build_chain_decode(wl, form, device)
        g = graph_of(lambda: issue_step_ours(wl, form), stream)
        side_steps = max(20, args.steps // 5)
        for name, fn in (("decode_chain", lambda: dchain.run(stream)), ("percall_graph", g.replay)):
            with torch.cuda.stream(stream):
                for _ in range(args.warmup):
                    fn()
                torch.cuda.synchronize()
                barrier(world)
                t = max_over_ranks(timed(fn, side_steps, stream), world, device)
            out[name] = {"ms_per_step": round(t, 5), "GB/s": round(world * wl["bytes"] / (t * 1e-3) / 1e9, 2),
                         "steps": side_steps}
        out["decode_chain"]["tok_s_gemv_only"] = round(1000.0 / out["decode_chain"]["ms_per_step"], 1)
        out["decode_chain"]["dependencies"] = (
            "a decode step's layers without attention: q/k/v read RMSNorm(resid), o reads q's output "
            "(standing in for attention) and adds into resid, gate/up read RMSNorm(resid) as one SwiGLU "
            "pair, down adds into resid, the next layer after down; norms, SwiGLU and residual adds fused "
            "into the GEMVs, activations handed over inside one launch")
        out["percall_graph"]["launch"] = "112 single-GEMV C-ABI calls in a CUDA graph, programmatic dependent launch"
        torch.cuda.synchronize()
        del g
        dchain.close()
    pipe.close()
    if ops.device_error() != 0:
        raise RuntimeError("a kernel gave up on a bounded wait")
    return out


def workload_config(args, wl, world):
    return {
        "workload": f"llama-3.2-1b per-layer GEMV set, batch 1, {args.form.upper()}, 16 layers x 7 "
                    "shapes (Wq/Wk/Wv/Wo/gate/up/down), fresh seed per layer",
        "calls_per_step": len(wl["calls"]),
        "bytes_per_step": wl["bytes"],
        "parallelism": f"dp{world} (independent decode streams, one replica per GPU)",
        "l2": "inputs larger than L2: 1.04 GB of weights per step vs 126 MB L2",
    }


def base_line(args, world, ms, value, config):
    return {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32" if args.form == "w8a32" else "i8xi8->i32,f32",
        "data": "synthetic: N(0,0.02) weights quantised int8 group-64 (reference scheme), N(0,1) activations"
                + (", 1% channels x20" if args.form == "w8a8" else ""),
        "config": config,
    }


def run_reference(args):
    """The reference's own kernels (oracle/_ref/libmli_ref.so: matmul_int8 /
    quantize_activation + matmul_dp4a of src/model_cuda_v2_shared.cu,
    compiled unmodified for sm_100a) on the same workload, launched the way
    the reference launches them: legacy default stream, one eager launch per
    call.  value = kernel time with inputs resident; e2e = the same with the
    step's activations copied in and outputs copied out.  Runs on one GPU
    (rank 0 under torchrun; the other ranks exit without work)."""
    torch.cuda.set_device(0)
    device = torch.device("cuda", 0)
    wl = build_workload(args.form, device, 0)
    issue, _ref = make_ref_issuer(wl, args.form, device)
    run_stream = torch.cuda.default_stream(device)  # the legacy stream the reference uses
    sampler = ClockSampler(0)

    def step_e2e():
        wl["x_dev"].copy_(wl["x_host"], non_blocking=True)
        issue()
        wl["y_host"].copy_(wl["y_dev"], non_blocking=True)

    with torch.cuda.stream(run_stream):
        for _ in range(args.warmup):
            issue()
        torch.cuda.synchronize()
        ms = timed(issue, args.steps, run_stream, sampler)
        for _ in range(args.warmup):
            step_e2e()
        torch.cuda.synchronize()
        ms_e2e = timed(step_e2e, e2e_steps(args), run_stream)
    torch.cuda.synchronize()
    err = check_outputs(wl, args.form)
    value = wl["bytes"] / (ms * 1e-3) / 1e9
    world = int(os.environ.get("WORLD_SIZE", "1"))
    line = base_line(args, 1, ms, value, workload_config(args, wl, 1))
    e2e_v = round(wl["bytes"] / (ms_e2e * 1e-3) / 1e9, 2)
    line.update({
        "impl": "reference",
        "launch": "reference launchers (oracle/_ref), legacy default stream, one eager launch per call",
        "e2e": {"value": e2e_v, "unit": "GB/s", "ms_per_step": round(ms_e2e, 5),
                "h2d_bytes_per_step": wl["x_host"].numel() * 4, "d2h_bytes_per_step": wl["y_host"].numel() * 4,
                "steps": e2e_steps(args),
                "copies": "pinned host buffers, in order on the legacy stream"},
        "clocks": sampler.summary(),
        "check": {"max_abs_rel_vs_oracle_layer0": err, "tolerance": 1e-5 if args.form == "w8a32" else 1e-6},
        "gpu_launches": 0,
        "cpu_baseline": {
            "value": round(value, 2), "unit": "GB/s", "cores": 1, "kind": "reference",
            "sample": "the reference's own CUDA kernels (src/model_cuda_v2_shared.cu, compiled unmodified "
                      "for sm_100a into oracle/_ref) over the full workload, one host thread launching "
                      "through the reference's launchers; weights built with plain torch ops"},
        "note": "the reference runs on one GPU; " + (
            f"under torchrun with {world} ranks only rank 0 runs it, so compare it with the 1-GPU line"
            if world > 1 else "compare with the 1-GPU line"),
    })
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=500)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--form", choices=["w8a32", "w8a8"], default="w8a32")
    ap.add_argument("--allgather", choices=["p2p", "nccl"], default="p2p",
                    help="classifier: fused GEMV + NVLink peer stores (p2p) or GEMV + NCCL")
    ap.add_argument("--m", type=int, default=256, help="gemm3b workload: tokens per batch")
    ap.add_argument("--gemm-steps", type=int, default=50)
    ap.add_argument("--ffn-steps", type=int, default=50)
    ap.add_argument("--workload", choices=["llama1b", "classifier", "gemm3b", "ffn"], default="llama1b",
                    help="llama1b: the 16-layer per-layer GEMV set (default, with every other workload "
                         "as an extra key); classifier / gemm3b / ffn: that workload alone")
    ap.add_argument("--extras", default="w8a8,classifier,ffn,gemm3b,decode",
                    help="extra keys of the default line (comma list; empty for none)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--per-shape", action="store_true", help="also time each shape in isolation")
    ap.add_argument("--profile-shape", default=None,
                    help="run --launches launches of one shape (wq, wk, ..., wcls) and exit")
    ap.add_argument("--launches", type=int, default=3)
    ap.add_argument("--launch-flags", type=int, default=None,
                    help="override the library's launch flags (MLI_LAUNCH_* bits)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return  # the reference arm runs on rank 0 only
        if args.workload != "llama1b":
            why = {"gemm3b": "the reference has no batched (multi-token) int8 GEMM",
                   "classifier": "the reference has no sharded or int8 classifier (it runs an fp32 matmul "
                                 "on one GPU); compare with --workload llama1b",
                   "ffn": "the reference has no sharded FFN (one GPU); compare with --workload llama1b"}
            print(json.dumps({"impl": "reference", "unavailable": why[args.workload]}))
            return
        run_reference(args)
        return

    if args.launch_flags is not None:
        from minillama_infra_b200._lib import lib
        lib().mli_set_launch_flags(args.launch_flags)
    if args.profile_shape:
        torch.cuda.set_device(0)
        profile_case(torch.device("cuda", 0), args.form, args.profile_shape, args.launches)
        return
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    peak, peak_kind = measured_peaks()
    sampler = ClockSampler(local)
    try:
        if args.workload != "llama1b":
            run_single_workload(args, device, rank, world, sampler)
            return
        wl = build_workload(args.form, device, rank)
        main_res = llama1b_measure(args, wl, args.form, device, rank, world, sampler)
        ms, ms_e2e = main_res["ms"], main_res["ms_e2e"]
        value = world * wl["bytes"] / (ms * 1e-3) / 1e9
        line = base_line(args, world, ms, value, workload_config(args, wl, world))
        line.update({
            "impl": "ours",
            "launch": "one chain launch per step (mli_chain_run; no GEMV waits for another: each reads its "
                      "own fresh activation)",
            "e2e": {"value": round(world * wl["bytes"] / (ms_e2e * 1e-3) / 1e9, 2), "unit": "GB/s",
                    "ms_per_step": round(ms_e2e, 5), "h2d_bytes_per_step": wl["x_host"].numel() * 4,
                    "d2h_bytes_per_step": wl["y_host"].numel() * 4, "steps": e2e_steps(args),
                    "copies": "pinned host buffers; double buffered: step k+1's inputs in and step k's "
                              "outputs out on two copy streams while step k's chain runs"},
            "clocks": sampler.summary(),
            "check": {"max_abs_rel_vs_oracle_layer0": main_res["err"],
                      "tolerance": 1e-5 if args.form == "w8a32" else 1e-6},
            "decode_chain": main_res["decode_chain"], "percall_graph": main_res["percall_graph"],
            "decode_tok_s_gemv_only": main_res["decode_chain"]["tok_s_gemv_only"],
            "roofline": roofline_of(args.form, wl["bytes"], ms, peak, peak_kind),
            "gpu_launches": args.steps,
        })
        extras = [e for e in args.extras.split(",") if e]
        other = "w8a8" if args.form == "w8a32" else "w8a32"
        if other in extras:
            wl2 = build_workload(other, device, rank, calls=wl["calls"])
            r2 = llama1b_measure(args, wl2, other, device, rank, world)
            line[other] = {
                "value": round(world * wl["bytes"] / (r2["ms"] * 1e-3) / 1e9, 2), "unit": "GB/s",
                "ms_per_step": round(r2["ms"], 5),
                "e2e": {"value": round(world * wl["bytes"] / (r2["ms_e2e"] * 1e-3) / 1e9, 2), "unit": "GB/s",
                        "ms_per_step": round(r2["ms_e2e"], 5)},
                "roofline": roofline_of(other, wl["bytes"], r2["ms"], peak, peak_kind),
                "check": {"max_abs_rel_vs_oracle_layer0": r2["err"],
                          "tolerance": 1e-5 if other == "w8a32" else 1e-6},
                "decode_chain": r2["decode_chain"], "percall_graph": r2["percall_graph"],
                "data": "same weights; activations N(0,1)" + (" with 1% channels x20" if other == "w8a8" else ""),
            }
            del wl2
        del wl
        torch.cuda.empty_cache()
        if "classifier" in extras:
            line["classifier_rowshard"] = {f: classifier_measure(args, device, rank, world, f)
                                           for f in ("w8a32", "w8a8")}
        if "ffn" in extras:
            line["ffn_rowshard"] = {f: ffn_measure(args, device, rank, world, f) for f in ("w8a32", "w8a8")}
            line["ffn_chain_rowshard"] = {f: ffn_chain_measure(args, device, rank, world, f)
                                          for f in ("w8a32", "w8a8")}
        if "gemm3b" in extras:
            peak = int8_peak_measure(device)
            line["gemm3b"] = {f"m{m}": gemm3b_measure(args, device, rank, world, m, modes=("group", "per_call"),
                                                      int8_peak=peak["TOPS"])
                              for m in (16, 64, 256)}
            line["gemm3b"]["int8_tensor_peak_measured"] = peak
        if "decode" in extras and world == 1:
            line["decode_e2e"] = decode_e2e_measure(device)
        if world == 1 and not args.no_cpu_baseline:
            wl_cpu = build_workload(args.form, device, rank)
            line["cpu_baseline"] = cpu_baseline(wl_cpu, args.cpu_seconds)
            del wl_cpu
        if args.per_shape:
            line["per_shape"] = per_shape(device, args.form, args.steps)
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()


def run_single_workload(args, device, rank, world, sampler):
    """--workload classifier / gemm3b / ffn: that workload's own line."""
    if args.workload == "classifier":
        r = classifier_measure(args, device, rank, world, args.form, args.allgather, sampler)
        ms = r["us_per_step"] / 1e3
        config = {"workload": f"llama-3.2-1b classifier 128256x2048 {args.form.upper()}, rows sharded over "
                              f"{world} GPU(s), fp32 logits all-gathered ({r['gather']})",
                  "rows_per_gpu": r["rows_per_gpu"], "bytes_per_step": r["bytes_per_step"],
                  "parallelism": f"row-shard tp{world}",
                  "l2": f"steps rotate over {r['steps_per_replay']} copies of the shard, >= 2x the 126 MB L2",
                  "steps_per_replay": r["steps_per_replay"]}
        value = r["GB/s"]
        scaling = "strong"
        extra = {"classifier": r, "gpu_launches": args.steps * r["steps_per_replay"] * (1 if args.allgather == "p2p" else 2),
                 "e2e": {"value": round(r["bytes_per_step"] / (r["e2e_us_per_step"] * 1e-6) / 1e9, 2), "unit": "GB/s",
                         "ms_per_step": round(r["e2e_us_per_step"] / 1e3, 5),
                         "h2d_bytes_per_step": 2048 * 4 // r["steps_per_replay"],
                         "d2h_bytes_per_step": max(1, 8 // r["steps_per_replay"]),
                         "note": f"one H2D of x and one D2H of the argmax per graph replay of {r['steps_per_replay']} steps"}}
    elif args.workload == "ffn":
        r = ffn_measure(args, device, rank, world, args.form, sampler=sampler)
        ms = r["ms_per_step"]
        config = {"workload": f"llama-3.2-1b FFN blocks (gate/up/down, 16 layers) {args.form.upper()}, rows "
                              f"sharded over {world} GPU(s), NCCL all-gather of hb and xb",
                  "bytes_per_step": r["bytes_per_step"], "parallelism": f"row-shard tp{world}", "l2": r["l2"]}
        value = r["GB/s"]
        scaling = "strong"
        extra = {"ffn": r, "gpu_launches": args.ffn_steps * 16 * 2}
    else:
        peak = int8_peak_measure(device)
        r = gemm3b_measure(args, device, rank, world, args.m, sampler=sampler, int8_peak=peak["TOPS"])
        r["int8_tensor_peak_measured"] = peak
        ms = r["ms_per_layer"]
        config = {"workload": f"llama-3.2-3b per-layer projections (7 GEMMs) at M={args.m} tokens, W8A8, tcgen05 "
                              "kind::i8 path, one grouped launch per layer", "m": args.m,
                  "bytes_per_step": r["bytes_per_layer"], "ops_per_step": r["ops_per_layer"],
                  "parallelism": f"dp{world} (independent token batches)",
                  "l2": "4 layers with fresh seeds rotated, > 2x L2"}
        value = r["GB/s"]
        scaling = "weak"
        extra = {"gemm3b": r, "gpu_launches": args.gemm_steps * 4}
    if rank == 0:
        line = base_line(args, world, ms, value, config)
        line["scaling"] = scaling
        if args.workload == "gemm3b":
            line["dtype"] = "i8xi8->i32,f32"
        line.update(extra)
        line["clocks"] = sampler.summary()
        line["impl"] = "ours"
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
