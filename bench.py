"""Benchmark of the linear-layer hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (one "step" = one pass of the hot path over one batch): the four
projections of one TinyLlama-1.1B-shaped decoder layer at prefill M=512 tokens,
fp16, fused epilogues as the engine calls them:
    q/k/v   [512,2048] x [2560,2048]^T
    o_proj  [512,2048] x [2048,2048]^T  + residual
    gate/up [512,2048] x [11264,2048]^T + SwiGLU -> [512,5632]
    down    [512,5632] x [2048,5632]^T  + residual
45.10 GFLOP per step (2*M*N*K, epilogues not counted).  Weights ~N(0,0.02),
activations ~N(0,1), seeded, random-init (no checkpoint).  Steps rotate over 4
independent layer copies (352 MB of weights, > the 126 MB L2), so every step
streams its weights from HBM.

N > 1 (launched by torch.distributed.run): tensor parallel over N GPUs, the
same total work (strong scaling): q/k/v by heads (KV heads replicated when
N > 4), gate/up by intermediate feature, o/down by K followed by the fp32
reduction of the partial sums over NVLink peer memory (or ncclAllReduce with
--nccl-reduce) and the residual/rounding step.

--impl reference: the reference has no CPU implementation of this path, so the
reference arm times the CPU oracle's multithreaded fp32 GEMM (oracle/liborc.so)
on the same layer, one bounded slice of the layer's rows per step.

Prints one JSON line (rank 0).
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import re
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOAD = "tinyllama_layer_prefill_m512"
M, H, KVD, IM = 512, 2048, 256, 5632
N_HEADS, N_KV, HEAD_DIM = 32, 4, 64
QKV_N = H + 2 * KVD
GEMMS = {  # name: (N_out, K, epilogue)
    "qkv": (QKV_N, H, "none"),
    "o_proj": (H, H, "residual"),
    "gate_up": (IM, H, "swiglu"),
    "down": (H, IM, "residual"),
}
FLOPS = {"qkv": 2 * M * QKV_N * H, "o_proj": 2 * M * H * H, "gate_up": 2 * M * 2 * IM * H,
         "down": 2 * M * H * IM}
STEP_FLOPS = sum(FLOPS.values())  # 45.10e9
N_COPIES = 4
GRAPH_CHUNK = 500
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return p, "measured"
    except Exception:
        return FALLBACK_PEAKS, "fallback"


def profile_traffic(kernel: str) -> float | None:
    """DRAM bytes per launch of `kernel` on this workload, from the committed
    ncu summary (profiles/<kernel>_<workload>.md, line 'traffic_bytes_per_launch: X')."""
    path = os.path.join(ROOT, "profiles", f"{kernel}_{WORKLOAD}.md")
    try:
        txt = open(path).read()
    except OSError:
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", txt)
    return float(m.group(1)) if m else None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus: list[int]):
        self.gpus = gpus
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", ",".join(map(str, self.gpus)), "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
                self.lines = [l for l in out.splitlines() if l.strip()]
            except Exception:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                s, m_ = float(f[1]), float(f[2])
            except ValueError:
                continue
            mx = m_
            sm.append(s)
            for i, n in enumerate(names):
                if f[5 + i].lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": [], "samples": 0}
        loaded = [s for s in sm if s > 0.5 * (mx or max(sm))] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------- our arm

def make_layers(rank: int, world: int, dev):
    """N_COPIES layer weight sets, sharded for this rank (world 1 = whole)."""
    import orininfer_b200 as ob
    from orininfer_b200 import tp
    from orininfer_b200.synth import seeded

    layers = []
    for c in range(N_COPIES):
        s = 1000 * (c + 1)
        wq = seeded((H, H), s + 1, 0.02)
        wk = seeded((KVD, H), s + 2, 0.02)
        wv = seeded((KVD, H), s + 3, 0.02)
        wo = seeded((H, H), s + 4, 0.02)
        wg = seeded((IM, H), s + 5, 0.02)
        wu = seeded((IM, H), s + 6, 0.02)
        wd = seeded((H, IM), s + 7, 0.02)
        L = {}
        L["qkv"] = tp.shard_qkv(wq, wk, wv, N_HEADS, N_KV, HEAD_DIM, rank, world).to(dev)
        g, u = tp.shard_gate_up_rows(wg, wu, rank, world)
        L["gate_up"] = ob.pack_gate_up(g.to(dev), u.to(dev))
        if world == 1:
            L["o_proj"] = wo.to(dev)
            L["down"] = wd.to(dev)
        else:
            L["o_proj"] = tp.shard_cols(wo, rank, world).to(dev)
            L["down"] = tp.shard_cols(wd, rank, world).to(dev)
        layers.append(L)
    torch.cuda.synchronize()
    return layers


class Step:
    """One layer pass (4 projections), on the current stream."""

    def __init__(self, layers, rank, world, dev, comm=None, use_workspace=True):
        import orininfer_b200 as ob
        from orininfer_b200.synth import seeded

        self.ob = ob
        self.layers = layers
        self.world = world
        self.comm = comm
        qd_local = H // world
        im_local = IM // world
        # inputs of this step: normed hidden, attention output, residual
        # stream, post-attention normed hidden (synthetic, ~N(0,1))
        self.h = seeded((M, H), 11, 1.0).to(dev)
        self.attn = seeded((M, H), 12, 1.0).to(dev)[:, :qd_local].contiguous() if world > 1 \
            else seeded((M, H), 12, 1.0).to(dev)
        self.x = seeded((M, H), 13, 1.0).to(dev)
        self.h2 = seeded((M, H), 14, 1.0).to(dev)
        self.qkv = torch.empty((M, layers[0]["qkv"].shape[0]), dtype=torch.float16, device=dev)
        self.x1 = torch.empty((M, H), dtype=torch.float16, device=dev)
        self.act = torch.empty((M, im_local), dtype=torch.float16, device=dev)
        self.x2 = torch.empty((M, H), dtype=torch.float16, device=dev)
        self.partial = torch.empty((M, H), dtype=torch.float32, device=dev)
        # stream-K workspace shared by the step's GEMMs (one stream)
        self.ws = ob.linear_workspace(dev) if use_workspace else None
        # our kernels per step: 4 GEMMs (+ 2 all-reduce finish kernels under TP)
        self.launches = 4 if world == 1 else 6

    def run(self, i: int, events=None):
        L = self.layers[i % len(self.layers)]
        ob = self.ob
        s = torch.cuda.current_stream()

        def mark(name, which):
            if events is not None:
                events[name][which].record(s)

        ws = self.ws
        mark("qkv", 0)
        ob.linear_into(self.qkv, self.h, L["qkv"], workspace=ws)
        mark("qkv", 1)
        mark("o_proj", 0)
        if self.world == 1:
            ob.linear_into(self.x1, self.attn, L["o_proj"], epilogue="residual", residual=self.x,
                           workspace=ws)
        else:
            self.comm.linear_row(self.attn, L["o_proj"], residual=self.x, out=self.x1,
                                 partial=self.partial)
        mark("o_proj", 1)
        mark("gate_up", 0)
        ob.linear_into(self.act, self.h2, L["gate_up"], epilogue="swiglu", workspace=ws)
        mark("gate_up", 1)
        mark("down", 0)
        if self.world == 1:
            ob.linear_into(self.x2, self.act, L["down"], epilogue="residual", residual=self.x1,
                           workspace=ws)
        else:
            self.comm.linear_row(self.act, L["down"], residual=self.x1, out=self.x2,
                                 partial=self.partial)
        mark("down", 1)


def capture(step: Step, n: int, start: int = 0, events_per_step=None):
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            for i in range(n):
                step.run(start + i, events_per_step[i] if events_per_step else None)
    torch.cuda.current_stream().wait_stream(s)
    return g


_LIBCUDA = None


def upload_graph(g) -> None:
    """Upload an instantiated CUDA graph to the device (cuGraphUpload) on the
    current stream, so that its first replay inside a timed region does not
    pay the upload.  Nothing of the graph runs."""
    global _LIBCUDA
    if _LIBCUDA is None:
        _LIBCUDA = ctypes.CDLL("libcuda.so.1")
        _LIBCUDA.cuGraphUpload.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        _LIBCUDA.cuGraphUpload.restype = ctypes.c_int
    rc = _LIBCUDA.cuGraphUpload(ctypes.c_void_p(g.raw_cuda_graph_exec()),
                                ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    if rc != 0:
        raise RuntimeError(f"cuGraphUpload: CUresult {rc}")


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def time_steps(step: Step, steps: int, warmup: int, world: int, dev_index: int):
    """Warm up, then time exactly `steps` steps via CUDA graph chunks."""
    step.run(0)  # uncaptured first call: per-device set-up happens outside capture
    torch.cuda.synchronize()
    chunk = min(GRAPH_CHUNK, steps)
    g = capture(step, chunk)
    rem = steps % chunk
    g_rem = capture(step, rem) if rem else None
    g_warm = capture(step, warmup) if warmup > 0 else None
    if g_warm is not None:
        g_warm.replay()
    upload_graph(g)
    if g_rem is not None:
        upload_graph(g_rem)
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler([dev_index] if world == 1 else list(range(world))) as clk:
        start.record()
        for _ in range(steps // chunk):
            g.replay()
        if g_rem is not None:
            g_rem.replay()
        stop.record()
        torch.cuda.synchronize()
    barrier(world)
    ms = start.elapsed_time(stop)
    ms = max_over_ranks(ms, world)
    del g, g_rem, g_warm
    return ms, clk.summary()


def parity_report(step: Step) -> dict:
    """One step's four outputs against a plain PyTorch fp32 reference computed
    on the GPU from the same 16-bit inputs, with the reference's rounding
    points (kernels/matmul.cu:43, fused_swiglu.cu:11-15, softmax.cu:81): per
    projection the normwise max relative error max|y-r| / max|r|, the
    elementwise one max |y-r|/|r| over |r| >= 1e-2 max|r|, the mean absolute
    error and the share of bit-identical outputs.  Outside the timed region."""
    import torch.nn.functional as F

    if step.world != 1:
        return {}
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        step.run(0)
        torch.cuda.synchronize()
        L = step.layers[0]
        dt = step.h.dtype

        def r16(t):
            return t.to(dt).float()

        gu = L["gate_up"].view(IM // 64, 2, 64, H)
        wg, wu = gu[:, 0].reshape(IM, H), gu[:, 1].reshape(IM, H)
        g = r16(F.linear(step.h2.float(), wg.float()))
        u = r16(F.linear(step.h2.float(), wu.float()))
        acc_o = r16(F.linear(step.attn.float(), L["o_proj"].float()))
        acc_d = r16(F.linear(step.act.float(), L["down"].float()))
        refs = {
            "qkv": (step.qkv, r16(F.linear(step.h.float(), L["qkv"].float())), None),
            "o_proj": (step.x1, r16(step.x.float() + acc_o), acc_o),
            "gate_up": (step.act, r16(g / (1.0 + torch.exp(-g)) * u), None),
            "down": (step.x2, r16(step.x1.float() + acc_d), acc_d),
        }
        out = {}
        for k, (y, r, acc) in refs.items():
            y = y.float()
            d = (y - r).abs()
            ra = r.abs()
            mx = float(ra.max())
            keep = ra >= 1e-2 * mx
            out[k] = {"max_rel_normwise": float(d.max()) / mx,
                      "max_rel_elementwise": float((d[keep] / ra[keep]).max()),
                      "mae": float(d.mean()), "exact": float((d == 0).double().mean())}
            if acc is not None:
                # the residual outputs where x and round16(acc) do not cancel:
                # a one-unit flip of round16(acc) is ulp(acc), which on an
                # output far below |acc| is a large ratio that says nothing
                # about the kernel
                nc = keep & (ra >= 0.25 * acc.abs())
                out[k]["max_rel_elementwise_no_cancel"] = float((d[nc] / ra[nc]).max())
            out[k] = {kk: round(v, 6) for kk, v in out[k].items()}
        out["reference"] = "torch fp32 GEMM on the GPU, 16-bit rounding at the reference's points"
        out["bar"] = "max relative error <= 1e-2, mean absolute error <= 1e-3"
        out["elementwise"] = ("max |y-r|/|r| over |r| >= 1e-2 max|r|; for the residual "
                              "epilogues also over the outputs with |r| >= |round16(acc)|/4")
        return out
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def kernel_breakdown(step: Step, n: int):
    """Average device time per launch of each projection (CUDA events on the
    launching stream, inside a captured graph of n steps)."""
    events = [{k: (torch.cuda.Event(enable_timing=True, external=True),
                   torch.cuda.Event(enable_timing=True, external=True))
               for k in GEMMS} for _ in range(n)]
    g = capture(step, n, events_per_step=events)
    g.replay()  # warm
    torch.cuda.synchronize()
    g.replay()
    torch.cuda.synchronize()
    out = {}
    for k in GEMMS:
        ts = [e[k][0].elapsed_time(e[k][1]) for e in events]
        out[k] = statistics.mean(ts)
    del g
    return out


def cublas_bar(step: Step, steps: int) -> dict:
    """The reference's M>1 path on this workload: cublasGemmEx-equivalent
    fp16 GEMMs (torch.nn.functional.linear -> cuBLAS), unfused, with the
    reference's separate SwiGLU and residual-add passes, graph-timed like
    our arm.  A comparison bar only; nothing here is our kernel."""
    import torch.nn.functional as F

    L0 = step.layers
    gate_w = [L["gate_up"] for L in L0]  # packed rows: the same FLOPs

    def run(i):
        L = L0[i % len(L0)]
        q = F.linear(step.h, L["qkv"])
        o = F.linear(step.attn, L["o_proj"])
        x1 = step.x + o
        gu = F.linear(step.h2, gate_w[i % len(L0)])
        a = F.silu(gu[:, :IM]) * gu[:, IM:]
        d = F.linear(a, L["down"])
        x2 = x1 + d
        return q, x2

    run(0)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    n = min(steps, 200)
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            for i in range(n):
                run(i)
    torch.cuda.current_stream().wait_stream(s)
    g.replay()
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(5):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / (5 * n)
    del g
    return {"ms_per_step": round(ms, 5), "tflops": round(STEP_FLOPS / (ms / 1e3) / 1e12, 2),
            "what": "torch.nn.functional.linear (cuBLAS) x4 + unfused SiLU*up and residual adds, "
                    "CUDA graph, same weights"}


def e2e_through_abi(step: Step, steps: int, dev):
    """The same metric through the public API with host buffers: every step
    copies its four inputs from pinned host memory and reads its output back.
    As a serving loop would, the copies run on their own streams, double
    buffered, so step i+1's upload and step i-1's download overlap step i's
    GEMMs; the timed region spans the first upload to the last download."""
    names = ("h", "attn", "x", "h2")
    hosts = [{n: getattr(step, n).cpu().pin_memory() for n in names} for _ in range(2)]
    out_host = [torch.empty((M, H), dtype=torch.float16).pin_memory() for _ in range(2)]
    dev_in = [{n: torch.empty_like(getattr(step, n)) for n in names} for _ in range(2)]
    dev_out = [torch.empty_like(step.x2) for _ in range(2)]
    h2d = sum(t.numel() * t.element_size() for t in hosts[0].values())
    d2h = out_host[0].numel() * out_host[0].element_size()
    comp = torch.cuda.current_stream()
    up, down = torch.cuda.Stream(), torch.cuda.Stream()
    uploaded = [torch.cuda.Event() for _ in range(2)]
    computed = [torch.cuda.Event() for _ in range(2)]
    downloaded = [torch.cuda.Event() for _ in range(2)]
    consumed = [torch.cuda.Event() for _ in range(2)]
    saved = {n: getattr(step, n) for n in names + ("x2",)}

    def upload(i):
        b = i % 2
        with torch.cuda.stream(up):
            if i >= 2:
                up.wait_event(consumed[b])      # step i-2 has read these buffers
            for n in names:
                dev_in[b][n].copy_(hosts[b][n], non_blocking=True)
            uploaded[b].record(up)

    def compute(i):
        b = i % 2
        comp.wait_event(uploaded[b])
        if i >= 2:
            comp.wait_event(downloaded[b])      # step i-2's output has left
        for n in names:
            setattr(step, n, dev_in[b][n])
        step.x2 = dev_out[b]
        step.run(i)
        consumed[b].record(comp)
        computed[b].record(comp)

    def download(i):
        b = i % 2
        with torch.cuda.stream(down):
            down.wait_event(computed[b])
            out_host[b].copy_(dev_out[b], non_blocking=True)
            downloaded[b].record(down)

    def run(n):
        upload(0)
        for i in range(n):
            if i + 1 < n:
                upload(i + 1)
            compute(i)
            download(i)
        comp.wait_stream(down)

    try:
        run(5)
        torch.cuda.synchronize()
        start = torch.cuda.Event(enable_timing=True)
        stop = torch.cuda.Event(enable_timing=True)
        start.record(comp)
        up.wait_stream(comp)
        down.wait_stream(comp)
        run(steps)
        stop.record(comp)
        torch.cuda.synchronize()
        ms = start.elapsed_time(stop)
    finally:
        for n, t in saved.items():
            setattr(step, n, t)
    return ms, h2d, d2h


VOCAB, N_LAYERS = 32000, 22
DECODE_TOKENS = (1, 8, 32, 64)


def decode_path(dev, reps: int, with_cublas: bool = True) -> dict:
    """The decode-time GEMM path of a whole TinyLlama-shaped model: 22 layers x
    (q/k/v, o_proj + residual, gate/up + SwiGLU, down + residual) and the LM
    head (fp32 logits), at M in {1, 8, 32, 64} tokens, one CUDA graph per M.
    Attention and the norms are not part of the path: the o_proj input and the
    normed hidden are fixed synthetic buffers.  1.55 GB of random-init fp16
    weights (> L2), so every step streams them from HBM; GB/s counts the
    algorithmic bytes (weights once, activations in, outputs out)."""
    import torch.nn.functional as F

    import orininfer_b200 as ob

    gen = torch.Generator(device=dev)
    gen.manual_seed(2024)

    def weight(rows, cols):
        return (torch.randn((rows, cols), generator=gen, device=dev) * 0.02).half()

    layers = [{"qkv": weight(QKV_N, H), "o_proj": weight(H, H), "gate_up": weight(2 * IM, H),
               "down": weight(H, IM)} for _ in range(N_LAYERS)]
    lm_head = weight(VOCAB, H)
    w_bytes = 2 * (N_LAYERS * (QKV_N * H + H * H + 2 * IM * H + H * IM) + VOCAB * H)
    out = {"what": "22 layers x (q/k/v, o_proj+residual, gate/up+SwiGLU, down+residual) + "
                   "LM head (fp32 logits), CUDA graph per M, weights > L2",
           "weight_bytes": w_bytes, "launches_per_step": 4 * N_LAYERS + 1, "by_tokens": {}}
    peaks, _ = load_peaks()
    hbm = peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])

    def graph_ms(fn):
        fn()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                fn()
        torch.cuda.current_stream().wait_stream(s)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            g.replay()
        b.record()
        torch.cuda.synchronize()
        del g
        return a.elapsed_time(b) / reps

    for m in DECODE_TOKENS:
        x = (torch.randn((m, H), generator=gen, device=dev)).half()      # normed hidden
        attn = (torch.randn((m, H), generator=gen, device=dev)).half()   # attention output
        h = (torch.randn((m, H), generator=gen, device=dev)).half()      # residual stream
        h0 = h.clone()
        qkv = torch.empty((m, QKV_N), dtype=torch.float16, device=dev)
        act = torch.empty((m, IM), dtype=torch.float16, device=dev)
        logits = torch.empty((m, VOCAB), dtype=torch.float32, device=dev)

        def ours():
            h.copy_(h0)
            for L in layers:
                ob.linear_into(qkv, x, L["qkv"])
                ob.linear_into(h, attn, L["o_proj"], epilogue="residual", residual=h)
                ob.linear_into(act, x, L["gate_up"], epilogue="swiglu")
                ob.linear_into(h, act, L["down"], epilogue="residual", residual=h)
            ob.linear_into(logits, h, lm_head, epilogue="f32")

        ms = graph_ms(ours)
        ob.device_check()
        a_bytes = 2 * m * (N_LAYERS * (H + QKV_N + 3 * H + H + IM + IM + 2 * H) + H) + 4 * m * VOCAB
        gbs = (w_bytes + a_bytes) / (ms / 1e3) / 1e9
        rec = {"ms_per_step": round(ms, 4), "gbs": round(gbs, 1),
               "hbm_frac": round(gbs / hbm, 4)}
        if with_cublas:
            def ref():
                hh = h0.clone()
                for L in layers:
                    F.linear(x, L["qkv"], out=qkv)
                    hh = hh + F.linear(attn, L["o_proj"])
                    gu = F.linear(x, L["gate_up"]).view(m, IM // 64, 2, 64)
                    a_ = (F.silu(gu[:, :, 0].float()) * gu[:, :, 1].float()).half()
                    hh = hh + F.linear(a_.reshape(m, IM), L["down"])
                F.linear(hh, lm_head).float()

            cms = graph_ms(ref)
            rec["cublas_ms_per_step"] = round(cms, 4)
            rec["cublas_gbs"] = round((w_bytes + a_bytes) / (cms / 1e3) / 1e9, 1)
        out["by_tokens"][str(m)] = rec
        del x, attn, h, h0, qkv, act, logits
    out["peak_hbm_gbs"] = hbm
    del layers, lm_head
    torch.cuda.empty_cache()
    return out


def _graph_ms(fn, reps: int) -> float:
    """Average ms of one call of fn, replayed `reps` times as one captured
    CUDA graph (uploaded and warmed up first)."""
    fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    upload_graph(g)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    del g
    return a.elapsed_time(b) / reps


def single_linear_m1(dev, reps: int) -> dict:
    """Config 1: y = x . W^T with x [1, 2048], W [2048, 2048] fp16 (x ~ N(0,1),
    W ~ N(0, 0.02^2)), fp32 accumulate, fp16 out.  One call streams 8.4 MB, about
    1.3 us at the copy bandwidth, so 64 weight copies (537 MB, > 4x L2) rotate:
    each call reads a W that is not in L2.  A captured graph of 64 calls is
    replayed `reps` times; GB/s counts 2 (MK + NK + MN) bytes per call."""
    import torch.nn.functional as F

    import orininfer_b200 as ob

    K_, N_, copies = 2048, 2048, 64
    gen = torch.Generator(device=dev)
    gen.manual_seed(0)
    x = torch.randn((1, K_), generator=gen, device=dev).half()
    Ws = [(torch.randn((N_, K_), generator=gen, device=dev) * 0.02).half()
          for _ in range(copies)]
    y = torch.empty((1, N_), dtype=torch.float16, device=dev)

    def ours():
        for W in Ws:
            ob.linear_into(y, x, W)

    def cublas():
        for W in Ws:
            F.linear(x, W, out=y)

    per = 2 * (K_ + N_ * K_ + N_)
    ms = _graph_ms(ours, reps) / copies
    ob.device_check()
    cms = _graph_ms(cublas, reps) / copies
    peaks, _ = load_peaks()
    hbm = peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])
    gbs = per / (ms / 1e3) / 1e9
    out = {"workload": "single_linear_m1_2048x2048", "M": 1, "N": N_, "K": K_,
           "bytes_per_call": per, "us_per_call": round(ms * 1e3, 3), "gbs": round(gbs, 1),
           "hbm_frac": round(gbs / hbm, 4), "peak_hbm_gbs": hbm,
           "cublas_us_per_call": round(cms * 1e3, 3),
           "cublas_gbs": round(per / (cms / 1e3) / 1e9, 1),
           "l2": f"{copies} rotating weight copies ({copies * N_ * K_ * 2 >> 20} MiB)",
           "kernel": ob_plan(1, N_, K_, "none")}
    del Ws
    torch.cuda.empty_cache()
    return out


def llama3_decode(dev, reps: int) -> dict:
    """Config 4 at decode: one Llama-3-8B-shaped layer's projections (q/k/v
    6144x4096, o_proj 4096x4096 + residual, gate/up 28672x4096 + SwiGLU, down
    4096x14336 + residual) and the LM head (128256x4096, fp32 logits) at M = 1
    and 32 token rows, fp16, random-init weights (436 MB + 1050 MB, each far
    above L2), one captured graph per M; next to torch.nn.functional.linear
    (cuBLAS) with unfused epilogues.  GB/s = algorithmic bytes (weights once,
    activations in and out) / time."""
    import torch.nn.functional as F

    import orininfer_b200 as ob

    H_, IM_, V_ = L3_H, L3_IM, 128256
    QKV_ = (L3_HEADS + 2 * L3_KV) * L3_HD
    gen = torch.Generator(device=dev)
    gen.manual_seed(88)

    def w(r, c):
        return (torch.randn((r, c), generator=gen, device=dev) * 0.02).half()

    Wqkv, Wo, Wgu, Wd, Wlm = w(QKV_, H_), w(H_, H_), w(2 * IM_, H_), w(H_, IM_), w(V_, H_)
    w_layer = 2 * (QKV_ * H_ + H_ * H_ + 2 * IM_ * H_ + H_ * IM_)
    w_head = 2 * V_ * H_
    peaks, _ = load_peaks()
    hbm = peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])
    out = {"workload": "llama3_8b_decode_layer_and_lm_head", "weight_bytes_layer": w_layer,
           "weight_bytes_lm_head": w_head, "by_tokens": {}, "peak_hbm_gbs": hbm}
    for m in (1, 32):
        x = torch.randn((m, H_), generator=gen, device=dev).half()
        attn = torch.randn((m, H_), generator=gen, device=dev).half()
        h0 = torch.randn((m, H_), generator=gen, device=dev).half()
        h = h0.clone()
        qkv = torch.empty((m, QKV_), dtype=torch.float16, device=dev)
        act = torch.empty((m, IM_), dtype=torch.float16, device=dev)
        logits = torch.empty((m, V_), dtype=torch.float32, device=dev)

        def ours():
            h.copy_(h0)
            ob.linear_into(qkv, x, Wqkv)
            ob.linear_into(h, attn, Wo, epilogue="residual", residual=h)
            ob.linear_into(act, x, Wgu, epilogue="swiglu")
            ob.linear_into(h, act, Wd, epilogue="residual", residual=h)
            ob.linear_into(logits, h, Wlm, epilogue="f32")

        def cublas():
            F.linear(x, Wqkv, out=qkv)
            hh = h0 + F.linear(attn, Wo)
            gu = F.linear(x, Wgu).view(m, IM_ // 64, 2, 64)
            a_ = (F.silu(gu[:, :, 0].float()) * gu[:, :, 1].float()).half()
            hh = hh + F.linear(a_.reshape(m, IM_), Wd)
            logits.copy_(F.linear(hh, Wlm).float())

        ms = _graph_ms(ours, reps)
        ob.device_check()
        cms = _graph_ms(cublas, reps)
        a_bytes = 2 * m * (H_ + QKV_ + 4 * H_ + H_ + 2 * IM_ + H_) + 4 * m * V_
        total = w_layer + w_head + a_bytes
        gbs = total / (ms / 1e3) / 1e9
        out["by_tokens"][str(m)] = {
            "ms_per_step": round(ms, 4), "gbs": round(gbs, 1), "hbm_frac": round(gbs / hbm, 4),
            "cublas_ms_per_step": round(cms, 4),
            "cublas_gbs": round(total / (cms / 1e3) / 1e9, 1),
            "plans": {"qkv": ob_plan(m, QKV_, H_, "none"),
                      "gate_up": ob_plan(m, IM_, H_, "swiglu"),
                      "lm_head": ob_plan(m, V_, H_, "f32")}}
        del x, attn, h0, h, qkv, act, logits
    del Wqkv, Wo, Wgu, Wd, Wlm
    torch.cuda.empty_cache()
    return out


L3_M, L3_H, L3_IM, L3_HEADS, L3_KV, L3_HD = 4096, 4096, 14336, 32, 8, 128
L3_FLOPS = 2 * L3_M * ((L3_HEADS + 2 * L3_KV) * L3_HD * L3_H + L3_H * L3_H + 2 * L3_IM * L3_H
                       + L3_H * L3_IM)  # 1786.7 GFLOP


def llama3_tp_layer(rank: int, world: int, dev, comm, reps: int) -> dict:
    """Llama-3-8B-shaped decoder layer projections at prefill M=4096, tensor
    parallel over the job's GPUs: q/k/v column-parallel by heads (32/N query,
    8/N KV heads per rank), gate/up by intermediate feature, o_proj and
    down_proj row-parallel with the cross-GPU reduction, residual and SwiGLU
    fused as in the TinyLlama step.  Each rank draws its own random-init shard
    (the shapes are what a sharded checkpoint would give), rotated over enough
    copies to exceed L2.  1786.7 GFLOP per step for the whole job."""
    import math

    import orininfer_b200 as ob

    gen = torch.Generator(device=dev)
    gen.manual_seed(77 + rank)

    def w(r, c):
        return (torch.randn((r, c), generator=gen, device=dev) * 0.02).half()

    qkv_rows = (L3_HEADS // world + 2 * max(1, L3_KV // world)) * L3_HD
    im_l = L3_IM // world
    per_rank = 2 * (qkv_rows * L3_H + L3_H * (L3_H // world) + 2 * im_l * L3_H + L3_H * im_l)
    copies = max(1, min(4, math.ceil(300e6 / per_rank)))
    layers = [dict(qkv=w(qkv_rows, L3_H), o=w(L3_H, L3_H // world), gu=w(2 * im_l, L3_H),
                   d=w(L3_H, im_l)) for _ in range(copies)]
    x = w(L3_M, L3_H) * 50          # ~N(0,1) activations
    attn = w(L3_M, L3_H // world) * 50
    res = w(L3_M, L3_H) * 50
    qkv = torch.empty((L3_M, qkv_rows), dtype=torch.float16, device=dev)
    x1 = torch.empty((L3_M, L3_H), dtype=torch.float16, device=dev)
    act = torch.empty((L3_M, im_l), dtype=torch.float16, device=dev)
    x2 = torch.empty((L3_M, L3_H), dtype=torch.float16, device=dev)
    part = torch.empty((L3_M, L3_H), dtype=torch.float32, device=dev) if world > 1 else None

    def run(i):
        L = layers[i % copies]
        ob.linear_into(qkv, x, L["qkv"])
        if world == 1:
            ob.linear_into(x1, attn, L["o"], epilogue="residual", residual=res)
        else:
            comm.linear_row(attn, L["o"], residual=res, out=x1, partial=part)
        ob.linear_into(act, x, L["gu"], epilogue="swiglu")
        if world == 1:
            ob.linear_into(x2, act, L["d"], epilogue="residual", residual=x1)
        else:
            comm.linear_row(act, L["d"], residual=x1, out=x2, partial=part)

    run(0)
    torch.cuda.synchronize()
    n = 20
    g = torch.cuda.CUDAGraph()
    cs = torch.cuda.Stream()
    cs.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(cs):
        with torch.cuda.graph(g, stream=cs):
            for i in range(n):
                run(i)
    torch.cuda.current_stream().wait_stream(cs)
    g.replay()
    torch.cuda.synchronize()
    barrier(world)
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(a.elapsed_time(b) / (reps * n), world)
    del g
    ob.device_check()
    peaks, src = load_peaks()
    peak = peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])
    job = L3_FLOPS / (ms / 1e3) / 1e12
    return {"workload": "llama3_8b_layer_prefill_m4096", "tp": world, "ms_per_step": round(ms, 4),
            "tflops": round(job, 1), "tflops_per_gpu": round(job / world, 1),
            "frac_of_peak_per_gpu": round(job / world / peak, 4),
            "peak": f"{peak} TFLOP/s dense bf16 burst ({src})", "flops_per_step": L3_FLOPS,
            "steps": reps * n, "weight_copies": copies}


def cpu_baseline_layer(budget_s: float = 10.0) -> dict:
    """The oracle's fp32 multithreaded GEMM over the same layer shapes."""
    import numpy as np
    from oracle import oracle as orc

    threads = orc.max_threads()
    rng = np.random.default_rng(0)
    mats = {}
    for k, (n_out, kk, epi) in GEMMS.items():
        n_w = 2 * n_out if epi == "swiglu" else n_out
        mats[k] = (rng.standard_normal((M, kk), dtype=np.float32),
                   (rng.standard_normal((n_w, kk), dtype=np.float32) * 0.02))
    for k, (a, w) in mats.items():  # warm (thread pool, page faults)
        orc.gemm_f32(a[:8], w, threads)
    reps, t0 = 0, time.perf_counter()
    while True:
        for k, (a, w) in mats.items():
            orc.gemm_f32(a, w, threads)
        reps += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = time.perf_counter() - t0
    return {"value": STEP_FLOPS * reps / dt / 1e12, "unit": "TFLOP/s", "cores": threads,
            "kind": "port",
            "sample": f"{reps} full layer passes (4 fp32 GEMMs at M=512, oracle orc_gemm_f32), "
                      f"{dt:.1f} s"}


def ob_plan(M_, N_, K_, epi, workspace_bytes=0):
    import orininfer_b200 as ob
    p = ob.kernels.plan_info(M_, N_, K_, torch.float16, epi, workspace_bytes=workspace_bytes)
    sched = "stream-K" if p["stream_k"] else f"split{p['split_k']}"
    return (f"{p['kernel']} {'pair ' if p['cta_pair'] else ''}{p['tile_cols']}-wide {sched} "
            f"grid{p['grid']}")


def run_ours(args, rank, world, local_rank):
    import orininfer_b200  # noqa: F401  (fails loudly if the CUDA library is missing)
    from orininfer_b200 import tp

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    comm = None
    if world > 1:
        uid = tp.exchange_unique_id(rank)
        comm = tp.TPComm(rank, world, local_rank, uid, timeout_s=120.0)
        if not args.nccl_reduce:
            # o/down partial sums reduced over NVLink peer memory (falls back
            # to ncclAllReduce only where a call does not fit)
            comm.enable_p2p(max(M * H, L3_M * L3_H))
    layers = make_layers(rank, world, dev)
    step = Step(layers, rank, world, dev, comm, use_workspace=not args.no_workspace)

    ms, clocks = time_steps(step, args.steps, args.warmup, world, local_rank)
    ms_per_step = ms / args.steps
    value = STEP_FLOPS * args.steps / (ms / 1e3) / 1e12

    kt = kernel_breakdown(step, args.breakdown_steps) if world == 1 else None
    parity = parity_report(step) if world == 1 else None
    bar = cublas_bar(step, args.steps) if world == 1 and args.cublas_bar else None
    e2e_steps = max(1, min(args.steps, args.e2e_steps))
    e2e_ms, h2d, d2h = e2e_through_abi(step, e2e_steps, dev)
    e2e_ms = max_over_ranks(e2e_ms, world)
    e2e_value = STEP_FLOPS * e2e_steps / (e2e_ms / 1e3) / 1e12

    peaks, src = load_peaks()
    line = {
        "metric": "prefill GEMM throughput (TinyLlama layer q/k/v+o+gate/up+down, M=512)",
        "value": round(value, 2),
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 5),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f16",
        "data": "synthetic (seeded N(0,1) activations, N(0,0.02) random-init weights)",
        "config": {"workload": WORKLOAD, "M": M, "hidden": H, "intermediate": IM,
                   "q_heads": N_HEADS, "kv_heads": N_KV, "head_dim": HEAD_DIM,
                   "flops_per_step": STEP_FLOPS,
                   "parallelism": "tp%d" % world if world > 1 else "single",
                   "tp_reduce": ("nccl" if args.nccl_reduce else "nvlink-p2p") if world > 1
                   else None,
                   "gemm_workspace_bytes": step.ws.numel() if step.ws is not None else 0,
                   "l2": f"inputs larger than L2: {N_COPIES} rotating layer copies "
                         f"({N_COPIES * 88} MB of weights)"},
        "e2e": {"value": round(e2e_value, 3), "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": e2e_steps,
                "path": "orininfer_b200.linear_into -> orin_linear_ex (C ABI), pinned host "
                        "inputs copied in and the layer output copied out every step, "
                        "copies on their own streams overlapping the neighbouring steps"},
        "gpu_launches": step.launches * args.steps,
        "clocks": clocks,
    }
    if parity:
        line["parity"] = parity
    if kt is not None:
        dom = "gate_up"
        avg_ms = kt[dom]
        achieved = FLOPS[dom] / (avg_ms / 1e3) / 1e12
        peak = peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])
        line["roofline"] = {
            "kernel": "tc_linear_kernel<f16,256,SWIGLU> (gate/up + SwiGLU, 512x11264x2048)",
            "bound": "tensor", "achieved": round(achieved, 2), "peak": peak,
            "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
            "peak_source": f"{src} dense bf16 burst (MEASURED_PEAKS.json bf16_tflops)"
            if src == "measured" else "fallback 1590 TFLOP/s",
            "traffic": profile_traffic("gate_up"),
            "algorithmic_flops_per_launch": FLOPS[dom],
            "avg_launch_ms": round(avg_ms, 5),
        }
        line["kernels_ms"] = {k: round(v, 5) for k, v in kt.items()}
        wsb = step.ws.numel() if step.ws is not None else 0
        line["kernels_plan"] = {
            k: ob_plan(M, n, kk, epi, wsb) for k, (n, kk, epi) in GEMMS.items()}
        if bar is not None:
            line["cublas_bar"] = bar
        line["kernels_tflops"] = {k: round(FLOPS[k] / (kt[k] / 1e3) / 1e12, 1) for k in kt}
        line["cpu_baseline"] = cpu_baseline_layer(args.cpu_budget) if args.cpu_budget > 0 \
            else None
        if args.decode_reps > 0:
            line["decode"] = decode_path(dev, args.decode_reps, args.cublas_bar)
            line["single_linear_m1"] = single_linear_m1(dev, args.decode_reps)
            line["llama3_decode"] = llama3_decode(dev, args.decode_reps)
        if args.model_decode_reps > 0:
            # the whole model's greedy decode step; reported beside the layer
            # line, which stands on its own if this part fails
            for key, batch in (("model_decode", 1), ("model_decode_b16", 16)):
                try:
                    line[key] = run_model_decode(
                        argparse.Namespace(model_decode=args.model_decode_reps, warmup=5,
                                           batch=batch))
                except Exception as e:  # noqa: BLE001
                    line[key] = {"error": f"{type(e).__name__}: {e}"}
                torch.cuda.empty_cache()
    if args.llama3_reps > 0:
        line["llama3_tp"] = llama3_tp_layer(rank, world, dev, comm, args.llama3_reps)
    if comm is not None:
        torch.cuda.synchronize()
        comm.close()
    return line


# prefill attention calls timed by --attention: (new tokens, cached positions
# after the call, query heads, KV heads, head dim), n_sink 4, W 1024
ATTN_SHAPES = [(1028, 1028, 32, 4, 64), (1020, 2048, 32, 4, 64), (1028, 1028, 32, 8, 128),
               (300, 300, 32, 8, 128), (512, 512, 32, 4, 64), (256, 2048, 32, 4, 64),
               (128, 1028, 32, 4, 64), (64, 2048, 32, 4, 64), (32, 2048, 32, 4, 64)]


def run_attention(args):
    """Prefill attention alone (sink + sliding-window GQA over the ring pools),
    one call per shape of ATTN_SHAPES, random bf16 inputs: the average of
    --attention back-to-back calls after --warmup, CUDA events on the
    launching stream.  The kernel is the launcher's choice unless the
    ORIN_ATTN_KERNEL tuning override (mma, tc1, tc2) forces one.  Inputs fit
    in L2 (a few MB): these are kernel times, not HBM-cold ones."""
    from orininfer_b200 import kernels as K

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    n_sink, window = 4, 1024
    res = {"kernel": os.environ.get("ORIN_ATTN_KERNEL", "auto"), "dtype": "bf16",
           "n_sink": n_sink, "window": window, "calls": args.attention, "shapes": {}}
    gen = torch.Generator(device=dev)
    gen.manual_seed(0)
    ws = torch.zeros(64 << 20, dtype=torch.uint8, device=dev)  # arrival counters start zero
    for (s_len, c_len, nh, nkv, hd) in ATTN_SHAPES:
        q = torch.randn((s_len, nh, hd), generator=gen, device=dev).to(torch.bfloat16)
        kp = torch.randn((n_sink + window, nkv, hd), generator=gen, device=dev).to(torch.bfloat16)
        vp = torch.randn((n_sink + window, nkv, hd), generator=gen, device=dev).to(torch.bfloat16)
        out = torch.empty_like(q)

        def call():
            K.attention(out, q, kp, vp, s_len, c_len, nh, nkv, hd, hd ** -0.5, n_sink, window,
                        workspace=ws)

        for _ in range(args.warmup):
            call()
        K.device_check()
        torch.cuda.synchronize()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.attention):
            call()
        b.record()
        b.synchronize()
        K.device_check()
        us = a.elapsed_time(b) / args.attention * 1e3
        # 4 flops per (query head, attended key, head dim element): S and P V
        base = c_len - s_len
        pairs = sum(min(base + i + 1, n_sink + window) for i in range(s_len))
        res["shapes"][f"{s_len}x{c_len}_h{nh}/{nkv}x{hd}"] = {
            "us": round(us, 2), "tflops": round(4 * pairs * nh * hd / (us * 1e-6) / 1e12, 1)}
    return res


def run_one_kernel(args):
    """One projection of the layer, eagerly: a bounded case for profilers."""
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    layers = make_layers(0, 1, dev)
    step = Step(layers, 0, 1, dev)
    name = args.kernel
    ob = step.ob
    m = args.tokens if args.tokens is not None else M
    if not 1 <= m <= M:
        raise SystemExit(f"--tokens must be in [1, {M}]")

    def rows(t):
        return t[:m]  # leading rows of a row-major buffer: still contiguous

    def launch(i):
        L = layers[i % len(layers)]
        if name == "qkv":
            ob.linear_into(rows(step.qkv), rows(step.h), L["qkv"])
        elif name == "o_proj":
            ob.linear_into(rows(step.x1), rows(step.attn), L["o_proj"], epilogue="residual",
                           residual=rows(step.x))
        elif name == "gate_up":
            ob.linear_into(rows(step.act), rows(step.h2), L["gate_up"], epilogue="swiglu")
        else:
            ob.linear_into(rows(step.x2), rows(step.act), L["down"], epilogue="residual",
                           residual=rows(step.x1))

    for i in range(args.warmup):
        launch(i)
    torch.cuda.synchronize()
    ts = []
    for i in range(args.steps):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        launch(args.warmup + i)
        b.record()
        b.synchronize()
        ts.append(a.elapsed_time(b))
    ob.device_check()
    avg = statistics.mean(ts)
    n_out, kk, epi = GEMMS[name]
    n_w = 2 * n_out if epi == "swiglu" else n_out
    flops = FLOPS[name] * m // M
    # algorithmic bytes: weight + activation read, output written (+ residual read)
    nbytes = 2 * (n_w * kk + m * kk + m * n_out * (2 if epi == "residual" else 1))
    return {"kernel": name, "workload": WORKLOAD, "tokens": m, "launches": args.steps,
            "avg_ms": round(avg, 5), "tflops": round(flops / (avg / 1e3) / 1e12, 2),
            "gbs": round(nbytes / (avg / 1e3) / 1e9, 1), "algorithmic_bytes": nbytes,
            "plan": ob_plan(m, n_out, kk, epi)}


def run_model_decode(args) -> dict:
    """Greedy generation through the whole model:
    a 22-layer TinyLlama-shaped model (seeded random-init fp16 weights made on
    the device, 2.07 GB), sink + window KV cache (4 + 1024) per sequence,
    `args.batch` (default 1) 2048-token prompts, each prefilled in the
    reference's chunks of n_sink + W = 1028 and 1020 tokens, then one decode
    step of all sequences (embedding, 22 x the layer's seven launches with RoPE
    and the K/V append in the q/k/v epilogue (six with fold_norm), final
    norm, LM head + argmax, the tokens fed back on
    the device; the batch shares each weight stream) captured in a CUDA graph
    at position 2048 (a full window) and replayed `args.model_decode` times.
    Every replay does a full step's work: the same ring slot is rewritten and
    the same 1028 positions are attended.  tokens/s = batch / step time."""
    from orininfer_b200 import weights as Wt
    from orininfer_b200.layer import Decoder

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = dict(Wt.TINYLLAMA)
    gen = torch.Generator(device=dev)
    gen.manual_seed(2024)
    tensors = {}
    for name in Wt.reference_tensor_names(cfg["num_hidden_layers"]):
        if name.endswith("norm.weight"):
            dim = cfg["head_dim"] if ("q_norm" in name or "k_norm" in name) else cfg["hidden_size"]
            tensors[name] = torch.ones(dim, dtype=torch.float16, device=dev)
            continue
        shape = {"embed_tokens": (cfg["vocab_size"], H), "lm_head": (cfg["vocab_size"], H),
                 "q_proj": (H, H), "k_proj": (KVD, H), "v_proj": (KVD, H), "o_proj": (H, H),
                 "gate_proj": (IM, H), "up_proj": (IM, H), "down_proj": (H, IM)}
        key = next(k for k in shape if k in name)
        tensors[name] = (torch.randn(shape[key], generator=gen, device=dev) * 0.02).half()
    n_sink, window = 4, 1024
    B = int(getattr(args, "batch", 1))
    fold = bool(getattr(args, "fold_norm", False))
    model = Decoder(tensors, cfg, dev, n_sink=n_sink, window=window, max_tokens=n_sink + window,
                    batch=B, fold_norm=fold)
    del tensors
    prompts = [torch.randint(0, cfg["vocab_size"], (2048,), generator=gen, device=dev,
                             dtype=torch.int32) for _ in range(B)]
    # prefill of every sequence (eager launches), timed with events
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for seq, prompt in enumerate(prompts):
        model.step(prompt[:1028], 0, seq=seq)
        model.step(prompt[1028:], 1028, seq=seq)
    b.record()
    torch.cuda.synchronize()
    prefill_ms = a.elapsed_time(b)
    ids = model.tokens.clone()
    pos = 2048

    def decode():
        if B == 1:
            model.step(ids, pos)
        else:
            model.step_batch(ids, pos)
        ids.copy_(model.tokens)

    # eager step (host launch cost included)
    for _ in range(3):
        decode()
    torch.cuda.synchronize()
    a.record()
    for _ in range(10):
        decode()
    b.record()
    torch.cuda.synchronize()
    eager_ms = a.elapsed_time(b) / 10
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            decode()
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(max(3, args.warmup)):
        g.replay()
    torch.cuda.synchronize()
    a.record()
    for _ in range(args.model_decode):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / args.model_decode
    import orininfer_b200 as ob
    ob.device_check()
    del g
    L = cfg["num_hidden_layers"]
    w_bytes = 2 * (L * ((H + 2 * KVD) * H + H * H + 2 * IM * H + H * IM) + cfg["vocab_size"] * H)
    kv_bytes = L * 2 * (n_sink + window) * KVD * 2
    peaks, _ = load_peaks()
    hbm = peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])
    kv_bytes *= B
    gbs = (w_bytes + kv_bytes) / (ms / 1e3) / 1e9
    return {"metric": f"greedy decode tokens/s, 22-layer TinyLlama, batch {B}, "
                      "1028-position window",
            "value": round(B * 1e3 / ms, 1), "unit": "tokens/s", "batch": B,
            "ms_per_step": round(ms, 4), "ms_per_token": round(ms / B, 4),
            "eager_ms_per_step": round(eager_ms, 4),
            "prefill_ms_2048_tokens": round(prefill_ms / B, 3),
            "prefill_tokens_per_s": round(B * 2048 / (prefill_ms / 1e3), 1),
            "bytes_per_step": w_bytes + kv_bytes, "gbs": round(gbs, 1),
            "hbm_frac": round(gbs / hbm, 4), "peak_hbm_gbs": hbm,
            # per layer: norm, q/k/v, RoPE + append, attention (its key splits
            # merged by the last split CTA), o_proj, norm, gate/up, down; then
            # embedding, final norm, LM head (key reset, weight stream,
            # decode), token copy
            "launches_per_step": L * (6 if fold else 7) + (5 if fold else 6),
            "steps": args.model_decode,
            "dtype": "f16", "data": "synthetic (seeded random-init weights, random prompt)",
            "config": {"workload": "tinyllama_22l_greedy_decode", "n_sink": n_sink,
                       "window": window, "prompt": 2048, "batch": B, "graph": True,
                       "fold_norm": fold}}


# ---------------------------------------------------------------------------- reference arm

def run_reference(args):
    """The CPU oracle (the reference has no CPU path of its own) on the same
    layer: each step computes a bounded slice of the layer's token rows through
    all four GEMMs in fp32 with every host thread."""
    import numpy as np
    from oracle import oracle as orc

    threads = orc.max_threads()
    rng = np.random.default_rng(0)
    mats = {}
    for k, (n_out, kk, epi) in GEMMS.items():
        n_w = 2 * n_out if epi == "swiglu" else n_out
        mats[k] = (rng.standard_normal((M, kk), dtype=np.float32),
                   rng.standard_normal((n_w, kk), dtype=np.float32) * 0.02)
    # size the row slice so warmup + steps fit in about 90 s of CPU time
    t0 = time.perf_counter()
    for k, (a, w) in mats.items():
        orc.gemm_f32(a[:64], w, threads)
    per_row = (time.perf_counter() - t0) / 64
    budget = 90.0 / max(1, args.steps + args.warmup)
    rows = int(max(4, min(M, (budget / per_row) // 4 * 4)))
    flops_per_step = STEP_FLOPS * rows / M

    def step(i):
        r0 = (i * rows) % M
        r1 = min(M, r0 + rows)
        for k, (a, w) in mats.items():
            orc.gemm_f32(a[r0:r1], w, threads)
        return (r1 - r0)

    for i in range(args.warmup):
        step(i)
    done_rows = 0
    t0 = time.perf_counter()
    for i in range(args.steps):
        done_rows += step(i)
    dt = time.perf_counter() - t0
    value = STEP_FLOPS * (done_rows / M) / dt / 1e12
    sample = (f"{rows} of the {M} token rows per step through all four projections "
              f"(fp32, oracle orc_gemm_f32, {threads} threads)")
    return {
        "impl": "reference",
        "metric": "prefill GEMM throughput (TinyLlama layer q/k/v+o+gate/up+down, M=512)",
        "value": round(value, 4),
        "unit": "TFLOP/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(dt / args.steps * 1e3, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded N(0,1) activations, N(0,0.02) weights)",
        "config": {"workload": WORKLOAD, "M": M, "hidden": H, "intermediate": IM,
                   "flops_per_step": STEP_FLOPS, "parallelism": "host threads"},
        "cpu_baseline": {"value": round(value, 4), "unit": "TFLOP/s", "cores": threads,
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": "the reference runs this path only on a GPU (kernels/matmul.cu); its CPU "
                "counterpart here is the oracle's restatement of the same arithmetic",
    }


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-budget", type=float, default=10.0,
                    help="seconds of CPU work for the cpu_baseline figure (0: skip)")
    ap.add_argument("--e2e-steps", type=int, default=300,
                    help="steps of the end-to-end (host buffers, C ABI) measurement")
    ap.add_argument("--breakdown-steps", type=int, default=64,
                    help="steps of the per-projection CUDA-event breakdown")
    ap.add_argument("--decode-reps", type=int, default=20,
                    help="graph replays of the whole-model decode GEMM path per token count "
                         "(0: skip)")
    ap.add_argument("--llama3-reps", type=int, default=3,
                    help="graph replays (20 steps each) of the Llama-3-8B TP layer measurement "
                         "(0: skip)")
    ap.add_argument("--nccl-reduce", action="store_true",
                    help="N>1: reduce the row-parallel partial sums with ncclAllReduce instead "
                         "of the peer-memory kernels")
    ap.add_argument("--no-workspace", action="store_true",
                    help="run the projections without a GEMM workspace (no stream-K plans)")
    ap.add_argument("--no-cublas-bar", dest="cublas_bar", action="store_false",
                    help="skip timing the cuBLAS comparison bar")
    ap.add_argument("--kernel", choices=list(GEMMS), default=None,
                    help="run only this projection, eagerly, warmup+steps times, and print "
                         "its event-timed average (a small case for profilers)")
    ap.add_argument("--model-decode-reps", type=int, default=50,
                    help="graph replays of the whole-model greedy decode step reported as the "
                         "line's model_decode object (0: skip)")
    ap.add_argument("--model-decode", type=int, default=0,
                    help="instead of the layer bench: time this many graph-replayed greedy "
                         "decode steps of the whole 22-layer model (prefill of a 2048-token "
                         "prompt first) and print that line")
    ap.add_argument("--fold-norm", action="store_true",
                    help="with --model-decode: fold each RMSNorm into the projection after it")
    ap.add_argument("--batch", type=int, default=1,
                    help="with --model-decode: sequences decoded together (per-sequence KV "
                         "pools, one weight stream per step)")
    ap.add_argument("--attention", type=int, default=0,
                    help="instead of the layer bench: time this many back-to-back prefill "
                         "attention calls per shape (ORIN_ATTN_KERNEL forces a kernel) and "
                         "print that line")
    ap.add_argument("--tokens", type=int, default=None,
                    help="with --kernel: token rows M of that projection (default: the "
                         "workload's 512; 1..64 is the decode GEMV / skinny path)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.kernel is not None:
        print(json.dumps(run_one_kernel(args)), flush=True)
        return 0
    if args.model_decode > 0:
        print(json.dumps(run_model_decode(args)), flush=True)
        return 0
    if args.attention > 0:
        print(json.dumps(run_attention(args)), flush=True)
        return 0

    if args.impl == "reference":
        if rank != 0:
            return 0
        print(json.dumps(run_reference(args)), flush=True)
        return 0

    if world > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        line = run_ours(args, rank, world, local_rank)
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
