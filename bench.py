"""Benchmark: decoder-layer tokens/s on 1..N B200 GPUs, with per-kernel roofline fractions.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--no-suite]

Workload: one Llama-style decoder layer forward, f32, batch 1,
seq 128, hidden 512, 8 heads x 64, causal attention, RoPE theta 1e4, RMSNorm eps 1e-5,
SwiGLU ffn 1376, residual adds, weights N(0, 0.02), 128 token ids gathered from a 32000 x 512
table -- synthetic seeded data.  A step is one layer forward over the 128 tokens, driven
through the executor as the Runtime does and replayed as one captured CUDA graph.  With N
GPUs each rank runs its own replica (weak scaling; the layer is replicated, not sharded),
and the tensor-parallel SwiGLU MLP of configs[4] runs across all N ranks with one NCCL
all-reduce per MLP ("tp_mlp" in the JSON line).  Rank 0 prints one JSON line.

--impl reference times the reference's CPU path -- the C oracle restatement of its kernels,
since the reference's own CPU executor is a Rust crate that cannot be built here -- on all
host cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import faulthandler
import importlib
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
PACKAGE = "magnetar-provider-cuda_b200"
L2_BYTES = 126 * 1024 * 1024
PEAKS_PATH = os.path.join(ROOT, "MEASURED_PEAKS.json")
METRIC = "decoder-layer tokens/s"
UNIT = "tokens/s"


# ------------------------------------------------------------------------------------ helpers
def load_peaks():
    try:
        with open(PEAKS_PATH) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]),
                "bf16_tflops_sustained": float(p.get("bf16_tflops_sustained", p["bf16_tflops"])),
                "source": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """SM clock and clock-event (throttle) reasons of one GPU, polled through NVML every
    ~2 ms on a background thread while the timed region runs (read-only queries).  Falls back
    to ``nvidia-smi -lms 200`` when NVML is unavailable."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.sm, self.reasons, self.max_mhz = [], set(), None
        self.stop = threading.Event()
        self.thread = None
        self.proc = None
        self.lines = []

    def _nvml_handle(self):
        """The NVML handle of CUDA device ``self.gpu``, matched by PCI bus id (the CUDA and
        NVML orders can differ); by index when the id is unavailable."""
        import pynvml
        import torch
        pynvml.nvmlInit()

        def norm(bus):  # "0000:1B:00.0" / "00000000:1b:00.0" -> "1b:00.0"
            if isinstance(bus, bytes):
                bus = bus.decode()
            return str(bus).lower().split(":", 1)[-1] if str(bus).count(":") == 2 else str(bus).lower()

        props = torch.cuda.get_device_properties(self.gpu)
        bus, dev = getattr(props, "pci_bus_id", None), getattr(props, "pci_device_id", None)
        want = f"{bus:02x}:{dev:02x}.0" if isinstance(bus, int) and isinstance(dev, int) else norm(bus or "")
        if want:
            for i in range(pynvml.nvmlDeviceGetCount()):
                h = pynvml.nvmlDeviceGetHandleByIndex(i)
                if norm(pynvml.nvmlDeviceGetPciInfo(h).busId) == want:
                    return pynvml, h
        return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.gpu)

    def _poll(self, nv, h):
        flags = [(name, getattr(nv, attr, 0)) for name, attr in self.REASONS]
        while not self.stop.is_set():
            try:
                self.sm.append(float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)))
                active = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                for name, bit in flags:
                    if bit and active & bit:
                        self.reasons.add(name)
            except Exception:
                return
            self.stop.wait(0.002)

    def __enter__(self):
        try:
            nv, h = self._nvml_handle()
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            self.thread = threading.Thread(target=self._poll, args=(nv, h), daemon=True)
            self.thread.start()
        except Exception:
            try:
                self.proc = subprocess.Popen(
                    ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                     "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
                self.thread = threading.Thread(target=self._read_smi, daemon=True)
                self.thread.start()
            except Exception:
                self.proc = None
        return self

    def _read_smi(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                self.sm.append(float(parts[1]))
                self.max_mhz = float(parts[2])
            except ValueError:
                continue
            for (name, _), val in zip(self.REASONS, parts[5:9]):
                if val.lower() == "active":
                    self.reasons.add(name)

    def __exit__(self, *exc):
        self.stop.set()
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=5)

    def summary(self):
        return {"sm_mhz": statistics.median(self.sm) if self.sm else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.sm),
                "source": "nvml" if self.proc is None else "nvidia-smi"}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# ------------------------------------------------------------------------------------ reference arm
def oracle_layer(orc, cfg, w):
    x, _ = orc.embedding(w["table"], w["ids"])
    h = orc.rmsnorm(x, w["attn_norm"], cfg.eps)
    q, k, v = (orc.matmul(h, w[n]) for n in ("wq", "wk", "wv"))
    q = orc.rope(q, base=cfg.rope_theta, dimension=cfg.head_dim, head_count=cfg.heads)
    k = orc.rope(k, base=cfg.rope_theta, dimension=cfg.head_dim, head_count=cfg.heads)
    a = orc.attention(q, k, v, cfg.heads, cfg.head_dim, causal=True)
    x2 = orc.matmul(a, w["wo"], addend=x, addend_mode=2)
    h2 = orc.rmsnorm(x2, w["mlp_norm"], cfg.eps)
    return orc.matmul(orc.gated_matmul(h2, w["wg"], w["wu"]), w["wd"], addend=x2, addend_mode=2)


def cpu_layer_rate(cfg, w, budget_s: float, threads: int = 0):
    """Decoder-layer tokens/s of the oracle on the host cores over a bounded sample."""
    from oracle import oracle as orc
    if threads:
        orc.set_threads(threads)
    oracle_layer(orc, cfg, w)  # warm
    t0 = time.perf_counter()
    n = 0
    while True:
        oracle_layer(orc, cfg, w)
        n += 1
        el = time.perf_counter() - t0
        if el >= budget_s or n >= 1000:
            break
    return cfg.seq * n / el, n, orc.threads()


def bench_config(world: int) -> dict:
    """The ``config`` object both arms print (the same workload on the same inputs)."""
    return {"workload": "decoder-layer b1 s128 h512 8x64 ffn1376 causal, RoPE 1e4, RMSNorm 1e-5 (configs[0]); "
                        "one step = one layer forward over 128 tokens (layer.make_inputs seed 0 on rank 0)",
            "global_batch": world, "seq_len": 128, "parallelism": f"replicas x{world}",
            "l2": "flushed before every timed GPU step: 252 MB write, then 252 MB read of another buffer"}


def run_reference(args, world, rank):
    if rank != 0:
        return
    layer = importlib.import_module(PACKAGE + ".layer")
    cfg = layer.DecoderLayerConfig()
    w = layer.make_inputs(cfg, seed=0)
    from oracle import oracle as orc
    orc.build()
    per_step = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        oracle_layer(orc, cfg, w)
        if i >= args.warmup:
            per_step.append(time.perf_counter() - t0)
    total = sum(per_step)
    value = cfg.seq * args.steps / total
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": bench_config(world),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": orc.threads(), "kind": "port",
                         "sample": f"{args.steps} full layer forwards on the host cores (C oracle, OpenMP); the "
                                   "reference CPU executor (Rust providers-cpu) is not buildable here"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------ our arm
def gpu_busy(torch, us: float = 200.0):
    """Keeps the stream busy for about `us` microseconds (a spin kernel), so that the host
    has enqueued the timed work before the start event executes: the events then bracket
    device time only, not the host's launch latency."""
    torch.cuda._sleep(int(us * 2000))  # ~2 GHz cycles


def make_l2_flush(torch):
    """L2 flush between timed iterations: write a buffer twice the L2's size, then read
    another one of that size.  The read evicts the dirty lines the write left (their
    write-back happens here, outside the timed region), so the timed kernel starts with no
    input in L2 and no foreign dirty line to write back -- the state ncu's cache control
    gives a profiled kernel."""
    wr = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device="cuda")
    rd = torch.zeros(2 * L2_BYTES // 4, dtype=torch.float32, device="cuda")

    def flush():
        wr.zero_()
        rd.sum()

    return flush


def time_events(torch, fn, iters, flush=None, warmup=2, reps=1, busy_us=200.0):
    """Device time (ms) of one call of ``fn`` on the current stream, per iteration: the L2 is
    flushed before each iteration, which then runs ``fn`` ``reps`` times back to back between
    two events (``reps`` > 1 only for inputs larger than the L2).  An event pair with nothing
    between it reads ~2.7 us on a B200 (the clock itself ticks in 32 ns), so a single short
    call reads long by about that much; ``reps`` spreads it."""
    for _ in range(warmup):
        fn()
    times = []
    for _ in range(iters):
        if flush is not None:
            flush()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        gpu_busy(torch, busy_us)
        s.record()
        for _ in range(reps):
            fn()
        e.record()
        e.synchronize()
        times.append(s.elapsed_time(e) / reps)
    return times


def robust_mean(xs):
    """Mean of the middle 60% of the samples: robust to an outlier iteration."""
    xs = sorted(xs)
    cut = int(len(xs) * 0.2)
    mid = xs[cut:len(xs) - cut] or xs
    return sum(mid) / len(mid)


def measure_tf32_peak(torch):
    """cuBLAS f32 GEMM with TF32 tensor cores, 8192^3: the TF32 denominator (burst)."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    try:
        a = torch.randn(8192, 8192, device="cuda")
        b = torch.randn(8192, 8192, device="cuda")
        t = min(time_events(torch, lambda: torch.matmul(a, b), 5, warmup=2))
        return 2 * 8192 ** 3 / (t * 1e-3) / 1e12
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


EXACT_MS = (1, 16, 128, 2048)  # the matmul lines also timed with bfloat16-exact weights
Q8_MS = (1, 16)  # and with packed Q8_0 weights (the few-row path reads them packed)
ROT_COPIES = 6  # copies of the 64 MB B the M <= 128 lines rotate through (384 MB > the 126 MB L2)
NODE_COPIES = 8  # instances of a layer node per timed step (per-node times)


def kernel_suite(torch, mpc, kernels, peaks, tf32_tflops, filt=None, iters=5):
    """Configs 2-4: each kernel timed alone with CUDA events, as % of its roofline.  The L2 is
    flushed before every timed iteration; the memory-bound cases, whose inputs are larger than
    the L2, time 10 (softmax: 3) back-to-back launches per iteration, the matmul lines with
    M <= 128 one call on each of ROT_COPIES copies of B, the rest one launch.  Times are the
    mean of the middle 60% of at least 10 iterations.  ``filt`` keeps only the cases whose name contains it."""
    results = []
    flush = make_l2_flush(torch)

    def want(name):
        return filt is None or filt in name

    hbm = peaks["hbm_gbs"]
    eff = tf32_tflops / 3.0 if tf32_tflops > 0 else float("nan")

    def add(name, config, ms, bound, work, bf16x3=False):
        # compact entries: [name, ms, achieved, frac] -- achieved in GB/s (bound hbm, peak = the
        # measured copy bandwidth) or TFLOP/s (bound tensor, peak = 3xTF32-effective); the
        # attention line adds its fraction of bf16x3-effective (measured bf16 / 3)
        if bound == "hbm":
            achieved = work / (ms * 1e-3) / 1e9
            results.append([name, round(ms, 4), round(achieved, 1), round(achieved / hbm, 3)])
        else:
            achieved = work / (ms * 1e-3) / 1e12
            results.append([name, round(ms, 4), round(achieved, 1), round(achieved / eff, 3)])
            if bf16x3:  # the kernel issues three bf16 MMAs per product: its own ceiling
                results[-1].append(round(achieved / (peaks["bf16_tflops"] / 3.0), 3))

    def timed(fn, n=iters, warmup=2, reps=1):
        # the spin covers the host's enqueueing of all `reps` calls
        return robust_mean(time_events(torch, fn, max(n, 10), flush, warmup=warmup, reps=reps, busy_us=200.0 * reps))

    g = torch.Generator(device="cuda")
    g.manual_seed(0)
    W = kernels.wrap_tensor

    # config 2: f32 matmul sweep, N = K = 4096
    K = N = 4096
    # B as a model weight (written with write_weight_tensor: its tensor-core operand form is
    # built once and kept with it), and B as a plain tensor (operand form derived per call).
    if any(want(f"matmul M={M}") for M in (1, 16, 128, 2048, 8192)):
        b = torch.randn(K, N, device="cuda", generator=g) / math.sqrt(K)
        # Lines with M <= 128 (a call of a few tens of microseconds, B read once) run
        # ROT_COPIES back-to-back calls per event pair, each on its own copy of B, as the
        # layers of a model follow one another: every call streams its B from HBM (the copies
        # together are larger than the L2) and the event pair's fixed cost is spread.  Larger
        # M times one call on one B.
        copies = [b] + [b.clone() for _ in range(ROT_COPIES - 1)]
        rot = {"": [W(x).set_weight() for x in copies], " (B per-call)": [W(x) for x in copies]}
        if any(want(f"matmul M={M} (bf16-exact weight)") for M in EXACT_MS):
            # the same weights rounded to bfloat16 values (a bfloat16 checkpoint's): the GEMV
            # streams their compact bfloat16 form, and their prepared lo term is zero, so the
            # GEMM reads hi alone
            exact = [(x.view(torch.int32) & -65536).view(torch.float32) for x in copies]
            rot[" (bf16-exact weight)"] = [W(x).set_weight() for x in exact]
        if any(want(f"matmul M={M} (Q8_0 weight)") for M in Q8_MS):
            # packed Q8_0 weights (a checkpoint's [N, K] storage read as B [K, N]): seeded f16
            # scales between 2^-9 and 2^-5 and quants over -127..127
            rq = np.random.default_rng(5)
            nb = N * K // 32
            q8 = []
            for _ in range(ROT_COPIES):
                blk = np.empty((nb, 34), np.uint8)
                blk[:, :2] = rq.uniform(2.0 ** -9, 2.0 ** -5, nb).astype(np.float16).view(np.uint8).reshape(nb, 2)
                blk[:, 2:] = rq.integers(-127, 128, (nb, 32), dtype=np.int8).view(np.uint8)
                q8.append(kernels.upload_q8_0(blk, N, K, transposed=True))
            rot[" (Q8_0 weight)"] = q8
        for M in (1, 16, 128, 2048, 8192):
            if not want(f"matmul M={M}"):
                continue
            a = torch.randn(M, K, device="cuda", generator=g) / math.sqrt(K)
            c = torch.empty(M, N, device="cuda")
            da, dc = W(a), W(c)
            for label in ("", " (B per-call)", " (bf16-exact weight)", " (Q8_0 weight)"):
                exact = label == " (bf16-exact weight)"
                packed = label == " (Q8_0 weight)"
                if M <= 16 and label == " (B per-call)":
                    continue  # the GEMV path reads B as it is either way
                if label not in rot or (exact and M not in EXACT_MS) or (packed and M not in Q8_MS):
                    continue
                bufs = rot[label]
                if M <= 128:
                    turn = [0]

                    def call():
                        kernels.matmul(da, bufs[turn[0] % ROT_COPIES], out=dc)
                        turn[0] += 1

                    for _ in range(ROT_COPIES):  # builds each copy's prepared form (weights)
                        call()
                    ms = timed(call, n=max(iters, 15), reps=ROT_COPIES)
                else:
                    ms = timed(lambda: kernels.matmul(da, bufs[0], out=dc), n=iters)
                if M <= 16:  # B's bytes: 4 per value, 2 in the compact form, 1.125 packed (quant + f32 scale / 32)
                    add(f"matmul M={M}{label}", "configs[1]", ms, "hbm",
                        4.0 * (M * K + M * N) + (2.0 if exact else 1.125 if packed else 4.0) * K * N)
                else:
                    add(f"matmul M={M}{label}", "configs[1]", ms, "tensor", 2.0 * M * N * K)
            del a, c
        del b, copies, rot
        # the M = 8192 GEMMs run at the power cap: let the clocks recover before the next lines,
        # which are timed as kernels on their own
        torch.cuda.synchronize()
        time.sleep(2.0)
    # config 3: causal attention b4 h32 d128 s2048 (batch folded into 128 heads)
    S, H, D = 2048, 4 * 32, 128
    name = "attention causal b4 h32 d128 s2048"
    if want(name):
        q = torch.randn(S, H * D, device="cuda", generator=g)
        k_ = torch.randn(S, H * D, device="cuda", generator=g)
        v = torch.randn(S, H * D, device="cuda", generator=g)
        o = torch.empty(S, H * D, device="cuda")
        dq, dk, dv, do = W(q), W(k_), W(v), W(o)
        ms = timed(lambda: kernels.attention(dq, dk, dv, H, D, causal=True, out=do), max(3, iters // 2), 1)
        add(name, "configs[2]", ms, "tensor", 4.0 * H * S * S * D / 2, bf16x3=True)
        del q, k_, v, o
    # decode (the "next" row): one query row over a 32768-key history, GQA 32 / 8 heads of 128;
    # bound by reading K and V once (268 MB, larger than the L2)
    S, H, KVH, D = 32768, 32, 8, 128
    name = "attention decode q1 h32 kvh8 d128 kv32768"
    if want(name):
        q = torch.randn(1, H * D, device="cuda", generator=g)
        k_ = torch.randn(S, KVH * D, device="cuda", generator=g)
        v = torch.randn(S, KVH * D, device="cuda", generator=g)
        o = torch.empty(1, H * D, device="cuda")
        dq, dk, dv, do = W(q), W(k_), W(v), W(o)
        ms = timed(lambda: kernels.attention(dq, dk, dv, H, D, kv_head_count=KVH, causal=True, out=do), reps=3)
        add(name, "decode", ms, "hbm", 4.0 * (2 * S * KVH * D + 2 * H * D))
        del q, k_, v, o
    # config 3': softmax rows [262144, 2048]
    name = "softmax [262144,2048]"
    if want(name):
        x = torch.randn(262144, 2048, device="cuda", generator=g) * 2
        y = torch.empty_like(x)
        dx, dy = W(x), W(y)
        ms = timed(lambda: kernels.softmax_rows(dx, out=dy), max(3, iters // 2), 1, reps=3)
        add(name, "configs[2]", ms, "hbm", 2.0 * x.numel() * 4)
        del x, y
    # config 4: memory-bound suite on [8192, 4096]
    R, C = 8192, 4096
    names = ["rmsnorm", "rope h32x128 theta5e5", "silu", "add", "mul", "residual-add", "gelu", "row-scale"]
    if any(want(f"{n} [8192,4096]") for n in names):
        x = torch.randn(R, C, device="cuda", generator=g)
        y = torch.randn(R, C, device="cuda", generator=g)
        o = torch.empty(R, C, device="cuda")
        gain = 1 + 0.1 * torch.randn(C, device="cuda", generator=g)
        rs = torch.randn(R, device="cuda", generator=g)
        dx, dy, do, dg, drs = W(x), W(y), W(o), W(gain), W(rs)
        nb = R * C * 4
        suite = [
            ("rmsnorm", lambda: kernels.rmsnorm(dx, dg, 1e-5, out=do), 2 * nb + C * 4),
            ("rope h32x128 theta5e5",
             lambda: kernels.rope(dx, base=500000.0, dimension=128, head_count=32, out=do), 2 * nb),
            ("silu", lambda: kernels.silu(dx, out=do), 2 * nb),
            ("add", lambda: kernels.add(dx, dy, out=do), 3 * nb),
            ("mul", lambda: kernels.mul(dx, dy, out=do), 3 * nb),
            ("residual-add", lambda: kernels.residual_add(dx, dy, out=do), 3 * nb),
            # the remaining advertised elementwise forms (not in the configs: same shape)
            ("gelu", lambda: kernels.gelu_tanh(dx, out=do), 2 * nb),
            ("row-scale", lambda: kernels.row_scale(dx, drs, out=do), 2 * nb + R * 4),
        ]
        for nm, fn, work in suite:
            if want(f"{nm} [8192,4096]"):
                add(f"{nm} [8192,4096]", "configs[3]" if nm not in ("gelu", "row-scale") else "advertised ops",
                    timed(fn, reps=10), "hbm", work)
        del x, y, o
    for dt, tdt in (("f16", torch.float16), ("bf16", torch.bfloat16)):
        if not any(want(f"{op} {dt} [8192,4096]") for op in ("add-half", "mul-half")):
            continue
        ha = (torch.rand(R, C, device="cuda", generator=g) * 16 - 8).to(tdt)
        hb = (torch.rand(R, C, device="cuda", generator=g) * 16 - 8).to(tdt)
        ho = torch.empty_like(ha)
        dha, dhb, dho = W(ha), W(hb), W(ho)
        for op, fn in (("add-half", kernels.add_half), ("mul-half", kernels.mul_half)):
            if want(f"{op} {dt} [8192,4096]"):
                add(f"{op} {dt} [8192,4096]", "configs[3]", timed(lambda: fn(dha, dhb, out=dho), reps=10), "hbm",
                    3 * R * C * 2)
    torch.cuda.synchronize()
    return results


def tp_mlp_bench(torch, mpc, kernels, world, rank, steps, warmup, tf32_tflops):
    """SwiGLU MLP tokens 4096, hidden 8192, ffn 28672 across all ranks."""
    import torch.distributed as dist
    tp = importlib.import_module(PACKAGE + ".tensor_parallel")
    T, Hd, F = 4096, 8192, 28672
    s, e = tp.share(F, world, rank)
    g = torch.Generator(device="cuda")
    g.manual_seed(1234 + rank)
    x = torch.randn(T, Hd, device="cuda", generator=torch.Generator(device="cuda").manual_seed(7))
    gs = torch.randn(Hd, e - s, device="cuda", generator=g) * 0.02
    us = torch.randn(Hd, e - s, device="cuda", generator=g) * 0.02
    ds = torch.randn(e - s, Hd, device="cuda", generator=g) * 0.02
    y = torch.empty(T, Hd, device="cuda")
    group = tp.TpGroup.from_torch_distributed(kernels) if world > 1 else tp.TpGroup(kernels, 0, 1, tp.TpGroup.unique_id())
    W = kernels.wrap_tensor
    dx, dg, du, dd, dy = W(x), W(gs), W(us), W(ds), W(y)
    try:
        for _ in range(max(1, warmup)):
            group.mlp(dx, dg, du, dd, chunks=4, out=dy)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        st = torch.cuda.Event(enable_timing=True)
        en = torch.cuda.Event(enable_timing=True)
        with ClockSampler(torch.cuda.current_device()) as clocks:
            st.record()
            for _ in range(steps):
                group.mlp(dx, dg, du, dd, chunks=4, out=dy)
            en.record()
            en.synchronize()
        ms = st.elapsed_time(en) / steps
        # the split of a step (outside the timed loop, three calls): start -> last down chunk
        # done (GEMMs, with the overlapped all-reduces beside them), then the all-reduce time
        # left exposed after it; events on the compute stream, max over ranks
        group.set_mlp_timing(True)
        split = []
        for _ in range(3):
            group.mlp(dx, dg, du, dd, chunks=4, out=dy)
            split.append(group.mlp_timing())
        group.set_mlp_timing(False)
        t = torch.tensor([ms, min(c for c, _ in split), min(e for _, e in split)], device="cuda")
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, compute_ms, exposed_ms = (float(v) for v in t.tolist())
    finally:
        group.close()
    flops = 3 * 2.0 * T * Hd * F
    return {"workload": "configs[4] SwiGLU MLP tokens 4096 hidden 8192 ffn 28672, gate/up column-split, "
                        "down row-split, one NCCL all-reduce chunked x4 over the down projection",
            "n_gpus": world, "ms_per_step": round(ms, 3), "tokens_per_s": round(T / (ms * 1e-3), 1),
            "compute_ms": round(compute_ms, 3), "exposed_allreduce_ms": round(exposed_ms, 3),
            "tflops": round(flops / (ms * 1e-3) / 1e12, 2),
            "frac_of_3xtf32_effective_x_n": round(flops / (ms * 1e-3) / 1e12 / (world * tf32_tflops / 3), 4),
            "clocks": clocks.summary()}


def run_ours(args, world, rank, local):
    import torch
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    mpc = importlib.import_module(PACKAGE)
    layer = importlib.import_module(PACKAGE + ".layer")
    provider = mpc.CudaProvider.for_device(local)
    if not provider.is_available():
        raise SystemExit(f"cuda:{local} unavailable: {provider.unavailable_reason()}")
    kernels = provider.kernels()
    ex = provider.execution_api()
    # One non-default stream for torch's flushes/events and the provider's kernels, so that
    # events bracket exactly the provider's work and graph capture is legal.
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    kernels.set_stream(stream.cuda_stream)
    peaks = load_peaks()

    if args.only_suite is not None:
        res = kernel_suite(torch, mpc, kernels, peaks, 0.0, filt=args.only_suite, iters=args.steps)
        if rank == 0:
            print(json.dumps({"only_suite": args.only_suite, "kernels": res}), flush=True)
        provider.close()
        return

    cfg = layer.DecoderLayerConfig()
    w = layer.make_inputs(cfg, seed=rank)
    layer.load(ex, w)
    layer.capture(ex, cfg)
    flush = make_l2_flush(torch)

    # warm-up replays
    for _ in range(max(3, args.warmup)):
        ex.replay_steps(1)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()

    # ---- timed region: K steps, L2 flushed between steps (flush outside the events) --------
    launches0 = kernels.launch_count()
    step_ms = []
    with ClockSampler(local) as clocks:
        for _ in range(args.steps):
            flush()
            s = torch.cuda.Event(enable_timing=True)
            e = torch.cuda.Event(enable_timing=True)
            # the spin (before the start event) outlasts the host's enqueueing of the step even
            # when several ranks share the host's cores
            gpu_busy(torch, 200.0 if world == 1 else 1000.0)
            s.record()
            ex.launch_step()
            e.record()
            e.synchronize()
            step_ms.append(s.elapsed_time(e))
        ex.check_steps()  # the embedding-id check of all timed steps
        torch.cuda.synchronize()
    launches = kernels.launch_count() - launches0
    total_ms = sum(step_ms)
    t = torch.tensor([total_ms], device="cuda")
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    total_ms = float(t.item())
    value = world * cfg.seq * args.steps / (total_ms * 1e-3)

    # ---- e2e through the public API with host buffers ---------------------------------------
    ids_host = torch.from_numpy(w["ids"]).pin_memory()
    out_host = torch.empty((cfg.seq, cfg.hidden), dtype=torch.float32).pin_memory()

    # one public call per step: the ids copied in, the captured layer replayed, the output copied
    # out, one synchronisation (which also covers the embedding-id check)
    e2e_step = ex.step_io({"ids": ids_host}, {"out": out_host})

    for _ in range(max(3, args.warmup)):
        e2e_step()
    if world > 1:
        torch.distributed.barrier()
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(args.steps):
        e2e_step()
    e.record()
    e.synchronize()
    e2e_ms = s.elapsed_time(e)
    t = torch.tensor([e2e_ms], device="cuda")
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    e2e_value = world * cfg.seq * args.steps / (float(t.item()) * 1e-3)

    # ---- per-node times of the layer: the dominant kernel's roofline --------------------------
    # Each node is timed as NODE_COPIES instances of itself captured into one step, each on its
    # own copy of the layer's tensors (id prefixes), chained by programmatic dependent launch as
    # in the layer's step.  The L2 is flushed before every replay, so each instance reads its
    # weights from HBM; a node's time is the replay's over NODE_COPIES (the event pair's fixed
    # cost and the graph launch spread over the copies).  No host work and no flag read-back
    # inside the events.
    prefixes = [f"node{i}/" for i in range(NODE_COPIES)]
    for pfx in prefixes:
        layer.load(ex, w, pfx)
        layer.forward(ex, cfg, pfx)  # allocates the copy's intermediates
    ex.synchronize()
    copies = [layer.invocations(cfg, pfx) for pfx in prefixes]
    node_times = []
    for j, inv in enumerate(layer.invocations(cfg)):
        ex.begin_step_capture()
        try:
            for c in copies:
                ex.run(c[j])
        except Exception:
            ex.abort_step_capture()
            raise
        ex.end_step_capture()
        ms = robust_mean(time_events(torch, ex.launch_step, 15, flush, warmup=3)) / NODE_COPIES
        ex.check_steps()
        node_times.append((inv, ms))
    tf32 = measure_tf32_peak(torch) if rank == 0 else 0.0
    dom_inv, dom_ms = max(node_times, key=lambda x: x[1])
    roofline = dominant_roofline(cfg, dom_inv, dom_ms, peaks, tf32) if rank == 0 else None

    # The per-kernel suite before the tensor-parallel MLP: the MLP's seconds of dense GEMMs run
    # at the power cap and leave the clocks lower for whatever follows.
    suite = None
    if rank == 0 and world == 1 and not args.no_suite:
        suite = kernel_suite(torch, mpc, kernels, peaks, tf32)

    tp_line = None
    if not args.no_tp:
        tp_line = tp_mlp_bench(torch, mpc, kernels, world, rank, max(3, min(args.steps, 10)), 2,
                               tf32 if rank == 0 else 1.0)

    cpu = None
    if rank == 0 and world == 1:
        rate, n, cores = cpu_layer_rate(cfg, w, budget_s=10.0)
        cpu = {"value": round(rate, 1), "unit": UNIT, "cores": cores, "kind": "port",
               "sample": f"{n} decoder-layer forwards (128 tokens each) of the C oracle on the host cores, "
                         f"about 10 s; the reference CPU executor (Rust) is not buildable here"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": bench_config(world),
            "e2e": {"value": round(e2e_value, 1), "unit": UNIT, "h2d_bytes_per_step": cfg.seq * 4,
                    "d2h_bytes_per_step": cfg.seq * cfg.hidden * 4 + 4},
            "gpu_launches": int(launches),
            "roofline": roofline,
            "cpu_baseline": cpu,
            "clocks": clocks.summary(),
            "layer_nodes_ms": [{"kernel": inv.kernel, "output": inv.output, "ms": round(ms, 4)}
                               for inv, ms in node_times],
            "tf32_tflops_measured": round(tf32, 1),
            "peaks_source": peaks["source"],
        }
        if tp_line is not None:
            line["tp_mlp"] = tp_line
        if suite is not None:
            line["kernels_columns"] = ["kernel", "ms", "achieved", "frac", "frac_of_bf16x3_effective"]
            line["kernels_peaks"] = {"hbm_gbs": peaks["hbm_gbs"], "tensor_3xtf32_tflops": round(tf32 / 3.0, 1),
                                     "bf16x3_tflops": round(peaks["bf16_tflops"] / 3.0, 1),
                                     "units": "GB/s for HBM-bound lines (matmul M<=16, attention decode, "
                                              "softmax, [8192,4096] ops); TFLOP/s otherwise"}
            line["kernels"] = suite
        # the nested objects last but the headline keys first; a long "kernels" list sits
        # before tp_mlp so that a tail of the line still shows the multi-GPU numbers
        if "tp_mlp" in line:
            line["tp_mlp"] = line.pop("tp_mlp")
        print(json.dumps(line, separators=(",", ":")), flush=True)
    provider.close()
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


# DRAM bytes (read + write) per launch of each layer node, from ncu captures of one to three
# launches of each kernel of this bench command (dram__bytes_read.sum + dram__bytes_write.sum,
# caches flushed before each; the decoder-layer summary in profiles/), keyed by the node's output
# id.  Writes stay in the L2 at this size.
LAYER_NODE_TRAFFIC = {"x": 276480, "h": 285952, "q": 1362944, "k": 1362176, "v": 1362176, "qr": 320000,
                      "kr": 320000, "a": 837376, "x2": 1624576, "h2": 285952, "g": 5961728, "out": 3836672}


def dominant_roofline(cfg, inv, ms, peaks, tf32):
    """Roofline object of the layer's slowest node (algorithmic work per launch / time)."""
    s, h, f, d, H = cfg.seq, cfg.hidden, cfg.ffn, cfg.head_dim, cfg.heads
    flops = {
        "matmul": 2.0 * s * h * h, "matmul-residual": 2.0 * s * h * (h if inv.output == "x2" else f),
        "gated-matmul": 2 * 2.0 * s * h * f, "attention": 4.0 * H * s * s * d / 2,
    }
    if inv.kernel in flops:
        eff = tf32 / 3.0
        ach = flops[inv.kernel] / (ms * 1e-3) / 1e12
        return {"kernel": inv.kernel, "bound": "tensor", "achieved": round(ach, 3), "peak": round(eff, 1),
                "unit": "TFLOP/s", "frac": round(ach / eff, 5), "traffic": LAYER_NODE_TRAFFIC.get(inv.output),
                "peak_basis": "3xTF32-effective = measured cuBLAS TF32 / 3 (of measured)",
                "node": inv.output, "ms": round(ms, 5)}
    bytes_ = {"embedding": s * h * 4 * 2 + s * 4, "rmsnorm": 2 * s * h * 4 + h * 4, "rope": 2 * s * h * 4}
    b = bytes_.get(inv.kernel, 2 * s * h * 4)
    ach = b / (ms * 1e-3) / 1e9
    return {"kernel": inv.kernel, "bound": "hbm", "achieved": round(ach, 2), "peak": peaks["hbm_gbs"],
            "unit": "GB/s", "frac": round(ach / peaks["hbm_gbs"], 5), "traffic": LAYER_NODE_TRAFFIC.get(inv.output),
            "node": inv.output, "ms": round(ms, 5)}


def main():
    faulthandler.enable()  # a native crash prints every thread's Python stack
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-suite", action="store_true", help="skip the per-kernel roofline suite")
    ap.add_argument("--no-tp", action="store_true", help="skip the tensor-parallel MLP")
    ap.add_argument("--only-suite", default=None, metavar="FILTER",
                    help="profiling aid: run only the suite cases whose name contains FILTER, --steps times each")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world, rank, local = dist_setup()
    if args.impl == "reference":
        run_reference(args, world, rank)
        return
    run_ours(args, world, rank, local)


if __name__ == "__main__":
    main()
