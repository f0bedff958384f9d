"""Benchmark of the MXFP8 fused SwiGLU-LoRA MLP (forward + backward) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload layer|stack]

One step = the fused MLP forward + autograd backward (dX, dA, dB of the three LoRA adapters) over one
batch of tokens, plus, with N > 1 ranks, the NCCL all-reduce of the LoRA gradients (the only data
exchange of token-sharded data parallelism).

Workloads:
  layer  (default) one Qwen3.5-2B MLP layer (hidden 2048, intermediate 6144, LoRA r=16, alpha=32) over
         16,384 tokens per rank -- configs[1] at N=1; every rank adds its own 16,384-token shard
         ("scaling": "weak").
  stack  the 24-layer 2B MLP stack over one 142,336-token step (16 packed conversations of 8,896
         tokens), token-sharded over the ranks -- configs[3] ("scaling": "strong").

The metric is MLP layer-tokens per second over the whole job (tokens x layers / step time, max over
ranks), i.e. tokens/s for the single-layer workload.  Inputs are synthetic (seeded N(0,1)
activations, N(0,0.02) frozen weights, N(0,0.01) LoRA A/B).  The per-step working set (gu alone is
T x 2N bf16 = 384 MiB per layer) is larger than the 126 MB L2, so no explicit L2 flush is needed.

`--impl reference` times the reference algorithm on the host CPU (the oracle port, all host threads)
on a bounded token sample of the same workload, and prints the same JSON line with "impl": "reference".
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "train-model-template_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

H, N, R, ALPHA = 2048, 6144, 16, 32
SCALE = ALPHA / R
LAYER_TOKENS = 16384
GEMM_TRAFFIC_BYTES = 1352104960   # ncu dram__bytes_read + write, 4 GEMM launches, 16,384-token layer step
STACK_TOKENS, STACK_LAYERS = 142336, 24
METRIC = "MXFP8 fused-MLP fwd+bwd tokens/s (2B shape)"
UNIT = "tokens/s"
FLOP_PER_TOKEN = 12 * H * N             # MXFP8 GEMM flops per token per layer, fwd + bwd
LORA_FLOP_PER_TOKEN = 2 * R * (9 * H + 12 * N)


def _args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=("layer", "stack", "ckpt", "quant", "ragged"), default="layer",
                    help="layer: configs[1] (default); stack: configs[3]; ckpt: configs[3] with every layer "
                         "checkpointed (recompute with need_out=False, as the reference's shared-prefix step); "
                         "quant: the configs[2] quantizer sweep (HBM GB/s); ragged: configs[4] small-M latency")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end (host buffers) measurement")
    ap.add_argument("--tokens", type=int, default=0,
                    help="tokens per rank for the layer workload (default 16384; smaller cases for profiling)")
    return ap.parse_args()


# ----------------------------------------------------------------------------------------------- clocks
class ClockSampler:
    """SM clock, power and throttle reasons sampled while the timed region runs (read-only queries).

    NVML from a thread every 5 ms (a timed region of a few tens of milliseconds still gets samples);
    `nvidia-smi -lms 200` when NVML is not importable."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
    BITS = (0x8, 0x40, 0x20, 0x4)   # NVML clocks-event-reason bits of NAMES

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None
        self.thread = None
        self.rows = []

    def _nvml_handle(self, nv):
        try:
            import torch
            p = torch.cuda.get_device_properties(self.index)
            bus = f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0"
            return nv.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return nv.nvmlDeviceGetHandleByIndex(self.index)

    def start(self):
        try:
            import threading
            import pynvml as nv
            nv.nvmlInit()
            h = self._nvml_handle(nv)
            reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nv.nvmlDeviceGetCurrentClocksThrottleReasons
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            self.stop_ev = threading.Event()

            def run():
                while True:
                    try:
                        self.rows.append((float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)), int(reasons(h))))
                    except Exception:
                        pass
                    if self.stop_ev.wait(0.005):
                        break
            self.thread = threading.Thread(target=run, daemon=True)
            self.thread.start()
            return
        except Exception:
            self.thread = None
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.thread is not None:
            self.stop_ev.set()
            self.thread.join(timeout=5)
            if not self.rows:
                return None
            reasons = sorted({n for _, m in self.rows for n, b in zip(self.NAMES, self.BITS) if m & b})
            return {"sm_mhz": statistics.median(c for c, _ in self.rows), "sm_max_mhz": self.max_mhz,
                    "reasons": reasons, "samples": len(self.rows), "source": "nvml"}
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) >= 9:
                rows.append(f)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        reasons = sorted({n for r in rows for n, v in zip(self.NAMES, r[5:9]) if v.lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows), "source": "nvidia-smi"}


# ----------------------------------------------------------------------------------------------- our arm
def _make_layer(torch, fused_mlp, dev, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    w = lambda *s: (torch.randn(*s, generator=g) * 0.02).to(torch.bfloat16).to(dev)   # noqa: E731
    layer = fused_mlp.MXMLPWeights.from_bf16(w(N, H), w(N, H), w(H, N))
    shapes = ((R, H), (N, R), (R, H), (N, R), (R, N), (H, R))
    params = [(torch.randn(*s, generator=g) * 0.01).to(dev).requires_grad_(True) for s in shapes]
    return layer, params


def run_ours(a):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))

    import __graft_entry__
    __graft_entry__.build()
    import _mxlib
    import fused_linear
    import fused_mlp
    import mx_dp
    import mxfp8

    if a.workload == "layer":
        T, L = (a.tokens or LAYER_TOKENS), 1
        total_tokens = T * world
    else:
        r0, r1 = mx_dp.shard_rows(STACK_TOKENS, world, rank)
        T, L = r1 - r0, STACK_LAYERS
        total_tokens = STACK_TOKENS
    layers = [_make_layer(torch, fused_mlp, dev, seed=1000 + i) for i in range(L)]
    import torch.utils.checkpoint as tuc

    def ckpt_layer(layer, ps):
        # the reference's shared-prefix step (scripts/shared_prefix.py:200-203, 246-255): the forward inside
        # the backward's recompute runs with need_out=False (its output is never read)
        def fn(h):
            return fused_mlp.mlp_apply(layer, h, *ps, scaling=(SCALE, SCALE, SCALE),
                                       need_out=torch._C._current_graph_task_id() == -1)
        return fn
    params = [p for _, ps in layers for p in ps]
    gx = torch.Generator(device="cpu").manual_seed(7 + rank)
    x_host = torch.randn(T, H, generator=gx).to(torch.bfloat16).pin_memory()
    dy_host = torch.randn(T, H, generator=gx).to(torch.bfloat16).pin_memory()
    x = x_host.to(dev)
    dy = dy_host.to(dev)
    bucket = mx_dp.GradBucket(params, device=dev)    # the LoRA gradients: the only cross-rank exchange
    flat_host = torch.empty(bucket.flat.shape, dtype=torch.float32).pin_memory()

    def step(xin, dyin):
        fused_linear.new_step()
        h = xin.requires_grad_(False)
        h = h.detach().requires_grad_(True)
        y = h
        for layer, ps in layers:
            if a.workload == "ckpt":
                y = tuc.checkpoint(ckpt_layer(layer, ps), y, use_reentrant=False)
            else:
                y = fused_mlp.mlp_apply(layer, y, *ps, scaling=(SCALE, SCALE, SCALE))
        y.backward(dyin)
        if world > 1:   # bucketed all-reduce of every LoRA gradient (NCCL over NVLink)
            bucket.allreduce()
        for p in params:
            p.grad = None
        return h

    # GEMM launches timed with CUDA events on the launching stream (the roofline's dominant kernel)
    gemm_ms, gemm_flops, recording = [], [], [False]
    orig_mm, orig_lora = mxfp8.mx_mm, fused_mlp.mx_mm_lora

    def timed(fn):
        def wrap(a_, b_, *rest, **kw):
            if not recording[0]:
                return fn(a_, b_, *rest, **kw)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            out = fn(a_, b_, *rest, **kw)
            e1.record()
            gemm_ms.append((e0, e1))
            gemm_flops.append(2 * a_.shape[0] * a_.shape[1] * b_.shape[1])
            return out
        return wrap

    mxfp8.mx_mm = timed(orig_mm)
    fused_mlp.mx_mm_lora = timed(orig_lora)

    for _ in range(max(a.warmup, 3)):
        step(x, dy)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = ClockSampler(local)
    clk.start()
    launches0 = _mxlib.launch_count()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    recording[0] = True
    ev0.record()
    for _ in range(a.steps):
        step(x, dy)
    ev1.record()
    torch.cuda.synchronize()
    recording[0] = False
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = clk.stop()
    launches = _mxlib.launch_count() - launches0
    ms = ev0.elapsed_time(ev1) / a.steps
    g_ms = sum(e0.elapsed_time(e1) for e0, e1 in gemm_ms)
    g_fl = float(sum(gemm_flops))
    gemm_ms.clear()
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()

    # end to end through the public API: pinned host inputs -> device, step, LoRA grads -> host.  Every
    # step's x and dy are copied from pinned host memory inside the timed region; the copies of step i+1
    # run on a side stream into the second of two device buffer sets while step i computes (the usual
    # input pipelining of a training loop), so the step time is max(copy, compute), not their sum.
    recording[0] = False
    comp = torch.cuda.current_stream()
    copy_s = torch.cuda.Stream()
    xb, dyb = [x, torch.empty_like(x)], [dy, torch.empty_like(dy)]
    loaded = [torch.cuda.Event(), torch.cuda.Event()]
    freed = [torch.cuda.Event(), torch.cuda.Event()]

    def e2e_load(i):
        b = i % 2
        with torch.cuda.stream(copy_s):
            copy_s.wait_event(freed[b])          # step i-2 finished reading this buffer set
            xb[b].copy_(x_host, non_blocking=True)
            dyb[b].copy_(dy_host, non_blocking=True)
            loaded[b].record(copy_s)

    def e2e_step(i):
        b = i % 2
        comp.wait_event(loaded[b])
        fused_linear.new_step()
        h = xb[b].detach().requires_grad_(True)
        y = h
        for layer, ps in layers:
            if a.workload == "ckpt":
                y = tuc.checkpoint(ckpt_layer(layer, ps), y, use_reentrant=False)
            else:
                y = fused_mlp.mlp_apply(layer, y, *ps, scaling=(SCALE, SCALE, SCALE))
        y.backward(dyb[b])
        freed[b].record(comp)
        bucket.allreduce()
        flat_host.copy_(bucket.flat, non_blocking=True)
        for p in params:
            p.grad = None

    def e2e_run(n):
        for b in range(2):
            freed[b].record(comp)
        e2e_load(0)
        for i in range(n):
            if i + 1 < n:
                e2e_load(i + 1)
            e2e_step(i)

    e2e_ms = float("nan")
    if not a.no_e2e:
        e2e_run(2)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        e2e_run(a.steps)
        e1.record()
        torch.cuda.synchronize()
        e2e_ms = e0.elapsed_time(e1) / a.steps
    if world > 1 and not a.no_e2e:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = t.item()

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        cpu = cpu_baseline(a.workload)

    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return
    import json as _j
    peaks = {}
    try:
        peaks = _j.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    if peaks.get("bf16_tflops_sustained"):
        peak = 2.0 * float(peaks["bf16_tflops_sustained"])
        peak_note = "2 x measured sustained bf16 cuBLAS (MEASURED_PEAKS.json): dense MXFP8 rate is twice bf16"
    else:
        peak = 2.0 * 1400.0
        peak_note = "2 x fallback sustained bf16 1.4 PFLOP/s"
    achieved = g_fl / (g_ms * 1e-3) / 1e12 if g_ms > 0 else None
    tok = total_tokens * L
    line = {
        "metric": METRIC, "value": tok / (ms * 1e-3), "unit": UNIT, "n_gpus": world, "steps": a.steps,
        "warmup": max(a.warmup, 3), "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak" if a.workload == "layer" else "strong", "vs_baseline": None, "dtype": "mxfp8-e4m3/bf16",
        "data": "synthetic (seeded N(0,1) activations, N(0,0.02) frozen weights, N(0,0.01) LoRA A/B)",
        "config": {"workload": ((f"configs[1]: one Qwen3.5-2B MLP layer, {T} tokens per rank" if T == LAYER_TOKENS
                                 else f"one Qwen3.5-2B MLP layer, {T} tokens per rank (configs[1] holds {LAYER_TOKENS})")
                                if a.workload == "layer"
                                else "configs[3]: 24-layer Qwen3.5-2B MLP stack, 142336-token step, token-sharded"
                                + (", every layer checkpointed (recompute with need_out=False)"
                                   if a.workload == "ckpt" else "")),
                   "hidden": H, "intermediate": N, "lora_rank": R, "lora_alpha": ALPHA, "layers": L,
                   "tokens_per_rank": T, "parallelism": f"dp{world} (token shards, NCCL all-reduce of LoRA grads)",
                   "l2": f"per-step working set > L2 (gu alone {T * 4 * N // 2**20} MiB per layer); no flush"},
        "e2e": None if a.no_e2e else {"value": tok / (e2e_ms * 1e-3), "unit": UNIT,
                "h2d_bytes_per_step": x_host.numel() * 2 + dy_host.numel() * 2,
                "d2h_bytes_per_step": flat_host.numel() * 4},
        "gpu_launches": int(launches),
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": (achieved / peak) if achieved else None,
                     # DRAM bytes (read + write) of the step's four GEMM launches from one ncu capture of
                     # this workload (profiles/gemm_traffic_2B_T16384.md); other token counts: not captured
                     "traffic": GEMM_TRAFFIC_BYTES if (a.workload == "layer" and T == LAYER_TOKENS) else None,
                     "traffic_unit": "bytes per step (4 GEMM launches)",
                     "kernel": "k_mx_gemm (tcgen05 MXFP8 GEMMs, 4 launches per layer per step)",
                     "flops_per_step": g_fl / a.steps, "peak_source": peak_note},
        "mlp_tflops": FLOP_PER_TOKEN * tok / (ms * 1e-3) / 1e12,
        "clocks": clocks,
        "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------------------------- CPU leg
def _cpu_setup(tokens):
    """Seeded 2B-layer operands for the oracle port: frozen MX weights (quantized once), LoRA, x, dy."""
    import numpy as np
    from oracle import mx_oracle as O
    rng = np.random.default_rng(0)
    bf = lambda a: O.bf16_round(a.astype(np.float32))  # noqa: E731
    Wg, Wu = bf(rng.standard_normal((N, H)) * 0.02), bf(rng.standard_normal((N, H)) * 0.02)
    Wd = bf(rng.standard_normal((H, N)) * 0.02)
    W = O.MXWeights(Wg, Wu, Wd)              # frozen weights: quantized once per run, not per step
    lora = [(rng.standard_normal(s) * 0.01).astype(np.float32)
            for s in ((R, H), (N, R), (R, H), (N, R), (R, N), (H, R))]
    x = bf(rng.standard_normal((tokens, H)))
    dy = bf(rng.standard_normal((tokens, H)))
    return W, lora, x, dy


def _cpu_step(W, lora, x, dy):
    """One fwd+bwd of the oracle port (the reference algorithm in numpy); returns its wall time in s."""
    from oracle import mx_oracle as O
    t0 = time.perf_counter()
    y, ctx = O.mlp_forward(x, W, *lora, SCALE, SCALE, SCALE)
    O.mlp_backward(dy, ctx)
    return time.perf_counter() - t0


def _cpu_sample(workload, tokens):
    """Time the oracle port on `tokens` tokens of one 2B layer (up to 3 repetitions or ~10 s)."""
    W, lora, x, dy = _cpu_setup(tokens)
    t0 = time.perf_counter()
    reps = 0
    while True:
        _cpu_step(W, lora, x, dy)
        reps += 1
        if time.perf_counter() - t0 > 10.0 or reps >= 3:
            break
    dt = (time.perf_counter() - t0) / reps
    return tokens / dt, dt


def _threads():
    try:
        from threadpoolctl import threadpool_info
        n = [i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"]
        return max(n) if n else os.cpu_count()
    except Exception:
        return os.cpu_count()


def cpu_baseline(workload):
    tokens = 1024
    v, dt = _cpu_sample(workload, tokens)
    return {"value": v, "unit": UNIT, "cores": _threads(), "kind": "port",
            "sample": f"{tokens} tokens of one 2B MLP layer, fwd+bwd, numpy oracle port of the reference algorithm "
                      f"({dt:.2f} s per sample step; layer-tokens/s)"}


def run_reference(a):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    # each step is a bounded token sample (about 3.7 s per 1,024 tokens on 8 host threads); the sample
    # shrinks for long runs so that --steps K --warmup W stays within about two minutes
    steps, warm = max(1, a.steps), max(a.warmup, 3)
    tokens = int(min(1024, max(128, 120.0 / (3.7 * steps) * 1024)) // 128 * 128)
    W, lora, x, dy = _cpu_setup(tokens)
    for _ in range(warm):   # warm-up steps on a 128-token slice (numpy / BLAS threads, page-in)
        _cpu_step(W, lora, x[:128], dy[:128])
    vals = [tokens / _cpu_step(W, lora, x, dy) for _ in range(steps)]
    v = statistics.median(vals)
    line = {
        "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": world, "steps": steps, "warmup": warm,
        "ms_per_step": tokens / v * 1e3, "higher_is_better": True, "scaling": "weak" if a.workload == "layer" else "strong",
        "vs_baseline": None, "dtype": "mxfp8-e4m3/fp32 (CPU)", "data": "synthetic",
        "config": {"workload": "one Qwen3.5-2B MLP layer (hidden 2048, intermediate 6144, r 16), bounded token sample",
                   "tokens_per_sample": tokens},
        "impl": "reference",
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": _threads(), "kind": "port",
                         "sample": f"{tokens} tokens of one 2B MLP layer, fwd+bwd (numpy port of the reference algorithm)"},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------------------------- configs[2]
def _hbm_peak():
    try:
        return float(json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def run_quant(a):
    """the standalone MXFP8 quantizer over rows {4096, 16384, 65536, 142336} x cols {1024,
    2048, 3584, 6144} of N(0,1) bf16 with 0.5 % of entries x200 and 0.1 % exact zeros; row-wise
    (mx_quant), column-wise (mx_quant_t) and both from one read (mx_quant_pair).  Each timed call follows
    a 256 MiB write that evicts L2; the median of `steps` calls per case.  Algorithmic bytes: 3.03125 per
    element one way (read 2, write 1 + 1/32), 4.0625 both ways.  One GPU (rank 0 under torchrun)."""
    import torch
    rank, local = int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0"))
    if rank != 0:
        return
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    import __graft_entry__
    __graft_entry__.build()
    import _mxlib
    import mxfp8
    peak, src = _hbm_peak()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    g = torch.Generator(device=dev).manual_seed(0)
    modes = (("rows", mxfp8.mx_quant, 3.03125), ("cols", mxfp8.mx_quant_t, 3.03125),
             ("both", mxfp8.mx_quant_pair, 4.0625))
    clk = ClockSampler(local)
    clk.start()
    launches0 = _mxlib.launch_count()
    cases = []
    for rows in (4096, 16384, 65536, 142336):
        for cols in (1024, 2048, 3584, 6144):
            x = torch.randn(rows, cols, device=dev, generator=g)
            u = torch.rand(rows, cols, device=dev, generator=g)
            x = torch.where(u < 0.005, x * 200.0, x)
            x = torch.where((u >= 0.005) & (u < 0.006), torch.zeros_like(x), x).to(torch.bfloat16)
            del u
            case = {"R": rows, "K": cols}
            for name, fn, bpe in modes:
                for _ in range(max(a.warmup, 3)):
                    fn(x)
                evs = []
                for _ in range(a.steps):
                    flush.fill_(1)
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record()
                    out = fn(x)
                    e1.record()
                    evs.append((e0, e1))
                    del out
                torch.cuda.synchronize()
                us = statistics.median(e0.elapsed_time(e1) for e0, e1 in evs) * 1e3
                gbs = bpe * rows * cols / (us * 1e-6) / 1e9
                case[name] = {"us": round(us, 2), "gbs": round(gbs, 1), "frac": round(gbs / peak, 3)}
            cases.append(case)
            del x
    clocks = clk.stop()
    launches = _mxlib.launch_count() - launches0
    med = lambda k: statistics.median(c[k]["gbs"] for c in cases)  # noqa: E731
    big = [c for c in cases if c["R"] * c["K"] * 2 > (126 << 20)]
    line = {
        "metric": "MXFP8 quantizer achieved HBM GB/s (configs[2] sweep, row-wise, median over cases)",
        "value": med("rows"), "unit": "GB/s", "n_gpus": 1, "steps": a.steps, "warmup": max(a.warmup, 3),
        "ms_per_step": statistics.median(c["rows"]["us"] for c in cases) / 1e3, "higher_is_better": True,
        "scaling": "none", "vs_baseline": None, "dtype": "bf16 -> e4m3 + e8m0", "impl": "ours",
        "data": "synthetic N(0,1), 0.5 % x200 outliers, 0.1 % zeros (seeded)",
        "config": {"workload": "configs[2]: quantizer sweep rows {4096,16384,65536,142336} x cols "
                               "{1024,2048,3584,6144}", "l2": "256 MiB write before every timed call"},
        "median_gbs": {"rows": med("rows"), "cols": med("cols"), "both": med("both")},
        "median_gbs_inputs_over_l2": {k: statistics.median(c[k]["gbs"] for c in big) for k in ("rows", "cols", "both")},
        "roofline": {"bound": "hbm", "achieved": med("rows"), "peak": peak, "unit": "GB/s",
                     "frac": med("rows") / peak, "traffic": None, "kernel": "k_quant",
                     "peak_source": f"{src} copy bandwidth"},
        "cases": cases, "gpu_launches": int(launches), "clocks": clocks,
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------------------------- configs[4]
RAGGED_M = (1, 77, 1000, 2049, 10752)


def run_ragged(a):
    """latency of one fused-MLP fwd+bwd step at the 0.8B shape (hidden 1024, intermediate
    3584, LoRA r=16, alpha=32) for per-GPU token counts M in RAGGED_M (not multiples of 128), inputs
    N(0,1) with 1 % of entries x100.  With N > 1 ranks each rank runs its own M tokens and the step ends
    with the NCCL all-reduce of the LoRA gradients; the latency is the max over ranks of the CUDA-event
    time per step.  `graph_ms`: the same fwd+bwd captured once in a CUDA graph and replayed (static
    inputs), the all-reduce after each replay -- what a training loop that graphs its layer step sees."""
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank, local = int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    import __graft_entry__
    __graft_entry__.build()
    import _mxlib
    import fused_linear
    import fused_mlp
    import mx_dp
    Hs, Ns = 1024, 3584
    g = torch.Generator(device="cpu").manual_seed(11)
    w = lambda *s: (torch.randn(*s, generator=g) * 0.02).to(torch.bfloat16).to(dev)   # noqa: E731
    layer = fused_mlp.MXMLPWeights.from_bf16(w(Ns, Hs), w(Ns, Hs), w(Hs, Ns))
    shapes = ((R, Hs), (Ns, R), (R, Hs), (Ns, R), (R, Ns), (Hs, R))
    params = [(torch.randn(*s, generator=g) * 0.01).to(dev).requires_grad_(True) for s in shapes]
    bucket = mx_dp.GradBucket(params, device=dev)

    def sync_all():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    clk = ClockSampler(local)
    clk.start()
    launches0 = _mxlib.launch_count()
    res = []
    for M in RAGGED_M:
        gx = torch.Generator(device="cpu").manual_seed(100 + M + rank)
        def outl(t):
            u = torch.rand(t.shape, generator=gx)
            return torch.where(u < 0.01, t * 100.0, t)
        x = outl(torch.randn(M, Hs, generator=gx)).to(torch.bfloat16).to(dev)
        dy = outl(torch.randn(M, Hs, generator=gx)).to(torch.bfloat16).to(dev)

        def fwd_bwd():
            fused_linear.new_step()
            h = x.detach().requires_grad_(True)
            y = fused_mlp.mlp_apply(layer, h, *params, scaling=(SCALE, SCALE, SCALE))
            y.backward(dy)

        def step():
            fwd_bwd()
            if world > 1:
                bucket.allreduce()
            for p in params:
                p.grad = None

        def timed(fn):
            for _ in range(max(a.warmup, 3)):
                fn()
            sync_all()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(a.steps):
                fn()
            e1.record()
            torch.cuda.synchronize()
            return max_over_ranks(e0.elapsed_time(e1) / a.steps)

        eager = timed(step)
        # CUDA graph of the local fwd+bwd (captured on every rank alike; the all-reduce stays eager)
        graph_ms, err, graph = None, None, None
        try:
            for p in params:
                p.grad = None
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                for _ in range(3):
                    fwd_bwd()
                    for p in params:
                        p.grad = None
            torch.cuda.current_stream().wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                fwd_bwd()
        except Exception as e:   # capture is a host-side feature: report, keep the eager number
            err = f"{type(e).__name__}: {str(e)[:160]}"
            graph = None
        ok = graph is not None
        if world > 1:            # every rank times the graph, or none does (same collectives everywhere)
            t = torch.tensor([1 if ok else 0], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MIN)
            ok = bool(t.item())
        if ok:
            def replay():
                graph.replay()
                if world > 1:
                    bucket.allreduce()
            graph_ms = timed(replay)
        del graph
        for p in params:
            p.grad = None
        res.append({"M": M, "eager_ms": round(eager, 4), "graph_ms": None if graph_ms is None else round(graph_ms, 4),
                    **({"graph_error": err} if err else {})})
    clocks = clk.stop()
    launches = _mxlib.launch_count() - launches0
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": "fused-MLP fwd+bwd latency per step, 0.8B shape, ragged per-GPU M (mean over M, eager)",
        "value": statistics.mean(r["eager_ms"] for r in res), "unit": "ms", "n_gpus": world, "steps": a.steps,
        "warmup": max(a.warmup, 3), "ms_per_step": statistics.mean(r["eager_ms"] for r in res),
        "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "mxfp8-e4m3/bf16",
        "impl": "ours", "data": "synthetic N(0,1), 1 % x100 outliers (seeded)",
        "config": {"workload": "configs[4]: 0.8B MLP shape, per-GPU M in " + str(list(RAGGED_M)),
                   "hidden": Hs, "intermediate": Ns, "lora_rank": R, "lora_alpha": ALPHA,
                   "parallelism": f"dp{world} (each rank its own M tokens, NCCL all-reduce of LoRA grads)",
                   "l2": "small-M latency: working set in L2 by design, no flush"},
        "per_m": res, "gpu_launches": int(launches), "clocks": clocks,
    }
    print(json.dumps(line), flush=True)


def main():
    a = _args()
    if a.impl == "reference":
        run_reference(a)
    elif a.workload == "quant":
        run_quant(a)
    elif a.workload == "ragged":
        run_ragged(a)
    else:
        run_ours(a)


if __name__ == "__main__":
    main()
