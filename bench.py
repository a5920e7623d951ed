#!/usr/bin/env python
"""Benchmark of the FP8 hot path on B200 (FP8 3x3 conv, B=128, 128->128, 32x32).

One *step* is one training pass of an FP8 conv layer through the hot path, as
``Conv2dFP8Specialized`` runs it with current scaling (fp8_kernels.py:823-913):

    quantize X, quantize W  ->  conv fwd (Y)  ->  quantize dY  ->  conv dX  ->  conv dW

``value`` = algorithmic TFLOP/s of the step (3 x 2*M*N*K, M=B*H*W, N=Cout,
K=9*Cin), all ranks' work over the max-over-ranks device time, inputs resident
in HBM.  ``e2e`` = the same metric through the reference-facing API
(``triton_conv2d_fp8`` + autograd) with pinned host inputs and outputs, the
host<->device copies inside the timed region.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Multi-GPU (torchrun, one rank per GPU): every rank runs an independent replica
on its own batch (weak scaling; the path has no exchange step).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (ROOT / "diffusion-profiled_b200", ROOT / "oracle"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

import torch  # noqa: E402

METRIC = "FP8 conv/GEMM TFLOP/s (% FP8 peak); UNet train imgs/s at 1/2/4/8 B200"
UNIT = "TFLOP/s"
SHAPE = dict(cin=128, cout=128, h=32, w=32)
L2_BYTES = 126 * 1024 * 1024


def conv_flops(batch: int) -> float:
    m = batch * SHAPE["h"] * SHAPE["w"]
    return 2.0 * m * SHAPE["cout"] * 9 * SHAPE["cin"]


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--batch", type=int, default=128, help="images per GPU (config 2: 128)")
    ap.add_argument("--workload", choices=["layer", "fwd"], default="layer",
                    help="layer: fwd+dX+dW with the three quantizes; fwd: quantize X, W + conv fwd")
    ap.add_argument("--rotate", type=int, default=3, help="rotating input sets (per-step working set > L2)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-kernel-timing", action="store_true")
    ap.add_argument("--no-clocks", action="store_true", help="skip nvidia-smi sampling (profiling runs)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU baseline sample duration")
    ap.add_argument("--no-unet", action="store_true", help="skip the UNet training-step measurement")
    ap.add_argument("--no-sweep", action="store_true",
                    help="skip the per-config sweep (linear configs 1 / 3, conv at batch 512, delayed quantize)")
    ap.add_argument("--pdl", type=int, default=0, choices=(0, 1, 2),
                    help="programmatic dependent launch: 0 off (default), 1 tensor-core kernels, 2 every kernel")
    ap.add_argument("--bucket-mb", type=float, default=None,
                    help="gradient all-reduce bucket size of the data-parallel UNet step (MB of bf16)")
    ap.add_argument("--unet-steps", type=int, default=30, help="timed UNet training steps")
    return ap.parse_args()


# ============================================================================ helpers
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons while the GPU is under load."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, gpu_index: int, enabled: bool = True):
        self.gpu_index = gpu_index
        self.enabled = enabled
        self.proc = None
        self.t0 = self.t1 = 0.0

    def start(self):
        if not self.enabled:
            self.t0 = time.time()
            return
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.gpu_index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        self.t0 = time.time()

    def stop(self) -> dict:
        self.t1 = time.time()
        if self.proc is None:
            note = "sampling disabled" if not self.enabled else "nvidia-smi unavailable"
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "note": note}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = [r.split(",") for r in out.strip().splitlines() if r.count(",") >= 8]
        # drop the first sample (taken before the load started)
        rows = rows[1:] if len(rows) > 2 else rows
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        reasons = sorted({name for r in rows for name, v in zip(self.REASONS, r[5:9]) if v.strip() == "Active"})
        power = [float(r[3]) for r in rows if r[3].strip().replace(".", "").isdigit()]
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(smax) if smax else None,
            "reasons": reasons,
            "samples": len(rows),
            "power_w_max": max(power) if power else None,
        }


def physical_gpu_index(local_rank: int) -> int:
    cvd = os.environ.get("CUDA_VISIBLE_DEVICES")
    if cvd:
        parts = [p for p in cvd.split(",") if p.strip()]
        if local_rank < len(parts) and parts[local_rank].strip().isdigit():
            return int(parts[local_rank])
    return local_rank


def measured_peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        return {"hbm_gbs": d.get("hbm_gbs"), "bf16_tflops": d.get("bf16_tflops"),
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def ncu_traffic() -> dict:
    # JSON text: op name -> DRAM bytes (read + write) per launch from one ncu capture
    path = ROOT / "profiles" / "ncu_traffic_per_launch.txt"
    return json.loads(path.read_text()) if path.exists() else {}


def make_inputs(batch: int, device, seed: int):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(batch, SHAPE["cin"], SHAPE["h"], SHAPE["w"], generator=g).to(torch.bfloat16)
    dy = (torch.randn(batch, SHAPE["cout"], SHAPE["h"], SHAPE["w"], generator=g) * 1e-2).to(torch.bfloat16)
    cl = torch.channels_last
    return x.contiguous(memory_format=cl).to(device), dy.contiguous(memory_format=cl).to(device)


def make_weight(device, seed: int = 1234):
    torch.manual_seed(seed)
    conv = torch.nn.Conv2d(SHAPE["cin"], SHAPE["cout"], 3, padding=1, bias=False)  # kaiming_uniform(a=sqrt 5)
    return conv.weight.detach().to(torch.bfloat16).contiguous(memory_format=torch.channels_last).to(device)


def json_stdout():
    """A file on the process's original stdout, for the one JSON line.  File
    descriptor 1 itself is pointed at stderr, so text that native libraries print
    to stdout (NCCL's version banner, for one) cannot mix with that line."""
    sys.stdout.flush()
    out = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    return out


# ============================================================================ B200 arm
def run_b200(args) -> None:
    import torch.distributed as dist

    result_out = json_stdout()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        from datetime import timedelta

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local_rank))
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)

    import fp8_b200  # noqa: F401  (loads libfp8ops.so, fails loudly without it)
    from fp8_b200 import _lib, ops
    from fp8_b200.fp8_kernels import triton_conv2d_fp8

    _lib.set_pdl(args.pdl)

    batch = args.batch
    flops_conv = conv_flops(batch)
    n_convs = 3 if args.workload == "layer" else 1
    step_flops = n_convs * flops_conv

    w = make_weight(dev)
    sets = [make_inputs(batch, dev, seed=1000 * rank + i) for i in range(max(1, args.rotate))]

    def step(x, dy):
        xq, sx, wq, sw = ops.quantize_current_pair(x, w)  # the forward's input and weight together
        y = ops.conv3x3_fwd(xq, wq, sx, sw)
        if args.workload == "fwd":
            return (y,)
        dyq, sdy = ops.quantize_current(dy)
        dx, dw = ops.conv3x3_backward(dyq, wq, sdy, sw, xq, sx)  # dW on a side stream beside dX, as in autograd
        return (y, dx, dw)

    # eager warm-up: sets kernel attributes, counts launches of one step
    for x, dy in sets:
        step(x, dy)
    torch.cuda.synchronize()
    n0 = _lib.kernel_launch_count()
    step(*sets[0])
    torch.cuda.synchronize()
    launches_per_step = _lib.kernel_launch_count() - n0

    graphs = []
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for x, dy in sets:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                step(x, dy)
            graphs.append(g)
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize()

    def replay(k: int, offset: int = 0):
        for i in range(k):
            graphs[(offset + i) % len(graphs)].replay()

    replay(args.warmup)
    torch.cuda.synchronize()

    sampler = ClockSampler(physical_gpu_index(local_rank), enabled=not args.no_clocks)
    sampler.start()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    replay(args.steps)
    ev1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t_timed_wall = time.time() - sampler.t0
    # short timed regions get fewer than ~3 nvidia-smi samples: keep the same
    # step running for 1.5 s more under the same sampler
    sustain = t_timed_wall < 1.0 and not args.no_clocks
    if sustain:
        t_end = time.time() + 1.5
        while time.time() < t_end:
            replay(50)
            torch.cuda.synchronize()
    clocks = sampler.stop()
    clocks["window"] = "timed region + 1.5 s of the same step" if sustain else "timed region"

    ms = ev0.elapsed_time(ev1)
    t_max = torch.tensor([ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t_max, op=dist.ReduceOp.MAX)
    ms_total = float(t_max.item())
    ms_per_step = ms_total / max(args.steps, 1)
    value = world * step_flops * args.steps / (ms_total * 1e-3) / 1e12

    # ------------------------------------------------------------------ per-kernel timing (roofline)
    kernels = {} if args.no_kernel_timing else time_kernels(args, dev, w, sets)
    if world > 1:
        gathered = [None] * world
        dist.all_gather_object(gathered, clocks)
        reasons = sorted({r for c in gathered if c for r in c.get("reasons", [])})
        clocks["reasons"] = reasons
        clocks["ranks"] = world

    sweep = None
    if rank == 0 and not args.no_sweep:
        sweep = time_sweep(args, dev)

    # ------------------------------------------------------------------ end to end (host buffers)
    e2e = None
    if not args.no_e2e:
        e2e = time_e2e(args, dev, world, triton_conv2d_fp8, step_flops)

    # release graphs before tearing the process group down
    del graphs
    torch.cuda.synchronize()

    unet = None
    if not args.no_unet:
        unet = {"b200_path": time_unet(args, dev, world, fp8=True, scaling="delayed", skip_empty=True)}
        if world == 1:
            unet["b200_path_current_scaling"] = time_unet(args, dev, world, fp8=True, scaling="current")
            unet["bf16_reference_ops"] = time_unet(args, dev, world, fp8=False)
            unet["speedup_vs_bf16_reference_ops"] = round(
                unet["b200_path"]["value"] / unet["bf16_reference_ops"]["value"], 3)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_oracle_baseline(args, seconds=args.cpu_seconds)

    if rank == 0:
        peaks = measured_peaks()
        fp8_peak = 2.0 * peaks["bf16_tflops"]
        roof = roofline(kernels, peaks, batch)
        line = {
            "metric": METRIC,
            "value": round(value, 3),
            "unit": UNIT,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_per_step, 6),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "e4m3 (fp32 accumulate, bf16 out)",
            "data": "synthetic (seeded randn activations / dY, nn.Conv2d default-init weights)",
            "config": {
                "workload": ("conv3x3_fp8_layer_fwd_dgrad_wgrad" if args.workload == "layer"
                             else "conv3x3_fp8_fwd"),
                "baseline_config": "configs[1]: FP8 3x3 conv B=128 128->128 32x32 (M=131072 N=128 K=1152)",
                "batch_per_gpu": batch,
                "global_batch": batch * world,
                **SHAPE,
                "scaling": "current (per-tensor amax of X, W, dY each step)",
                "launch": ("plain stream order", "programmatic dependent launch of the tensor-core kernels",
                           "programmatic dependent launch of every kernel")[args.pdl],
                "flops_per_step": step_flops,
                "l2": f"{len(sets)} rotating input sets; per-step working set > 126 MB L2",
                "parallelism": f"replicas x{world} (no collective on the path)",
            },
            "gpu_launches": launches_per_step * args.steps,
            "gpu_launches_scope": f"per GPU ({launches_per_step} libfp8ops kernels per step x {args.steps} steps)",
            "pct_fp8_peak": round(100.0 * (value / world) / fp8_peak, 2),
            "fp8_peak_tflops": fp8_peak,
            "fp8_peak_basis": f"2 x {peaks['source']} cuBLAS bf16 burst ({peaks['bf16_tflops']} TFLOP/s)",
            "roofline": roof,
            "kernels": kernels,
            "clocks": clocks,
            "e2e": e2e,
            "cpu_baseline": cpu,
            "unet_train": unet,
            "sweep": annotate_sweep(sweep, peaks) if sweep else None,
        }
        print(json.dumps(line), file=result_out, flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _time_graph_loop(graphs, iters: int) -> float:
    """Average ms per graph replay, CUDA events on the current stream."""
    for g in graphs:
        g.replay()
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record()
    for i in range(iters):
        graphs[i % len(graphs)].replay()
    ev1.record()
    torch.cuda.synchronize()
    return ev0.elapsed_time(ev1) / iters


def time_kernels(args, dev, w, sets) -> dict:
    """Time each hot-path kernel alone (graph-replayed over rotating inputs > L2)."""
    from ctypes import c_void_p

    from fp8_b200 import _lib, ops

    lib = _lib.load()
    stream = lambda: c_void_p(torch.cuda.current_stream(dev).cuda_stream)  # noqa: E731
    p = lambda t: c_void_p(t.data_ptr())  # noqa: E731
    b = args.batch
    cin, cout, h, wd = SHAPE["cin"], SHAPE["cout"], SHAPE["h"], SHAPE["w"]
    # enough rotating operand sets that one pass over them exceeds L2
    per_set = b * h * wd * (cin + cout) * 3
    n_sets = max(4, math.ceil(3 * L2_BYTES / per_set))
    ops_in = []
    for i in range(n_sets):
        x, dy = sets[i % len(sets)] if i < len(sets) else make_inputs(b, dev, seed=777 + i)
        xq, sx = ops.quantize_current(x)
        wq, sw = ops.quantize_current(w)
        dyq, sdy = ops.quantize_current(dy)
        y = torch.empty((b, cout, h, wd), device=dev, dtype=torch.bfloat16, memory_format=torch.channels_last)
        dx = torch.empty((b, cin, h, wd), device=dev, dtype=torch.bfloat16, memory_format=torch.channels_last)
        dw = torch.empty((cout, cin, 3, 3), device=dev, dtype=torch.bfloat16, memory_format=torch.channels_last)
        ws_bytes = lib.fp8_conv3x3_wgrad_workspace_bytes(b, h, wd, cin, cout, 0)
        ws = torch.empty(ws_bytes // 4, device=dev, dtype=torch.float32)
        q_out = torch.empty_like(x, dtype=torch.float8_e4m3fn)
        s_out = torch.empty((), device=dev, dtype=torch.float32)
        qws = torch.empty(lib.fp8_quantize_workspace_bytes(x.numel()) // 4 + 1, device=dev, dtype=torch.float32)
        ops_in.append(dict(x=x, xq=xq, sx=sx, wq=wq, sw=sw, dyq=dyq, sdy=sdy, y=y, dx=dx, dw=dw, ws=ws,
                           q_out=q_out, s_out=s_out, qws=qws))
    torch.cuda.synchronize()

    calls = {
        "quantize_current (quant_resident_kernel: one launch, x read once)": lambda o: _lib.check(lib.fp8_quantize_current(
            p(o["x"]), p(o["q_out"]), p(o["s_out"]), p(o["qws"]), o["qws"].numel() * 4, o["x"].numel(), stream()),
            "q"),
        "conv3x3_fwd (conv_halo_t_fp8_kernel)": lambda o: _lib.check(lib.fp8_conv3x3_fwd(
            p(o["xq"]), p(o["wq"]), p(o["y"]), p(o["sx"]), p(o["sw"]), c_void_p(0), 0, b, h, wd, cin, cout,
            stream()), "fwd"),
        "conv3x3_dgrad (conv_halo_t_fp8_kernel, weights read in place)": lambda o: _lib.check(
            lib.fp8_conv3x3_dgrad_w(p(o["dyq"]), p(o["wq"]), p(o["dx"]), p(o["sdy"]), p(o["sw"]), b, h, wd, cin,
                                    cout, c_void_p(0), 0, stream()), "dgrad"),
        "conv3x3_wgrad (accumulator memset + wgrad_fp8_kernel halo with the bf16 conversion)": lambda o: _lib.check(lib.fp8_conv3x3_wgrad(
            p(o["xq"]), p(o["dyq"]), p(o["dw"]), p(o["sx"]), p(o["sdy"]), b, h, wd, cin, cout, 0, p(o["ws"]),
            o["ws"].numel() * 4, stream()), "wgrad"),
    }
    # One graph per op holding 2 * n_sets back-to-back calls that cycle through
    # the operand sets, so each call reads inputs another call evicted from L2 and
    # the per-replay launch cost of the graph is spread over many calls.
    per_graph = 2 * n_sets
    replays = max(3, min(args.steps, 400) // per_graph)
    out = {}
    side = torch.cuda.Stream(dev)
    for name, fn in calls.items():
        for o in ops_in:
            fn(o)  # eager warm-up
        torch.cuda.synchronize()
        side.wait_stream(torch.cuda.current_stream(dev))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):
            with torch.cuda.graph(g):
                for k in range(per_graph):
                    fn(ops_in[k % n_sets])
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize()
        ms = _time_graph_loop([g], replays) / per_graph
        out[name] = {"ms": round(ms, 6), "calls": replays * per_graph, "operand_sets": n_sets}
        del g
    return out


def _time_calls(fn, n_sets: int, replays: int, dev) -> float:
    """ms per call of fn(i): graph-replayed, cycling over n_sets operand sets (each graph 2 * n_sets calls)."""
    per_graph = 2 * n_sets
    for i in range(n_sets):
        fn(i)
    torch.cuda.synchronize()
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        with torch.cuda.graph(g):
            for k in range(per_graph):
                fn(k % n_sets)
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize()
    ms = _time_graph_loop([g], replays) / per_graph
    del g
    return ms


def time_sweep(args, dev) -> dict:
    """BASELINE configs 1, 3 and 5 (conv at batch 512, widths 128 / 256) and the delayed quantize, op by op.

    Operands rotate over enough sets that one pass exceeds L2; inputs already quantized (the
    quantize is timed on its own).  Work per call: 2*M*N*K FLOP; algorithmic bytes: the e4m3
    operands read once plus the bf16 output written once."""
    from fp8_b200 import ops

    out = {}
    g = torch.Generator(device=dev).manual_seed(0)
    cl = torch.channels_last

    def rnd(shape, std=1.0):
        return (torch.randn(*shape, generator=g, device=dev) * std).to(torch.bfloat16)

    # configs 1 and 3: the FP8 linears (x [M, K] @ W^T, W in nn.Linear [N, K] layout), bias on config 1
    for name, m, k, n, bias in (("linear config 1 (4096x512 @ 512x2048 + bias)", 4096, 512, 2048, True),
                                ("attn qkv config 3 (32768x256 @ 256x768)", 32768, 256, 768, False),
                                ("attn out config 3 (32768x256 @ 256x256)", 32768, 256, 256, False)):
        per_set = m * k + m * n * 2
        n_sets = max(2, -(-3 * 126 * 2**20 // per_set))
        xs = [ops.quantize_current(rnd((m, k))) for _ in range(n_sets)]
        wq, sw = ops.quantize_current(rnd((n, k), 0.02))
        bvec = rnd((n,), 0.01) if bias else None
        epi = ops.EPILOGUE_BIAS if bias else ops.EPILOGUE_NONE
        ms = _time_calls(lambda i: ops.gemm(xs[i][0], wq, xs[i][1], sw, bvec, epi), n_sets, 50, dev)
        out[name] = {"ms": round(ms, 5), "flop": 2.0 * m * n * k, "bytes": m * k + n * k + 2 * m * n + (2 * n if bias else 0)}
        del xs
        # the op end to end on bf16 inputs: the pair quantize of X and W (current scaling), then the GEMM
        xb = [rnd((m, k)) for _ in range(n_sets)]
        wb = rnd((n, k), 0.02)
        ms_q = _time_calls(lambda i: ops.quantize_current_pair(xb[i], wb), n_sets, 50, dev)
        out[f"{name}: quantize X + W"] = {"ms": round(ms_q, 5), "flop": None, "bytes": 3 * (m * k + n * k)}

        def full(i):
            xq, sx, wq2, sw2 = ops.quantize_current_pair(xb[i], wb)
            return ops.gemm(xq, wq2, sx, sw2, bvec, epi)

        ms_f = _time_calls(full, n_sets, 50, dev)
        out[f"{name}: whole op (quantize X + W, GEMM)"] = {
            "ms": round(ms_f, 5), "flop": 2.0 * m * n * k,
            "bytes": 2 * (m * k + n * k) + 2 * m * n + (2 * n if bias else 0)}
        del xb

    # the quantize at config 2's X and at 4x that size (batch 512), which separates the fixed
    # cost of a launch (start-up, first bytes, tail) from the streaming rate: delayed is one pass
    # (2 B read + 1 B written per element), current reads x twice (or once, shared-memory
    # resident, where the per-SM shares fit) and writes once; both quoted on 3 B/element
    prev = torch.tensor(0.01, device=dev)
    for b, n_sets in ((128, 4), (512, 2)):
        n_el = b * 128 * 32 * 32
        xs = [rnd((b, 128, 32, 32)).contiguous(memory_format=cl) for _ in range(n_sets)]
        tag = f"config 2 X, batch {b} ({n_el / 1e6:.1f} M elements)"
        ms = _time_calls(lambda i: ops.quantize_delayed(xs[i], prev), n_sets, 50, dev)
        out[f"quantize delayed {tag}"] = {"ms": round(ms, 5), "flop": None, "bytes": 3 * n_el}
        ms = _time_calls(lambda i: ops.quantize_current(xs[i]), n_sets, 50, dev)
        out[f"quantize current {tag}"] = {"ms": round(ms, 5), "flop": None, "bytes": 3 * n_el}
        if b == 512:  # too large to stay in shared memory: two passes read x twice (5 B/element)
            out[f"quantize current {tag}"]["bytes_moved"] = 5 * n_el
        del xs
        torch.cuda.empty_cache()
    # config 5: the config-2 conv at batch 512, widths 128 and 256 (last: these run the GPU at its
    # power limit, and the short kernels above are timed before that)
    for c in (128, 256):
        b, hw = 512, 32
        n_sets = 2
        xs = [ops.quantize_current(rnd((b, c, hw, hw)).contiguous(memory_format=cl)) for _ in range(n_sets)]
        dys = [ops.quantize_current(rnd((b, c, hw, hw), 1e-2).contiguous(memory_format=cl))
               for _ in range(n_sets)]
        wq, sw = ops.quantize_current(rnd((c, c, 3, 3), 0.05).contiguous(memory_format=cl))
        flops = 2.0 * b * hw * hw * c * 9 * c
        name = f"conv3x3 B=512 {c}->{c} 32x32"
        fns = {
            "fwd": lambda i: ops.conv3x3_fwd(xs[i][0], wq, xs[i][1], sw),
            "dgrad": lambda i: ops.conv3x3_dgrad(dys[i][0], wq, dys[i][1], sw),
            "wgrad": lambda i: ops.conv3x3_wgrad(xs[i][0], dys[i][0], xs[i][1], dys[i][1]),
        }
        for op, fn in fns.items():
            ms = _time_calls(fn, n_sets, 20, dev)
            out[f"{name} {op}"] = {"ms": round(ms, 5), "flop": flops, "bytes": None}
        del xs, dys
        torch.cuda.empty_cache()

    return out


def annotate_sweep(sweep: dict, peaks: dict) -> dict:
    """Adds TFLOP/s and GB/s with their fractions of the measured peaks (FP8 = 2 x bf16 burst)."""
    fp8_peak = 2.0 * peaks["bf16_tflops"]
    res = {}
    for name, r in sweep.items():
        e = dict(r)
        s = r["ms"] * 1e-3
        if r["flop"]:
            e["tflops"] = round(r["flop"] / s / 1e12, 1)
            e["frac_fp8_peak"] = round(e["tflops"] / fp8_peak, 4)
        if r["bytes"]:
            e["gbs"] = round(r["bytes"] / s / 1e9, 1)
            e["frac_hbm"] = round(e["gbs"] / peaks["hbm_gbs"], 4)
        if r.get("bytes_moved"):  # the bytes the kernels actually move, where they exceed the algorithmic ones
            e["gbs_moved"] = round(r["bytes_moved"] / s / 1e9, 1)
            e["frac_hbm_moved"] = round(e["gbs_moved"] / peaks["hbm_gbs"], 4)
        res[name] = e
    return res


def roofline(kernels: dict, peaks: dict, batch: int) -> dict | None:
    if not kernels:
        return None
    fp8_peak = 2.0 * peaks["bf16_tflops"]
    flops = conv_flops(batch)
    cin, cout, h, w = SHAPE["cin"], SHAPE["cout"], SHAPE["h"], SHAPE["w"]
    pix = batch * h * w
    algo = {
        "quantize_current (quant_resident_kernel: one launch, x read once)": ("hbm", pix * cin * 3.0),  # read bf16 once + write e4m3
        "conv3x3_fwd (conv_halo_t_fp8_kernel)": ("tensor", flops),
        "conv3x3_dgrad (conv_halo_t_fp8_kernel, weights read in place)": ("tensor", flops),
        "conv3x3_wgrad (accumulator memset + wgrad_fp8_kernel halo with the bf16 conversion)": ("tensor", flops),
    }
    name = max(kernels, key=lambda k: kernels[k]["ms"])
    bound, work = algo[name]
    sec = kernels[name]["ms"] * 1e-3
    traffic = ncu_traffic().get(name)
    if bound == "tensor":
        achieved = work / sec / 1e12
        return {"kernel": name, "bound": "tensor", "achieved": round(achieved, 1), "peak": fp8_peak,
                "unit": "TFLOP/s", "frac": round(achieved / fp8_peak, 4), "traffic": traffic,
                "peak_note": f"FP8 dense = 2 x {peaks['source']} bf16 burst",
                "algorithmic": f"2*M*N*K = {work:.4g} FLOP per launch"}
    achieved = work / sec / 1e9
    return {"kernel": name, "bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"],
            "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": traffic,
            "peak_note": f"{peaks['source']} HBM copy bandwidth",
            "algorithmic": f"3 B/elem = {work:.4g} B per call"}


def time_unet(args, dev, world, fp8: bool, scaling: str = "delayed", skip_empty: bool = False) -> dict:
    """BASELINE configs 4/5: the CUDA-graph UNet training step (B images per GPU,
    data parallel with the bucketed bf16 all-reduce when world > 1).

    ``skip_empty``: delayed scaling where an all-zero tensor records scale 0 in its
    history (the configuration that meets the 200-step 2 % loss bar; the reference's
    semantics record 1.0, which runs the same kernels at the same speed)."""
    import torch.distributed as dist

    from fp8_b200.train import GraphedTrainStep, TrainConfig, build_model, images_per_second

    rank = int(os.environ.get("RANK", "0"))
    # the B200 path: FP8 convs + fused norm/activation ops; the comparison: the
    # reference's bf16 model with its torch ops
    model = build_model(fp8=fp8, scaling=scaling, device=dev, seed=0, fused_norm=fp8, skip_empty=fp8 and skip_empty)
    cfg = TrainConfig(batch_size=args.batch, fused_optimizer=fp8)  # the reference-ops arm keeps torch's AdamW
    if args.bucket_mb:
        cfg.allreduce_bucket_mb = args.bucket_mb
    step = GraphedTrainStep(model, cfg, dev)
    torch.manual_seed(100 + rank)
    step.prepare()
    g = torch.Generator().manual_seed(200 + rank)
    images = [(torch.rand(args.batch, 3, 32, 32, generator=g) * 2 - 1).to(memory_format=torch.channels_last)
              .to(dev) for _ in range(2)]
    for i in range(3):
        step.step(images[i % 2])
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record()
    for i in range(args.unet_steps):
        step.step(images[i % 2])
    ev1.record()
    torch.cuda.synchronize()
    t = torch.tensor([ev0.elapsed_time(ev1)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item()) / args.unet_steps
    loss = step.loss_acc.item() / (args.unet_steps + 3)
    n_fp8 = sum(1 for m in model.modules() if hasattr(m, "uses_fp8"))
    allreduce = step.dp.bytes_per_step() if step.dp is not None else 0
    step.release()
    del step, model
    torch.cuda.synchronize()
    return {"metric": "UNet train imgs/s", "value": round(images_per_second(args.batch, world, ms), 1),
            "unit": "imgs/s", "ms_per_step": round(ms, 4), "steps": args.unet_steps, "batch_per_gpu": args.batch,
            "global_batch": args.batch * world, "n_gpus": world, "mean_loss": round(loss, 4),
            "fp8": (f"whitelisted 3x3 convs, {scaling} scaling"
                    + (", all-zero tensors record scale 0 in the histories" if skip_empty and scaling == "delayed"
                       else "") if fp8 else "off (bf16 autocast)"),
            "norm_activation": ("fused GroupNorm/FiLM/SiLU/dropout kernels (the FP8 conv input written as e4m3), "
                                "LayerNorm kernels in the attention blocks, fused nearest resampling + skip "
                                "concatenation" if fp8 else "torch ops (reference)"),
            "scale_history": ("device-side (the casts read and update the histories; batched weight quantize)"
                              if fp8 and scaling == "delayed" else None),
            "optimizer": ("clip + AdamW + EMA in one pass (fp8_b200.optim)" if fp8
                          else "clip_grad_norm_ + torch fused AdamW + foreach EMA"),
            "conv_modules": n_fp8, "allreduce_bf16_bytes_per_step": allreduce,
            "step": "noise + UNet fwd/bwd (bf16 autocast) + grad all-reduce + clip 1.0 + AdamW 2e-4 + EMA, "
                    "one CUDA graph replay"}


def time_e2e(args, dev, world, conv_api, step_flops) -> dict:
    """Same step through the reference-facing API with pinned host buffers."""
    import torch.distributed as dist

    b = args.batch
    cin, cout, h, w = SHAPE["cin"], SHAPE["cout"], SHAPE["h"], SHAPE["w"]

    # Host buffers are contiguous NHWC ([Cout][3][3][Cin] for weights), i.e. the
    # channels_last memory order, so every transfer is one contiguous DMA; the
    # logical NCHW views the API takes are permutations of them.
    def pinned(*shape):
        return torch.empty(shape, dtype=torch.bfloat16, pin_memory=True)

    nhwc = (0, 2, 3, 1)
    nchw = (0, 3, 1, 2)
    x_h, dy_h = pinned(b, h, w, cin), pinned(b, h, w, cout)
    x0, dy0 = make_inputs(b, "cpu", seed=4242)
    x_h.copy_(x0.permute(*nhwc))
    dy_h.copy_(dy0.permute(*nhwc))
    w_h = pinned(cout, 3, 3, cin)
    w_h.copy_(make_weight("cpu").permute(*nhwc))
    y_h, dx_h, dw_h = pinned(b, h, w, cout), pinned(b, h, w, cin), pinned(cout, 3, 3, cin)
    h2d = x_h.numel() * 2 + w_h.numel() * 2 + (dy_h.numel() * 2 if args.workload == "layer" else 0)
    d2h = y_h.numel() * 2 + ((dx_h.numel() + dw_h.numel()) * 2 if args.workload == "layer" else 0)
    train = args.workload == "layer"

    # Steps are pipelined over three streams, as a serving loop would run them:
    # the host->device copy of step i+1 and the device->host copy of step i-1
    # overlap the compute of step i (the two copy directions use separate copy
    # engines).  Every step still copies all of its inputs in and all of its
    # results out inside the timed region.
    comp = torch.cuda.current_stream(dev)
    copy_in, copy_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    slots = 2
    x_d = [torch.empty(x_h.shape, dtype=torch.bfloat16, device=dev) for _ in range(slots)]
    w_d = [torch.empty(w_h.shape, dtype=torch.bfloat16, device=dev) for _ in range(slots)]
    dy_d = [torch.empty(dy_h.shape, dtype=torch.bfloat16, device=dev) for _ in range(slots)]
    ready = [torch.cuda.Event() for _ in range(slots)]
    free = [torch.cuda.Event() for _ in range(slots)]

    def h2d_step(i):
        s = i % slots
        with torch.cuda.stream(copy_in):
            copy_in.wait_event(free[s])  # step i - slots has finished reading this slot
            x_d[s].copy_(x_h, non_blocking=True)
            w_d[s].copy_(w_h, non_blocking=True)
            if train:
                dy_d[s].copy_(dy_h, non_blocking=True)
            ready[s].record(copy_in)

    def compute_step(i):
        s = i % slots
        comp.wait_event(ready[s])
        x = x_d[s].permute(*nchw).requires_grad_(train)
        wt = w_d[s].permute(*nchw).requires_grad_(train)
        y = conv_api(x, wt)
        outs = [(y, y_h)]
        if train:
            gx, gw = torch.autograd.grad(y, (x, wt), dy_d[s].permute(*nchw))
            outs += [(gx, dx_h), (gw, dw_h)]
        free[s].record(comp)
        copy_out.wait_stream(comp)
        with torch.cuda.stream(copy_out):
            for t, host in outs:
                host.copy_(t.permute(*nhwc), non_blocking=True)
                t.record_stream(copy_out)

    def run(n):
        copy_in.wait_stream(comp)
        for i in range(min(slots, n)):
            h2d_step(i)
        for i in range(n):
            compute_step(i)
            if i + slots < n:
                h2d_step(i + slots)
        comp.wait_stream(copy_out)
        comp.wait_stream(copy_in)

    run(3)
    torch.cuda.synchronize()
    k = max(5, min(args.steps, 50))
    if world > 1:
        dist.barrier()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record()
    run(k)
    ev1.record()
    torch.cuda.synchronize()
    t = torch.tensor([ev0.elapsed_time(ev1)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    return {"value": round(world * step_flops * k / (ms * 1e-3) / 1e12, 3), "unit": UNIT,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": k,
            "ms_per_step": round(ms / k, 4),
            "path": ("fp8_kernels.triton_conv2d_fp8 + torch.autograd.grad, pinned host buffers; "
                     "copies in / compute / copies out of consecutive steps on three streams")}


# ============================================================================ CPU oracle (baseline / reference arm)
def _oracle_step(oracle, x, w, dy, workload: str):
    xq, sx = oracle.quantize_tensor(x)
    wq, sw = oracle.quantize_tensor(w)
    oracle.conv_fwd(xq, wq, sx, sw)
    if workload == "layer":
        dyq, sdy = oracle.quantize_tensor(dy)
        oracle.conv_dx(dyq, wq, sdy, sw)
        oracle.conv_dw(xq, dyq, sx, sdy)


def _cpu_setup():
    torch.set_num_threads(os.cpu_count() or 1)
    import fp8_oracle as oracle

    return oracle


def cpu_oracle_baseline(args, seconds: float, batch: int = 4) -> dict:
    """The CPU restatement of the reference (oracle port) on a bounded sample."""
    oracle = _cpu_setup()
    x, dy = make_inputs(batch, "cpu", seed=99)
    w = make_weight("cpu")
    _oracle_step(oracle, x, w, dy, args.workload)  # warm-up
    n = 0
    t0 = time.perf_counter()
    while True:
        _oracle_step(oracle, x, w, dy, args.workload)
        n += 1
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    flops = (3 if args.workload == "layer" else 1) * conv_flops(batch) * n
    return {"value": round(flops / dt / 1e12, 5), "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{n} passes of the step at batch {batch} (of 128), {dt:.1f} s, oracle/fp8_oracle.py "
                      "(numpy e4m3 quantize + torch fp32 CPU conv)"}


def run_reference(args) -> None:
    """--impl reference: the reference's CPU path (the oracle port) on this host's cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    oracle = _cpu_setup()
    w = make_weight("cpu")
    # size the per-step sample so that warm-up + steps stay within ~2 minutes
    x1, dy1 = make_inputs(1, "cpu", seed=5)
    t0 = time.perf_counter()
    _oracle_step(oracle, x1, w, dy1, args.workload)
    t1 = time.perf_counter() - t0
    total_steps = max(1, args.steps + args.warmup)
    batch = int(max(1, min(args.batch, 120.0 / (total_steps * max(t1, 1e-4)))))
    x, dy = make_inputs(batch, "cpu", seed=6)
    for _ in range(args.warmup):
        _oracle_step(oracle, x, w, dy, args.workload)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        _oracle_step(oracle, x, w, dy, args.workload)
    dt = time.perf_counter() - t0
    step_flops = (3 if args.workload == "layer" else 1) * conv_flops(batch)
    value = step_flops * args.steps / dt / 1e12
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 5),
        "unit": UNIT,
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")),
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(dt * 1e3 / max(args.steps, 1), 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "e4m3 (fp32 accumulate, bf16 out)",
        "data": "synthetic (seeded randn activations / dY, nn.Conv2d default-init weights)",
        "config": {
            "workload": ("conv3x3_fp8_layer_fwd_dgrad_wgrad" if args.workload == "layer" else "conv3x3_fp8_fwd"),
            "baseline_config": "configs[1]: FP8 3x3 conv B=128 128->128 32x32 (M=131072 N=128 K=1152)",
            "batch_per_step_sample": batch,
            **SHAPE,
        },
        "cpu_baseline": {"value": round(value, 5), "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
                         "sample": f"batch {batch} of 128 per step (the reference has no CPU implementation of "
                                   "its Triton kernels; this is the oracle port of their arithmetic)"},
        "e2e": {"value": round(value, 5), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
