"""MoE-layer benchmark (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload prefill|decode|pr1|fine|sweep]
                    [--impl ours|reference]

Default workload: the prefill layer (16384 tokens, d_model 4096, d_ff 14336,
8 experts top-2, INT4 group-128 SwiGLU experts, capacity factor 1.25) on one GPU;
with N > 1 ranks (torchrun) the experts are sharded expert-parallel, tokens are
sharded by rank and exchanged over NVLink peer memory (``--exchange peer``, the
default) or NCCL all-to-all (``--exchange nccl``) (strong scaling: the 16384
tokens are split over the ranks).

value     MoE-layer tokens/s of the whole job, device-timed (CUDA events, max over ranks),
          inputs resident in HBM.
e2e       the same metric through ``MoELayer.forward`` with the input copied from pinned
          host memory and the output read back every step.
roofline  the dominant kernel (grouped W4A16 gate/up GEMM), device-timed inside the timed
          steps.  Compute-bound workloads (prefill, pr1, fine): algorithmic FLOPs per launch
          against the measured bf16 tensor peak -- the burst figure when the sampled SM clock
          stayed at its maximum, the sustained (power-capped) one otherwise; both fractions are
          printed.  Weight-stream-bound workloads (decode): algorithmic bytes per launch (the
          packed weights, scales and zeros of every expert with a kept row, plus activation
          rows in and out) against the measured HBM copy bandwidth.
cpu_baseline  the reference's own CPU path (its torch-routing MoELayer in fp32, restated
          in oracle/torch_path.py and pinned against the reference's outputs) on every host
          thread, rank 0 only, on a bounded token sample (about 10 s of work).

``--impl reference`` times that CPU implementation alone on the same workload and
prints its line with ``"impl": "reference"``.
"""

from __future__ import annotations

import argparse
import dataclasses
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "llm-serving-kernel-optimization_b200"))

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "MoE-layer tokens/s"
UNIT = "tokens/s"

# DRAM bytes (read + write) per launch of the dominant kernel (the gate/up GEMM),
# averaged over the launches of the timed loop in one ncu capture of this bench's
# own command:
#   ncu --metrics gpu__time_duration.sum,dram__bytes_read.sum,dram__bytes_write.sum \
#       --clock-control none --profile-from-start off \
#       python bench.py [--workload decode] --steps 2 --warmup 3 --no-cpu
# prefill: 980.4 MB read (algorithmic 757: token rows 268 + weights 489) and 911.4 MB
# written (940 of intermediate rows, part still in L2 at the end); decode (the stage is
# the token-term pass and the 8-bit-operand GEMM): 1.1 + 489.7 MB read (the weights of
# the 8 experts), 2.7 MB written.
NCU_TRAFFIC = {
    "prefill": 980.4e6 + 911.4e6,
    "decode": 1.1e6 + 489.7e6 + 2.7e6,
}


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (FileNotFoundError, OSError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=2)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# distributed helpers
# ---------------------------------------------------------------------------
def init_dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import datetime
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return ws, rank, local


def barrier(ws):
    if ws > 1:
        torch.distributed.barrier()


def max_over_ranks(v: float, ws: int) -> float:
    if ws == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# CPU oracle timing (baseline / reference arm)
# ---------------------------------------------------------------------------
def cpu_port_setup(w):
    """fp32 inputs of the CPU baseline (untimed): dequantized INT4 experts, gate weight,
    gate bias and the workload's tokens, on the host."""
    from lightning_router.quantization.pack_weights import dequantize_tensor
    from lightning_router.workloads import make_layer
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    t = make_layer(w, device=dev, gen_device=dev)
    # nn.Linear layout (out, in), as the reference's unquantized experts hold them
    experts = [{n: dequantize_tensor(q, s, z, w.group_size, s.shape[1]).float().t().contiguous()
                .cpu() for n, (q, s, z) in ex.items()} for ex in t.experts]
    x = t.x.float().cpu()
    wg = t.gate_w.float().cpu()
    bias = None if t.bias is None else t.bias.float().cpu()
    del t
    if dev == "cuda":
        torch.cuda.empty_cache()
    return x, wg, bias, experts


def cpu_port_step(w, x, wg, bias, experts):
    # the reference's torch-routing MoELayer restated (the timed baseline, not the product)
    from oracle import torch_path
    return torch_path.moe_layer(x, wg, experts, w.top_k, gated=w.activation == "swiglu",
                                bias=bias)


def run_cpu(w, steps: int, warmup: int, step_budget_s: float = 25.0):
    """Times the reference's CPU path (its torch-routing MoELayer in fp32, restated in
    ``oracle/torch_path.py``) with every host thread; returns (tokens/s, sample, threads).

    Each step runs the first ``sample`` tokens of the workload, ``sample`` sized by an
    untimed calibration step on 256 tokens so that one step takes at most about
    ``step_budget_s`` seconds (at most the whole workload; the calibration's small
    batches run slower per token, so the timed step is usually shorter).  The torch path applies no capacity, so the work
    per token does not depend on the sample size.
    """
    torch.set_num_threads(os.cpu_count() or 1)
    threads = torch.get_num_threads()
    with torch.no_grad():
        x, wg, bias, experts = cpu_port_setup(w)
        n0 = min(w.tokens, 256)
        t0 = time.perf_counter()
        cpu_port_step(w, x[:n0], wg, bias, experts)
        rate = n0 / max(time.perf_counter() - t0, 1e-9)
        sample = int(min(w.tokens, max(n0, rate * step_budget_s)))
        sample = max(n0, sample - sample % 64) if sample < w.tokens else w.tokens
        xs = x[:sample].contiguous()
        for _ in range(max(0, warmup)):
            cpu_port_step(w, xs, wg, bias, experts)
        t0 = time.perf_counter()
        for _ in range(max(1, steps)):
            cpu_port_step(w, xs, wg, bias, experts)
        dt = time.perf_counter() - t0
    n = max(1, steps)
    desc = (f"{n} step(s) of the first {sample} of {w.tokens} tokens through the reference's "
            f"torch-routing MoELayer path restated in fp32 (gate, softmax, top-k, per-expert "
            f"mask + index_add_, dequantized INT4 experts as fp32 matmuls, no capacity), "
            f"torch on {threads} host threads; weights dequantized outside the timed region")
    return sample * n / dt, desc, threads


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def workload_desc(w):
    act = "SwiGLU" if w.activation == "swiglu" else "up-SiLU-down"
    s = (f"{w.name}: {w.tokens} tokens, d_model {w.d_model}, d_ff {w.d_ff}, {w.experts} experts "
         f"top-{w.top_k}, INT4 g{w.group_size} {act}, cf {w.capacity_factor}")
    if w.zipf_s:
        s += f", Zipf({w.zipf_s}) gate bias"
    return s


def stage_times(events, steps):
    """Average per-stage milliseconds from (name, event) marks of `steps` forwards."""
    acc = {}
    prev = None
    for name, ev in events:
        if name == "begin":
            prev = ev
            continue
        if prev is not None:
            acc.setdefault(name, []).append(prev.elapsed_time(ev))
        prev = ev
    return {k: sum(v) / len(v) for k, v in acc.items()}


def gemm_roofline(w, layer, model, x, st, clk, peaks, peak_kind, workload, ws, rank):
    """Roofline of the dominant kernel, the grouped gate/up GEMM (its stage time).

    Per launch: FLOPs = 2 * kept rows * (2 if SwiGLU else 1) * d_model * d_ff;
    algorithmic bytes = packed weights + scales + zeros of every local expert with a
    kept row + kept rows in (d_model fp16) and out (d_ff fp16).  The bound is the
    one whose roof is lower at that arithmetic intensity.
    """
    gated = w.activation == "swiglu"
    if hasattr(model, "last_kept_per_expert"):
        kept_e = model.last_kept_per_expert()
    else:
        _, plan = layer.route(x)
        kept_e = plan.kept_counts.cpu().tolist()
    kept = int(sum(kept_e))
    nmat = 2 if gated else 1
    d, f, g = w.d_model, w.d_ff, w.group_size
    per_expert = nmat * (d * f // 2 + (d // g) * f * 2 + (d // g) * (f // 8) * 4)
    gemm_bytes = sum(per_expert for c in kept_e if c) + kept * (d + f) * 2
    gemm_flops = 2 * kept * nmat * d * f
    gemm_ms = st.get("ffn_in")
    burst = float(peaks.get("bf16_tflops"))
    sustained = float(peaks.get("bf16_tflops_sustained", burst))
    hbm = float(peaks["hbm_gbs"])
    sm, smax = clk.get("sm_mhz"), clk.get("sm_max_mhz")
    at_max = sm is not None and smax and sm >= 0.95 * smax
    tensor_peak = burst if at_max or sm is None else sustained
    hbm_bound = gemm_flops / max(gemm_bytes, 1) < tensor_peak * 1e12 / (hbm * 1e9)
    out = {"kernel": "w4a16 grouped GEMM, gate/up (" + ("SwiGLU" if gated else "SiLU") +
                     " epilogue)",
           "launch_ms": gemm_ms, "flops_per_launch": gemm_flops,
           "bytes_per_launch": gemm_bytes,
           "traffic": NCU_TRAFFIC.get(workload) if ws == 1 else None,
           "stage_ms": {k: round(v, 4) for k, v in st.items()}}
    if not gemm_ms:
        return {"bound": "hbm" if hbm_bound else "tensor", "achieved": None, **out}
    tflops = gemm_flops / (gemm_ms / 1e3) / 1e12
    gbs = gemm_bytes / (gemm_ms / 1e3) / 1e9
    if hbm_bound:
        out.update({"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s",
                    "frac": gbs / hbm, "peak_kind": f"{peak_kind} HBM copy bandwidth",
                    "tflops": tflops})
    else:
        out.update({"bound": "tensor", "achieved": tflops, "peak": tensor_peak,
                    "unit": "TFLOP/s", "frac": tflops / tensor_peak,
                    "peak_kind": (f"{peak_kind} bf16 " + ("burst" if tensor_peak == burst
                                                          else "sustained") +
                                  f" (median SM clock {sm} of {smax} MHz)"),
                    "frac_burst": tflops / burst, "frac_sustained": tflops / sustained,
                    "gbs": gbs})
    return out


def run_gpu(args, ws, rank, local):
    from lightning_router.kernels.expert_routing import SMALL_BATCH_TOKENS
    from lightning_router.workloads import WORKLOADS, build_layer
    w = WORKLOADS[args.workload]
    if args.tokens:
        w = dataclasses.replace(w, tokens=args.tokens)
    dev = torch.device("cuda", local)
    peaks, peak_kind = _peaks()

    if ws > 1:
        from lightning_router.serving.ep import ExpertParallelMoE
        layer, t = build_layer(w, device=dev, gen_device=dev)
        model = ExpertParallelMoE.from_layer(layer, ws, rank, exchange=args.exchange)
        T_local = w.tokens // ws
        x = t.x[rank * T_local:(rank + 1) * T_local].contiguous()
        del t
        fwd = model.forward
        stage_owner = model
        parallel = f"ep{ws}"
    else:
        layer, t = build_layer(w, device=dev, gen_device=dev)
        x = t.x
        model = layer
        fwd = layer.forward
        stage_owner = layer
        T_local = w.tokens
        parallel = "ep1"
    torch.cuda.synchronize()

    # warm-up
    for _ in range(args.warmup):
        fwd(x)
    torch.cuda.synchronize()
    barrier(ws)

    # --graph (one GPU): the layer forward captured once as a CUDA graph and
    # replayed each step (same kernels and buffers; no per-launch host overhead).
    # Stage times then come from an extra eager pass after the timed region.
    graph = None
    if args.graph and ws == 1:
        static_x = x.clone()
        gpool = torch.cuda.graph_pool_handle()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, pool=gpool):
            static_out, _static_aux = layer(static_x)
        torch.cuda.synchronize()
        eager_fwd = fwd

        def fwd(xi, _g=graph, _x=static_x, _o=static_out):
            if xi is not _x:
                _x.copy_(xi)
            _g.replay()
            return _o, _static_aux
        x = static_x
        for _ in range(args.warmup):
            fwd(x)
        torch.cuda.synchronize()

    def fwd_e2e(xi):
        # the pipeline copies each output back while the next step runs: hand it
        # a copy of the graph's static output buffer
        out, aux = fwd(xi)
        return (out.clone(), aux) if graph is not None else (out, aux)

    # timed region (device time, max over ranks).  cudaProfilerStart/Stop bracket
    # it so `ncu --profile-from-start off` lists exactly the timed launches.  No
    # stage events are recorded in it: the stage times come from a separate eager
    # pass afterwards.
    stage_owner.stage_events = None
    clocks = ClockSampler(torch.cuda.current_device() if "CUDA_VISIBLE_DEVICES" not in os.environ
                          else local)
    clocks.start()
    time.sleep(0.3)
    torch.cuda.synchronize()
    barrier(ws)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    wall0 = time.perf_counter()
    torch.cuda.cudart().cudaProfilerStart()
    start.record()
    for _ in range(args.steps):
        fwd(x)
    end.record()
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStop()
    wall = time.perf_counter() - wall0
    barrier(ws)
    clk = clocks.stop()
    ms_local = start.elapsed_time(end)
    ms = max_over_ranks(ms_local, ws)
    # stage times: an extra eager pass (after one untimed forward, so it times
    # warm launches); every rank runs it, so the exchange's collectives match
    eager = eager_fwd if graph is not None else fwd
    eager(x)
    torch.cuda.synchronize()
    stage_owner.stage_events = []
    n_stage = min(args.steps, 10)
    for _ in range(n_stage):
        eager(x)
    torch.cuda.synchronize()
    st = stage_times(stage_owner.stage_events, n_stage)
    stage_owner.stage_events = None
    value = w.tokens * args.steps / (ms / 1e3)

    roofline = gemm_roofline(w, layer, model, x, st, clk, peaks, peak_kind, args.workload, ws,
                             rank)

    # end to end through the public API with host buffers (pinned), max over ranks: every
    # step copies its input from pinned host memory and its output back, through the
    # package's serving loop (copies on their own stream, overlapping the next / previous
    # step's compute)
    from lightning_router.serving.pipeline import HostPipeline
    xh = x.cpu().pin_memory()
    outh = [torch.empty_like(xh).pin_memory() for _ in range(2)]
    pipe = HostPipeline(fwd_e2e, x, dev)
    pipe.run([xh] * max(1, args.warmup), [outh[i % 2] for i in range(max(1, args.warmup))])
    torch.cuda.synchronize()
    barrier(ws)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    pipe.run([xh] * args.steps, [outh[i % 2] for i in range(args.steps)])
    e1.record()
    torch.cuda.synchronize()
    barrier(ws)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), ws)
    e2e = {"value": w.tokens * args.steps / (e2e_ms / 1e3), "unit": UNIT,
           "h2d_bytes_per_step": int(xh.numel() * 2) * ws,
           "d2h_bytes_per_step": int(outh[0].numel() * 2) * ws,
           "overlap": "host copies on a second stream, double-buffered (HostPipeline)",
           "api": "MoELayer.forward" if ws == 1 else "ExpertParallelMoE.forward"}

    # gate, route, permute/route_rows, 2 GEMMs, combine; the peer exchange adds
    # its plan and gather kernels; one GPU with at most 256 tokens runs the gate
    # inside the route launch
    if ws > 1:
        launches_per_step = 8 if args.exchange == "peer" else 6
    else:
        launches_per_step = 5 if w.tokens <= SMALL_BATCH_TOKENS else 6
    # segments of at most 32 rows on 8-bit operands: each GEMM adds its token-term pass
    from lightning_router.kernels import quantized_matmul as qm
    from lightning_router.kernels.expert_routing import expert_capacity
    cap = expert_capacity(T_local * ws * w.top_k, w.experts, w.capacity_factor)
    if qm.INT8_OPERANDS and cap <= 32 and w.group_size % 128 == 0 and \
            w.d_model % 128 == 0 and w.d_ff % 128 == 0:
        launches_per_step += 2
    if ws > 1:
        barrier(ws)
        model.close()
    result = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": workload_desc(w), "global_batch": w.tokens, "seq_len": None,
                   "parallelism": parallel,
                   **({"gemm_operands": "f16"} if args.operands == "f16" else {}),
                   **({"exchange": args.exchange} if ws > 1 else {}),
                   **({"cuda_graph": True} if graph is not None else {}),
                   "l2": "inputs larger than L2 (INT4 weights "
                         f"{w.experts} experts, activations {w.tokens * w.d_model * 2 >> 20} MiB)"},
        "e2e": e2e,
        "roofline": roofline,
        "clocks": clk,
        "gpu_launches": launches_per_step * args.steps,
        "wall_s_timed": wall,
    }
    if ws == 1 and rank == 0 and not args.no_cpu:
        v, desc, cores = run_cpu(w, steps=1, warmup=0)
        result["cpu_baseline"] = {"value": v, "unit": UNIT, "cores": cores, "kind": "port",
                                  "sample": desc}
    return result


def run_sweep(args, ws, rank, local):
    """Dispatch/combine sweep (routing kernels only): HBM GB/s against the measured copy peak.

    Each step is one fused top-k gating + dispatch (route + permute kernels) from given
    fp32 logits, then one combine with identity experts.  L2 is flushed between steps
    (a 512 MiB write outside the timed events).
    """
    from lightning_router.kernels.expert_routing import combine, topk_gating_dispatch
    from lightning_router.workloads import (SWEEP_D, SWEEP_E, SWEEP_K, SWEEP_TOKENS,
                                            combine_bytes, dispatch_bytes, sweep_inputs)
    dev = torch.device("cuda", local)
    peaks, peak_kind = _peaks()
    hbm = float(peaks["hbm_gbs"])
    flush = torch.empty(512 << 20, dtype=torch.uint8, device=dev)
    tokens = SWEEP_TOKENS if args.tokens is None else (args.tokens,)
    rows = []
    for cf in (1.0, 2.0):
        for i, T in enumerate(tokens):
            x, logits = sweep_inputs(T, SWEEP_TOKENS.index(T) if T in SWEEP_TOKENS else 0,
                                     device=dev, gen_device=dev)
            times = {"dispatch": [], "combine": []}
            plan = None
            for it in range(args.warmup + args.steps):
                flush.zero_()
                e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
                e[0].record()
                plan = topk_gating_dispatch(x, logits, SWEEP_K, cf, fill_dropped=False)
                e[1].record()
                out = combine(plan.permuted, plan.gate_weights, plan.slot_pos, T, SWEEP_K)
                e[2].record()
                torch.cuda.synchronize()
                if it >= args.warmup:
                    times["dispatch"].append(e[0].elapsed_time(e[1]))
                    times["combine"].append(e[1].elapsed_time(e[2]))
            kept = int(plan.kept_counts.sum())
            S = T * SWEEP_K
            db = dispatch_bytes(T, SWEEP_D, SWEEP_E, S, kept)
            cb = combine_bytes(T, SWEEP_D, S, kept)
            dms = statistics.median(times["dispatch"])
            cms = statistics.median(times["combine"])
            rows.append({"tokens": T, "cf": cf, "kept_slots": kept,
                         "dispatch_ms": dms, "dispatch_gbs": db / dms / 1e6,
                         "combine_ms": cms, "combine_gbs": cb / cms / 1e6,
                         "dispatch_bytes": db, "combine_bytes": cb})
            del x, logits, plan, out
    head = max(rows, key=lambda r: (r["tokens"], -r["cf"]))
    head = [r for r in rows if r["tokens"] == head["tokens"] and r["cf"] == 1.0][0]
    return {
        "metric": "dispatch HBM GB/s", "value": head["dispatch_gbs"], "unit": "GB/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": head["dispatch_ms"], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": f"dispatch/combine sweep: d_model {SWEEP_D}, {SWEEP_E} experts "
                               f"top-{SWEEP_K}, logits N(0,1) given; headline T={head['tokens']} "
                               "cf 1.0", "l2": "flushed between steps (512 MiB write)"},
        "roofline": {"kernel": "route + permute (dispatch)", "bound": "hbm",
                     "achieved": head["dispatch_gbs"], "peak": hbm, "unit": "GB/s",
                     "frac": head["dispatch_gbs"] / hbm, "peak_kind": f"{peak_kind} copy",
                     "traffic": None, "combine_gbs": head["combine_gbs"],
                     "combine_frac": head["combine_gbs"] / hbm},
        "sweep": rows,
        "gpu_launches": 3 * args.steps * len(rows),
    }


def run_reference(args, ws, rank):
    from lightning_router.workloads import WORKLOADS
    w = WORKLOADS["prefill" if args.workload == "sweep" else args.workload]
    if rank != 0:
        return None
    # the whole --steps/--warmup run stays within about three minutes
    per_step = min(10.0, 180.0 / max(1, args.steps + args.warmup))
    v, desc, cores = run_cpu(w, steps=max(1, args.steps), warmup=args.warmup,
                             step_budget_s=per_step)
    return {
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": workload_desc(w), "global_batch": w.tokens,
                   "parallelism": "cpu"},
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": cores, "kind": "port", "sample": desc},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="prefill",
                    choices=["prefill", "decode", "pr1", "fine", "sweep"])
    ap.add_argument("--tokens", type=int, default=None,
                    help="override the token count (smaller profiling cases)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    ap.add_argument("--graph", action="store_true",
                    help="one GPU: replay the layer forward as a captured CUDA graph")
    ap.add_argument("--exchange", default="peer", choices=["peer", "nccl"],
                    help="expert-parallel token exchange (N > 1)")
    ap.add_argument("--operands", default="auto", choices=["auto", "f16"],
                    help="expert GEMM operands: auto (8-bit for segments of at most 32 "
                         "rows) or f16 everywhere")
    args = ap.parse_args()
    if args.operands == "f16":
        from lightning_router.kernels import quantized_matmul as qm
        qm.INT8_OPERANDS = False
    if args.warmup < 3:
        args.warmup = 3
    ws, rank, local = init_dist()
    try:
        if args.impl == "reference":
            res = run_reference(args, ws, rank)
        elif args.workload == "sweep":
            res = run_sweep(args, ws, rank, local)
        else:
            res = run_gpu(args, ws, rank, local)
        if rank == 0 and res is not None:
            print(json.dumps(res), flush=True)
    finally:
        if ws > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
