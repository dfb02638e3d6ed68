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
roofline  the dominant kernel (grouped W4A16 gate/up GEMM): algorithmic FLOPs per launch /
          its CUDA-event duration inside the timed steps, against the measured sustained
          bf16 tensor peak.
cpu_baseline  the CPU oracle (numpy fp32 restatement of the reference path) on the host
          cores, rank 0 only, on a bounded token sample.

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

# DRAM bytes (read + write) per launch of the dominant kernel (the gate/up GEMM)
# from full-size ncu captures of the bench's own timed steps, keyed by workload
# (profiles/launches_prefill16k.md, profiles/launches_decode64.md); None until
# captured.
NCU_TRAFFIC = {
    "prefill": 809.0e6 + 907.3e6,   # rows in 268 MB + weights 487 MB, rows out 940 MB
    "decode": 489.8e6 + 2.6e6,      # weights 487 MB
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
def cpu_threads() -> int:
    try:
        from threadpoolctl import threadpool_info
        n = [i.get("num_threads", 0) for i in threadpool_info() if i.get("user_api") == "blas"]
        if n:
            return int(max(n))
    except Exception:
        pass
    return os.cpu_count() or 1


def cpu_oracle_setup(w, sample_tokens: int):
    """Dequantized fp32 expert weights on the host (untimed load) and a token sample."""
    import oracle as orc  # the CPU restatement, used here as the timed baseline
    from lightning_router.quantization.pack_weights import dequantize_tensor
    from lightning_router.workloads import make_layer
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    t = make_layer(w, device=dev, gen_device=dev, tokens=sample_tokens)
    experts = []
    for ex in t.experts:
        experts.append({n: dequantize_tensor(q, s, z, w.group_size, s.shape[1]).float().cpu().numpy()
                        for n, (q, s, z) in ex.items()})
    x = t.x.cpu().numpy()
    wg = t.gate_w.cpu().numpy()
    bias = None if t.bias is None else t.bias.cpu().numpy()
    del t
    if dev == "cuda":
        torch.cuda.empty_cache()
    return orc, x, wg, bias, experts


def cpu_oracle_step(orc, w, x, wg, bias, experts):
    logits = orc.gate_logits(x, wg, bias)
    out, aux, _ = orc.moe_layer(x, logits, w.top_k, w.capacity_factor, experts)
    return out


def run_cpu(w, steps: int, warmup: int, budget_s: float = 20.0):
    """Times the CPU oracle; returns (tokens/s, sample description, threads)."""
    sample = min(w.tokens, 512 if w.d_ff >= 8192 else 1024)
    orc, x, wg, bias, experts = cpu_oracle_setup(w, sample)
    for _ in range(max(0, warmup)):
        cpu_oracle_step(orc, w, x, wg, bias, experts)
    n, t0 = 0, time.perf_counter()
    while n < max(1, steps):
        cpu_oracle_step(orc, w, x, wg, bias, experts)
        n += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    desc = (f"{n} step(s) of {sample} of {w.tokens} tokens through the numpy fp32 oracle "
            f"(gate, top-k, capacity {w.capacity_factor}, dequantized INT4 experts, combine); "
            f"weights dequantized once outside the timed region")
    return sample * n / dt, desc, cpu_threads()


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
    # it so `ncu --profile-from-start off` lists exactly the timed launches.
    stage_owner.stage_events = []
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
    if graph is not None:
        stage_owner.stage_events = []
        n_stage = min(args.steps, 10)
        for _ in range(n_stage):
            eager_fwd(x)
        torch.cuda.synchronize()
        st = stage_times(stage_owner.stage_events, n_stage)
    else:
        st = stage_times(stage_owner.stage_events, args.steps)
    stage_owner.stage_events = None
    value = w.tokens * args.steps / (ms / 1e3)

    # dominant kernel roofline: grouped gate/up GEMM (2/3 of the FFN FLOPs for SwiGLU)
    plan_kept = model.last_kept_rows() if hasattr(model, "last_kept_rows") else None
    if plan_kept is None:
        _, plan = layer.route(x)
        plan_kept = int(plan.kept_counts.sum())
    gated = w.activation == "swiglu"
    gemm_in_flops = 2 * plan_kept * (2 if gated else 1) * w.d_model * w.d_ff
    gemm_ms = st.get("ffn_in")
    achieved = gemm_in_flops / (gemm_ms / 1e3) / 1e12 if gemm_ms else None
    peak = float(peaks.get("bf16_tflops_sustained", peaks.get("bf16_tflops")))
    roofline = {
        "kernel": "w4a16_grouped_gemm (gate/up, SwiGLU epilogue)",
        "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
        "frac": (achieved / peak) if achieved else None,
        "peak_kind": f"{peak_kind} sustained bf16",
        "traffic": NCU_TRAFFIC.get(args.workload),
        "flops_per_launch": gemm_in_flops,
        "launch_ms": gemm_ms,
        "stage_ms": {k: round(v, 4) for k, v in st.items()},
    }

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
    if ws > 1:
        barrier(ws)
        model.close()
    result = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": workload_desc(w), "global_batch": w.tokens, "seq_len": None,
                   "parallelism": parallel,
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
        v, desc, cores = run_cpu(w, steps=2, warmup=0)
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
    v, desc, cores = run_cpu(w, steps=max(1, args.steps), warmup=min(args.warmup, 1),
                             budget_s=60.0)
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
    args = ap.parse_args()
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
