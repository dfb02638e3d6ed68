"""Ablation of the B200 MoE-layer path: what each piece contributes.

The reference's ``benchmarks/ablation_study.py`` toggles Triton routing and
INT4 experts.  Here the routing kernels are always on (the layer has no other
routing path) and the configurations are, on the SAME weights (the fp16
experts hold ``dequantize_tensor`` of the packed INT4 weights, so every
configuration computes the same function up to accumulation order):

1. fp16 experts: one cuBLAS ``nn.Linear`` chain per expert on its kept rows
   (the reference's unquantized expert path, with its per-expert host reads);
2. INT4 experts: the grouped tcgen05 W4A16 GEMMs (gate/up with the SwiGLU
   epilogue, then down), no host synchronisation;
3. INT4 experts replayed as a CUDA graph of the whole layer.

Throughput is tokens / mean step time (CUDA events per step, after warm-up).

    python benchmarks/ablation_study.py [--workload prefill|decode|...] [--steps N]
"""

from __future__ import annotations

import argparse
import dataclasses
import json
import statistics
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))


def _fp16_twin(layer, w):
    """A layer with nn.Linear experts holding the dequantized INT4 weights."""
    from lightning_router.config import KernelConfig, ModelConfig, MoEConfig, QuantizationConfig
    from lightning_router.models.moe_layer import MoELayer
    from lightning_router.quantization.pack_weights import dequantize_tensor
    twin = MoELayer(ModelConfig(hidden_size=w.d_model, intermediate_size=w.d_ff),
                    MoEConfig(num_experts=w.experts, num_experts_per_token=w.top_k,
                              expert_capacity_factor=w.capacity_factor,
                              expert_activation=w.activation, gate_bias=w.zipf_s > 0),
                    QuantizationConfig(enabled=False), KernelConfig())
    twin = twin.to(layer.gate.gate_proj.weight.device)
    with torch.no_grad():
        twin.gate.load_state_dict(layer.gate.state_dict())
        twin.gate.gate_proj.half()
        for src, dst in zip(layer.experts.experts, twin.experts.experts):
            for m in (("gate", "up", "down") if w.activation == "swiglu" else ("up", "down")):
                W = dequantize_tensor(getattr(src, f"{m}_qweight"), getattr(src, f"{m}_scales"),
                                      getattr(src, f"{m}_zeros"), w.group_size,
                                      getattr(src, f"{m}_N"))          # (in, out) fp16
                lin = getattr(dst, f"{m}_proj")
                lin.weight.data = W.t().contiguous().half()
    return twin


def _time(fn, x, steps, warmup):
    for _ in range(warmup):
        fn(x)
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(steps)]
    for a, b in ev:
        a.record()
        fn(x)
        b.record()
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in ev]


def run(workload: str, steps: int, warmup: int) -> dict:
    from lightning_router.workloads import WORKLOADS, build_layer
    w = WORKLOADS[workload]
    dev = torch.device("cuda", 0)
    layer, t = build_layer(w, device=dev, gen_device=dev)
    x = t.x
    rows = []

    def record(name, fn, peak_fn=None):
        torch.cuda.reset_peak_memory_stats(dev)
        with torch.inference_mode():
            ms = _time(fn, x, steps, warmup)
        mean = statistics.mean(ms)
        rows.append({"config": name, "mean_ms": mean, "median_ms": statistics.median(ms),
                     "std_ms": statistics.stdev(ms) if len(ms) > 1 else 0.0,
                     "tokens_per_s": w.tokens / (mean / 1e3),
                     "peak_mem_mb": torch.cuda.max_memory_allocated(dev) / 2**20})

    twin = _fp16_twin(layer, w)
    with torch.inference_mode():
        ref16, _ = twin(x)
        out4, _ = layer(x)
    agree = float((ref16.float() - out4.float()).norm() / ref16.float().norm())
    record("fp16 experts (cuBLAS per expert)", lambda a: twin(a))
    del twin
    torch.cuda.empty_cache()
    record("INT4 experts (tcgen05 grouped GEMM)", lambda a: layer(a))

    static_x = x.clone()
    g = torch.cuda.CUDAGraph()
    with torch.inference_mode():
        layer(static_x)
        torch.cuda.synchronize()
        with torch.cuda.graph(g):
            layer(static_x)
    record("INT4 experts, CUDA graph", lambda a: g.replay())

    base = rows[0]["mean_ms"]
    for r in rows:
        r["speedup"] = base / r["mean_ms"]
    return {"workload": workload, "tokens": w.tokens, "d_model": w.d_model, "d_ff": w.d_ff,
            "experts": w.experts, "top_k": w.top_k, "steps": steps, "warmup": warmup,
            "fp16_vs_int4_rel_l2": agree, "rows": rows}


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--workload", default="prefill")
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--output", default=None, help="write the results as JSON here")
    args = ap.parse_args()
    res = run(args.workload, args.steps, args.warmup)
    print(f"{res['workload']}: {res['tokens']} tokens, d {res['d_model']} -> {res['d_ff']}, "
          f"{res['experts']} experts top-{res['top_k']} (fp16 vs INT4 outputs rel-L2 "
          f"{res['fp16_vs_int4_rel_l2']:.2e})")
    print(f"  {'configuration':<38} {'mean ms':>9} {'speed-up':>9} {'tokens/s':>14} {'peak MB':>9}")
    for r in res["rows"]:
        print(f"  {r['config']:<38} {r['mean_ms']:>9.3f} {r['speedup']:>8.2f}x "
              f"{r['tokens_per_s']:>14,.0f} {r['peak_mem_mb']:>9.0f}")
    if args.output:
        Path(args.output).write_text(json.dumps(res, indent=2))


if __name__ == "__main__":
    main()
