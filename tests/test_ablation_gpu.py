"""The B200 ablation (``benchmarks/ablation_study.py``, after the reference's
``benchmarks/ablation_study.py:123-128``) as a driver-run check: on the same
weights, the fp16 experts (cuBLAS ``nn.Linear`` per expert, the reference's
unquantized path) and the INT4 grouped tcgen05 GEMMs compute the same layer,
and at decode -- where the weight stream is the cost -- the INT4 path is
faster, with the CUDA-graph replay no slower than the eager step.  The table
is printed (``pytest -s``) and returned."""

from __future__ import annotations

import importlib.util
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

SCRIPT = (Path(__file__).resolve().parents[1] / "llm-serving-kernel-optimization_b200" /
          "benchmarks" / "ablation_study.py")


def _ablation():
    spec = importlib.util.spec_from_file_location("ablation_study", SCRIPT)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_decode_ablation():
    res = _ablation().run("decode", steps=30, warmup=5)
    rows = {r["config"].split(" (")[0].split(",")[0]: r for r in res["rows"]}
    for r in res["rows"]:
        print(f"{res['workload']}: {r['config']:<38} {r['mean_ms']:.3f} ms "
              f"{r['speedup']:.2f}x {r['tokens_per_s']:,.0f} tokens/s")
    assert res["fp16_vs_int4_rel_l2"] < 2e-3
    fp16 = rows["fp16 experts"]["mean_ms"]
    int4 = [r for r in res["rows"] if r["config"].startswith("INT4 experts (")][0]["mean_ms"]
    graph = [r for r in res["rows"] if "CUDA graph" in r["config"]][0]["mean_ms"]
    assert int4 * 1.3 < fp16, (int4, fp16)
    assert graph <= int4 * 1.05, (graph, int4)
