"""Time the reference's own CUDA kernel, compiled for sm_100a by
oracle/build_ref.py, on the same seeded workloads as bench.py -- a GPU
comparator only (BENCH INFRASTRUCTURE; never imported by the product).

Runs in its own process because the reference library registers the same
torch.ops.glm53_sparse_mla namespace as this repository's op. The reference
supports 8, 16 or 32 heads per launch (csrc/sparse_mla.cu:488-496), so a
64-head workload is timed as two 32-head launches per step, which is how the
reference would serve 64 heads on one GPU (two ranks' worth of work).

    python oracle/ref_gpu_bench.py --workload c2 --steps 200 --warmup 10
    python oracle/ref_gpu_bench.py --workload c2,c4,c5,c5f,c3
"""

from __future__ import annotations

import argparse
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
sys.path.insert(0, os.path.join(REPO, "vllm-sparse-mla-blackwell_b200"))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--workload", default="c2",
                    help="c2, c3, c4, c5 or c5f (C5 with fp8 KV); a comma-separated list runs "
                         "each in turn and prints one JSON line per workload")
    ap.add_argument("--heads", type=int, default=0)
    ap.add_argument("--kv", choices=["bf16", "fp8"], default="bf16")
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--sets", type=int, default=8)
    args = ap.parse_args()

    import torch
    so = os.path.join(HERE, "_ref", "ref_sparse_mla_sm100.so")
    if not os.path.exists(so):
        print(json.dumps({"impl": "reference-gpu", "unavailable": "oracle/_ref not built"}))
        return
    torch.ops.load_library(so)
    # workloads.py imports only numpy/torch; importing the package __init__
    # would load this repository's op, so load the module file directly
    import importlib.util
    spec = importlib.util.spec_from_file_location(
        "wl", os.path.join(REPO, "vllm-sparse-mla-blackwell_b200", "glm53_sparse_mla", "workloads.py"))
    W = importlib.util.module_from_spec(spec)
    sys.modules["wl"] = W          # dataclasses resolve their module through sys.modules
    spec.loader.exec_module(W)

    dev = torch.device("cuda", 0)
    for wl in args.workload.split(","):
        run_one(args, W, torch, dev, wl)


def run_one(args, W, torch, dev, wl):
    kv = "fp8" if wl == "c5f" else args.kv
    mk = {"c2": lambda s: W.config_c2(device=dev, seed=s),
          "c3": lambda s: W.config_c3(device=dev, seed=s),
          "c4": lambda s: W.config_c4(device=dev, seed=s),
          "c5": lambda s: W.config_c5(device=dev, seed=s, kv_dtype=kv),
          "c5f": lambda s: W.config_c5(device=dev, seed=s, kv_dtype="fp8")}[wl]
    n_sets = args.sets if wl in ("c2", "c4") else min(args.sets, 2)
    steps = args.steps if wl in ("c2", "c4") else max(2, args.steps // 10)
    sets = [mk(100 + s) for s in range(n_sets)]
    if args.heads:
        for w in sets:
            w.q = w.q[:, :args.heads].contiguous()
    H = sets[0].H
    parts = [(h0, min(32, H - h0)) for h0 in range(0, H, 32)]
    qs = [[w.q[:, h0:h0 + n].contiguous() for h0, n in parts] for w in sets]
    outs = [[torch.empty_like(x) for x in qq] for qq in qs]
    op = torch.ops.glm53_sparse_mla.sparse_fwd

    def step(k):
        j = k % len(sets)
        w = sets[j]
        for x, o in zip(qs[j], outs[j]):
            op(x, w.kv, w.indices, w.sm_scale, w.kv_scale, o)

    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        for k in range(args.warmup):
            step(k)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for k in range(steps):
            step(k)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        g.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    w = sets[0]
    print(json.dumps({"impl": "reference-gpu (csrc/sparse_mla.cu built for sm_100a)",
                      "workload": wl, "heads": H, "launches_per_step": len(parts),
                      "tokens": w.T, "ms_per_step": round(ms, 5),
                      "value": round(w.T / (ms / 1e3), 1), "unit": "query-tokens/s",
                      "gathered_GBps": round(w.n_valid() * 512 * w.kv.element_size() * len(parts)
                                             / (ms / 1e3) / 1e9, 1)}), flush=True)
    del g, sets, qs, outs
    torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
