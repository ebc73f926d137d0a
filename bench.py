#!/usr/bin/env python
"""Benchmark: sparse-MLA query-tokens/s at 64 heads, top-k 2048 (C2 decode batch).

One step = one launch of the sparse-MLA op over one decode batch: 32 query
tokens x 64 heads, top-k 2048 over a 131072-slot paged bf16 KV pool (block 64,
random block tables, context 8192). Inputs are synthetic and seeded
(glm53_sparse_mla.workloads.config_c2); the reference measures on no public
dataset.

Device number (`value`): K steps captured in one CUDA graph and replayed,
timed with CUDA events on the launching stream between a barrier and a device
synchronisation on both sides; max over ranks. Steps rotate over --sets
independent input sets (own KV pool, q, indices), whose pools together are
several times the 126 MB L2, so each step's gather is served from HBM.

End-to-end number (`e2e`): the same metric through the public Python API
(glm53_sparse_mla.sparse_fwd -> torch op -> C ABI) with host buffers: every
step copies q and indices from pinned host memory, runs the op and copies the
output back. The KV pool is resident device state (the paged cache). Each
step's three operations are ordered on its input set's stream and consecutive
steps overlap, as the steps of a serving loop do; the timed region covers every
step's copies. (The step is PCIe-bound: its 4.5 MB of host copies take about
80 us, against 27 us of kernel time.)

`roofline`: algorithmic bytes per launch (gathered KV rows per valid index,
q, out, indices) / average launch time, against the measured HBM copy
bandwidth in MEASURED_PEAKS.json; `traffic` is DRAM bytes per launch from the
committed ncu capture summary (profiles/), or null.

`cpu_baseline`: the CPU oracle (numpy fp32 restatement of the reference's
tests/reference.py) timed on this host's cores over a bounded sample of the
same workload, rank 0 only.

Multi-GPU (torchrun, one process per GPU): --shard tokens (default) gives
every rank its own decode batch with all 64 heads (data-parallel attention,
weak scaling, no collective on the data path); --shard heads splits the 64
heads of one batch across ranks (tensor-parallel heads, strong scaling), with
--allgather adding the NCCL all-gather of the output shards.

--impl reference times the reference's CPU implementation of the path (the
oracle port) on the host cores instead, on rank 0 only.

--op cache_write measures the latent KV-cache writer instead (the write that
feeds the attention): --tokens new tokens per step (default 8192, a
chunked-prefill step) into a 524288-slot paged cache, --kv fp8 (default bf16)
for the plain fp8 cache, same JSON line with its own metric and roofline.
--op indexer measures the indexer's fp8 paged MQA logits over --rows decode
rows of --ctx cached positions (64 heads, block 64, 8 rotating caches).
--op decode_step chains the four (cache write, indexer logits, top-2048,
paged attention) as one sparse decode step of --rows sequences at --ctx.
--op topk measures the indexer's per-row top-2048 over --rows decode rows of
--ctx logits (default 32 x 8192, C2's batch and context), with vLLM's
compiled op of the same contract timed alongside when it loads.
"""

from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "vllm-sparse-mla-blackwell_b200"))
sys.path.insert(0, REPO)

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "sparse-MLA query-tokens/s @64 heads, topk=2048 (C2 decode, bf16 KV)"
UNIT = "query-tokens/s"


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--op", choices=["attention", "paged", "cache_write", "indexer", "topk",
                                     "decode_step"],
                    default="attention",
                    help="attention (the headline), the latent KV-cache writer, the indexer's "
                         "fp8 paged logits, its per-row top-k, or the four chained as one "
                         "sparse decode step")
    ap.add_argument("--tokens", type=int, default=8192,
                    help="cache_write: new tokens per step (a chunked-prefill step)")
    ap.add_argument("--rows", type=int, default=32, help="topk: decode rows (query tokens)")
    ap.add_argument("--ctx", type=int, default=8192, help="topk: context length per row")
    ap.add_argument("--workload", choices=["c2", "c3", "c4", "c5"], default="c2")
    ap.add_argument("--heads", type=int, default=0, help="heads per launch (0 = workload's)")
    ap.add_argument("--kv", choices=["bf16", "fp8"], default="bf16", help="C5 KV dtype")
    ap.add_argument("--sets", type=int, default=8, help="rotating input sets")
    ap.add_argument("--splits", type=int, default=0, help="force a split count (0 = auto)")
    ap.add_argument("--shard", choices=["tokens", "heads"], default="tokens")
    ap.add_argument("--allgather", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-clocks", action="store_true")
    ap.add_argument("--no-spread", action="store_true", help="skip the median / p10 / p90 replays")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the extra keys of the default line (the other configs, the "
                         "reference's GPU kernel, the W_UV projection)")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# process group
# ---------------------------------------------------------------------------
class Dist:
    def __init__(self, want: int):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        if want != self.world and not (want == 1 and self.world == 1):
            if self.world == 1 and want > 1:
                raise SystemExit(f"--gpus {want} needs torchrun with {want} processes")
        self.pg = None

    def init(self, backend: str):
        if self.world > 1:
            # NCCL's version banner (NCCL_DEBUG=VERSION) would precede the one
            # JSON line rank 0 prints; warnings and above still show
            if os.environ.get("NCCL_DEBUG", "VERSION").upper() == "VERSION":
                os.environ["NCCL_DEBUG"] = "WARN"
            import datetime
            torch.distributed.init_process_group(
                backend, timeout=datetime.timedelta(seconds=180),
                device_id=torch.device("cuda", self.local) if backend == "nccl" else None)
            self.pg = True

    def barrier(self):
        if self.pg:
            torch.distributed.barrier()

    def max(self, x: float, device) -> float:
        if not self.pg:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg:
            torch.distributed.destroy_process_group()


# ---------------------------------------------------------------------------
# workloads
# ---------------------------------------------------------------------------
def make_workload(args, W, seed: int, device, heads: int, head_offset: int = 0):
    if args.workload == "c2":
        w = W.config_c2(device=device, seed=seed, heads=64)
    elif args.workload == "c3":
        w = W.config_c3(device=device, seed=seed)
    elif args.workload == "c4":
        w = W.config_c4(device=device, seed=seed)
    else:
        w = W.config_c5(device=device, seed=seed, heads=64, kv_dtype=args.kv)
    if heads and heads != w.H:
        w.q = w.q[:, head_offset:head_offset + heads].contiguous()
    return w


def attention_config(args, w, heads_total: int, world: int) -> dict:
    """The `config` object of the attention arms; the reference arm prints the
    same one, computed from the arguments and the workload's shapes only."""
    cfg = workload_desc(args, w, heads_total)
    n_sets = max(1, args.sets)
    pool_gb = n_sets * w.kv.numel() * w.kv.element_size() / 1e9
    cfg.update({"parallelism": (f"dp{world}" if args.shard == "tokens" else f"tp{world}-heads"),
                "l2": f"{n_sets} rotating input sets, {pool_gb:.2f} GB of KV pools "
                      "(>> 126 MB L2); consecutive steps share no memory",
                "timing": "K steps in one CUDA graph, CUDA events, max over ranks",
                "splits": args.splits or "auto",
                "allgather": bool(args.allgather and world > 1 and args.shard == "heads")})
    return cfg


def workload_desc(args, w, heads_total: int) -> dict:
    d = {"c2": "C2 decode bf16: 32 seqs x 1 token, 64 heads, topk 2048, pool 131072 slots",
         "c3": "C3 mixed: 4096-token prefill + 31 decode tokens, 32 heads, topk 2048",
         "c4": "C4 fp8 decode: 64 seqs x 1 token, 16 heads, topk 2048, ctx 65536",
         "c5": f"C5 MTP: 128 seqs x 4 tokens, topk 2048, ctx 32768, {args.kv} KV"}[args.workload]
    return {"workload": d, "tokens_per_step": w.T, "heads_per_gpu": w.H,
            "heads_total": heads_total, "topk": w.topk, "kv_rows": int(w.kv.shape[0]),
            "kv_dtype": "fp8_e4m3" if w.kv.dtype == torch.float8_e4m3fn else "bf16"}


# ---------------------------------------------------------------------------
# measurement helpers
# ---------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,"
              "clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int, enabled: bool = True):
        self.proc = None
        self.lines = []
        self.enabled = enabled
        self.idx = device_index

    def __enter__(self):
        if not self.enabled:
            return self
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.idx), "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, ValueError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.thread.join(timeout=2)

    def summary(self):
        rows = []
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 10:
                continue
            try:
                rows.append({"sm": float(parts[1]), "max": float(parts[2]),
                             "util": float(parts[4]) if parts[4] not in ("[N/A]", "") else 0.0,
                             "hw": parts[6], "hwt": parts[7], "swt": parts[8], "pcap": parts[9]})
            except ValueError:
                continue
        if not rows:
            return None
        busy = [r for r in rows if r["util"] > 0] or rows
        reasons = []
        for key, name in (("hw", "hw_slowdown"), ("hwt", "hw_thermal_slowdown"),
                          ("swt", "sw_thermal_slowdown"), ("pcap", "sw_power_cap")):
            if any(r[key].lower() == "active" for r in busy):
                reasons.append(name)
        return {"sm_mhz": statistics.median(r["sm"] for r in busy),
                "sm_max_mhz": max(r["max"] for r in rows), "reasons": reasons,
                "samples": len(rows), "samples_busy": len(busy)}


def measured_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def _profile_text(workload: str):
    path = os.path.join(REPO, "profiles", f"sparse_mla_fwd_{workload}.md")
    return open(path).read() if os.path.exists(path) else None


def profiled_traffic(workload: str):
    """DRAM bytes per launch recorded in the committed ncu summary, if it was
    captured from the current kernel source (its recorded source digest
    matches); None otherwise, so a stale capture is never reported."""
    text = _profile_text(workload)
    if text is None:
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9]+)", text)
    d = re.search(r"kernel_source_sha256_16:\s*([0-9a-f]{16})", text)
    if not m or not d or d.group(1) != kernel_source_digest():
        return None
    return int(m.group(1))


def traffic_source(workload: str) -> str:
    text = _profile_text(workload)
    if text is None:
        return "no ncu summary for this workload"
    d = re.search(r"kernel_source_sha256_16:\s*([0-9a-f]{16})", text)
    cur = kernel_source_digest()
    if d and d.group(1) == cur:
        return f"profiles/sparse_mla_fwd_{workload}.md, ncu capture of kernel source {cur}"
    return (f"profiles/sparse_mla_fwd_{workload}.md predates the current kernel source "
            f"{cur}: traffic not reported")


def kernel_source_digest() -> str:
    """First 16 hex digits of the sha256 of the attention kernel's source, as
    the ncu summaries under profiles/ record it for the capture they hold."""
    import hashlib
    path = os.path.join(REPO, "vllm-sparse-mla-blackwell_b200", "csrc", "sparse_mla_sm100.cu")
    with open(path, "rb") as f:
        return hashlib.sha256(f.read()).hexdigest()[:16]


def graph_ms(step, n_steps: int, stream, reps: int = 3) -> float:
    """Device ms per step of `step(k)`, k < n_steps, captured in one CUDA graph
    (after an eager warm-up), best of `reps` timed replays. For the extra keys
    of the bench line; the headline number uses the contract's timing."""
    with torch.cuda.stream(stream):
        for k in range(min(n_steps, 3)):
            step(k)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for k in range(n_steps):
            step(k)
    torch.cuda.synchronize()
    g.replay()
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            a.record(stream)
            g.replay()
            b.record(stream)
        b.synchronize()
        best = min(best, a.elapsed_time(b) / n_steps)
    del g
    torch.cuda.synchronize()
    return best


def gather_roof_ms(G, sets, stream, n_steps: int):
    """The bare gather of the same rows (glm53_gather_roof, one CTA per SM over
    the flattened index list) on the same rotating sets: ms per launch. None
    for an fp8 pool (the probe moves 1 KiB bf16 rows)."""
    import ctypes
    if sets[0].kv.dtype != torch.bfloat16:
        return None
    lib = ctypes.CDLL(G.library_path())
    lib.glm53_gather_roof.restype = ctypes.c_int
    lib.glm53_gather_roof.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                      ctypes.c_int64, ctypes.c_int64, ctypes.c_int,
                                      ctypes.c_void_p, ctypes.c_void_p]
    sms = torch.cuda.get_device_properties(stream.device).multi_processor_count
    sink = torch.empty(sms, dtype=torch.int32, device=stream.device)

    def step(k):
        w = sets[k % len(sets)]
        rc = lib.glm53_gather_roof(w.kv.data_ptr(), w.indices.data_ptr(), w.T, w.topk,
                                   w.kv.shape[0], sms, sink.data_ptr(),
                                   torch.cuda.current_stream().cuda_stream)
        assert rc == 0, rc
    return graph_ms(step, n_steps, stream)


def extra_configs(args, G, W, device, stream, hbm_peak: float) -> dict:
    """The other benchmark configurations, timed the same way as the headline
    (a CUDA graph of back-to-back launches over rotating input sets, CUDA
    events): C3 mixed prefill + decode, C4 decode with fp8 KV (and the same
    shape with bf16 KV, for the fp8-vs-bf16 comparison), C5 MTP with bf16
    and fp8 KV. Each reports ms per step, query-tokens/s and the fraction of the
    HBM roofline (algorithmic bytes / time / measured copy bandwidth)."""
    out = {}
    for key, mk, n_sets, steps in (
            ("c3", lambda s: W.config_c3(device=device, seed=s), 2, 6),
            ("c4_fp8", lambda s: W.config_c4(device=device, seed=s), 8, 50),
            ("c4_bf16", lambda s: W.config_c4(device=device, seed=s, kv_dtype="bf16"), 8, 50),
            ("c5_bf16", lambda s: W.config_c5(device=device, seed=s, heads=64), 2, 10),
            ("c5_fp8", lambda s: W.config_c5(device=device, seed=s, heads=64, kv_dtype="fp8"), 2, 10)):
        sets = [mk(200 + s) for s in range(n_sets)]
        outs = [torch.empty_like(w.q) for w in sets]

        def step(k):
            w = sets[k % n_sets]
            torch.ops.glm53_sparse_mla.sparse_fwd(w.q, w.kv, w.indices, w.sm_scale, w.kv_scale,
                                                  outs[k % n_sets])
        ms = graph_ms(step, steps, stream)
        w = sets[0]
        ab = w.algorithmic_bytes()
        out[key] = {"ms_per_step": round(ms, 5), "value": round(w.T / (ms / 1e3), 1),
                    "unit": UNIT, "tokens": w.T, "heads": w.H,
                    "kv_dtype": "fp8_e4m3" if w.kv.dtype == torch.float8_e4m3fn else "bf16",
                    "frac": round(ab / (ms / 1e3) / 1e9 / hbm_peak, 4),
                    "algorithmic_bytes_per_launch": ab, "sets": n_sets}
        del sets, outs
        torch.cuda.empty_cache()
    return out


def reference_gpu_leg(timeout_s: float = 240.0):
    """Comparator: the reference's own kernel (csrc/sparse_mla.cu, built for
    sm_100a into oracle/_ref/ by oracle/build_ref.py) timed on the same
    workloads in a separate process (it registers the same op namespace). A
    baseline, never this repository's number; None when it was not built."""
    so = os.path.join(REPO, "oracle", "_ref", "ref_sparse_mla_sm100.so")
    if not os.path.exists(so):
        return {"unavailable": "oracle/_ref not built"}
    cmd = [sys.executable, os.path.join(REPO, "oracle", "ref_gpu_bench.py"),
           "--workload", "c2,c4,c5,c5f,c3", "--steps", "50", "--warmup", "3"]
    try:
        res = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout_s, cwd=REPO)
    except subprocess.TimeoutExpired:
        return {"unavailable": f"did not finish in {timeout_s:.0f} s"}
    out = {}
    for ln in res.stdout.splitlines():
        try:
            d = json.loads(ln)
        except ValueError:
            continue
        if "workload" in d:
            out[d["workload"]] = {"ms_per_step": d["ms_per_step"], "value": d["value"],
                                  "launches_per_step": d["launches_per_step"]}
    if not out:
        return {"unavailable": (res.stderr or res.stdout)[-300:]}
    out["kernel"] = "reference csrc/sparse_mla.cu (mma.sync), sm_100a build, 32 heads per launch"
    return out


def w_uv_leg(stream, device, attention_ms: dict) -> dict:
    """The W_UV up-projection vLLM runs after this op (MLAAttention._v_up_proj:
    out [T, H, 512] -> transpose -> batched GEMM with W_UV [H, 512, 128] ->
    [T, H * 128]), timed at the C2 and C5 shapes next to the attention, with
    random weights: the measured size of the work a fused epilogue would take
    over."""
    res = {}
    for key, T in (("c2", 32), ("c5", 512)):
        H = 64
        x = torch.randn(T, H, 512, device=device).to(torch.bfloat16)
        wuv = torch.randn(H, 512, 128, device=device).to(torch.bfloat16) * 0.05
        y = torch.empty(T, H * 128, device=device, dtype=torch.bfloat16)

        def step(k):
            t = torch.bmm(x.transpose(0, 1), wuv)          # [H, T, 128]
            y.view(T, H, 128).copy_(t.transpose(0, 1))
        ms = graph_ms(step, 20, stream)
        res[key] = {"w_uv_ms": round(ms, 5), "attention_ms": attention_ms.get(key),
                    "w_uv_share": (round(ms / attention_ms[key], 4) if attention_ms.get(key) else None),
                    "weights_bytes": H * 512 * 128 * 2}
    return res


def eager_ms(step, n_steps: int, stream) -> float:
    """Device ms per step of `step(k)` launched eagerly (3 warm-up steps, then
    n_steps between CUDA events on `stream`)."""
    with torch.cuda.stream(stream):
        for k in range(3):
            step(k)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        a.record(stream)
        for k in range(n_steps):
            step(k)
        b.record(stream)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / n_steps


def head_shard_leg(S, W, device, stream, dist, steps: int = 10) -> dict:
    """The north star's head-sharding sweep, on the MTP shape (C5: 128
    sequences x 4 tokens, top-k 2048, bf16 KV): rank r of N serves heads
    [r * 64 / N, (r + 1) * 64 / N) of the same batch, index lists and pool
    replicated (vLLM TP). Times per step, max over ranks, from a CUDA graph of
    `steps` steps (eager launches if the symmetric-memory barrier cannot be
    captured; `timing` says which):
      kernel_ms    the op alone (this rank's heads, local output)
      nccl_ms      the op, then NCCL all_gather_into_tensor and the head
                   reorder copy into [T, 64, 512]
      fused_ms     the op writing its heads straight into every rank's
                   [T, 64, 512] buffer (symmetric memory, plain peer stores),
                   then a symmetric-memory barrier: no all-gather, no copy
      copy_ms      one launch per wave into the own buffer, each wave's head
                   slice pushed to the peers by the copy engines while the
                   next wave computes, then the barrier
    value = tokens / the faster of fused_ms and copy_ms (`gather_used`)
    (strong scaling: the same 512 tokens for every
    N). Every rank gathers the same KV bytes whatever its head count (one
    latent head), so per-GPU time stays nearly flat as N grows."""
    world, rank = dist.world, dist.rank
    h0, h = S.head_range(rank, world, 64)
    sets = [W.config_c5(device=device, seed=300 + s, heads=64) for s in range(2)]
    qs = [w.q[:, h0:h0 + h].contiguous() for w in sets]
    outs = [torch.empty_like(q) for q in qs]
    op = torch.ops.glm53_sparse_mla.sparse_fwd

    def kstep(k):
        w = sets[k % 2]
        op(qs[k % 2], w.kv, w.indices, w.sm_scale, w.kv_scale, outs[k % 2])

    res = {"workload": "C5 MTP: 128 seqs x 4 tokens, topk 2048, ctx 32768, bf16 KV",
           "tokens": sets[0].T, "heads_total": 64, "heads_per_gpu": h, "n_gpus": world,
           "kv_bytes_per_gpu": sets[0].n_valid() * 1024}
    res["kernel_ms"] = round(dist.max(graph_ms(kstep, steps, stream), device), 5)
    res["timing"] = {"kernel": "graph"}
    if world == 1:
        res["fused_ms"] = res["kernel_ms"]
    else:
        staging = torch.empty(world, sets[0].T, h, 512, dtype=torch.bfloat16, device=device)

        def nstep(k):
            kstep(k)
            S.gather_heads(outs[k % 2], world, staging=staging)
        res["nccl_ms"] = round(dist.max(graph_ms(nstep, steps, stream), device), 5)
        res["timing"]["nccl"] = "graph"
        gather = S.HeadShardGather(sets[0].T, 64, device=device)

        def fstep(k):
            w = sets[k % 2]
            gather(qs[k % 2], w.kv, w.indices, w.sm_scale, w.kv_scale)

        # diagnostic: the fused kernel without the closing barrier (not a
        # usable result on its own: nothing orders the peers' stores yet)
        def fstep_nb(k):
            w = sets[k % 2]
            gather(qs[k % 2], w.kv, w.indices, w.sm_scale, w.kv_scale, barrier=False)
        res["fused_no_barrier_ms"] = round(dist.max(graph_ms(fstep_nb, steps, stream), device), 5)
        dist.barrier()
        try:
            t_fused, how = graph_ms(fstep, steps, stream), "graph"
        except RuntimeError:
            torch.cuda.synchronize()
            dist.barrier()
            t_fused, how = eager_ms(fstep, steps, stream), "eager"
        res["fused_ms"] = round(dist.max(t_fused, device), 5)
        res["timing"]["fused"] = how
        dist.barrier()
        del gather
        # the same exchange by the copy engines: one launch per wave into the
        # own buffer, each wave's head slice pushed to the peers meanwhile
        cgather = S.HeadShardGather(sets[0].T, 64, device=device, mode="copy")

        def cstep(k):
            w = sets[k % 2]
            cgather(qs[k % 2], w.kv, w.indices, w.sm_scale, w.kv_scale)
        try:
            t_copy, how = graph_ms(cstep, steps, stream), "graph"
        except RuntimeError:
            torch.cuda.synchronize()
            dist.barrier()
            t_copy, how = eager_ms(cstep, steps, stream), "eager"
        res["copy_ms"] = round(dist.max(t_copy, device), 5)
        res["timing"]["copy"] = how
        dist.barrier()
        del cgather
    best = min(res["fused_ms"], res.get("copy_ms", res["fused_ms"]))
    res["gather_used"] = "copy" if res.get("copy_ms", 1e9) < res["fused_ms"] else "fused"
    res["value"] = round(sets[0].T / (best / 1e3), 1)
    res["unit"] = UNIT
    del sets, qs, outs
    torch.cuda.empty_cache()
    return res


def set_splits(n: int):
    if n:
        os.environ["GLM53_SPLITS"] = str(n)


# ---------------------------------------------------------------------------
# arms
# ---------------------------------------------------------------------------
def run_ours(args, dist: Dist):
    torch.cuda.set_device(dist.local)
    device = torch.device("cuda", dist.local)
    dist.init("nccl")
    set_splits(args.splits)
    import glm53_sparse_mla as G
    from glm53_sparse_mla import sharding as S
    from glm53_sparse_mla import workloads as W

    heads_total = 64 if args.workload in ("c2", "c5") else (32 if args.workload == "c3" else 16)
    if args.heads:
        heads_total = args.heads
    if args.shard == "heads" and dist.world > 1:
        head_off, heads = S.head_range(dist.rank, dist.world, heads_total)
        seed_of = lambda s: 100 + s                       # same batch on every rank
    else:
        heads = heads_total
        head_off = 0
        seed_of = lambda s: 100 + s + 1000 * dist.rank    # own batch per rank
    sets = [make_workload(args, W, seed_of(s), device, heads, head_off)
            for s in range(max(1, args.sets))]
    w0 = sets[0]
    outs = [torch.empty_like(w.q) for w in sets]
    gathered = None
    if args.allgather and dist.world > 1 and args.shard == "heads":
        gathered = torch.empty(dist.world, w0.T, heads, 512, dtype=torch.bfloat16, device=device)

    def step(k):
        w = sets[k % len(sets)]
        torch.ops.glm53_sparse_mla.sparse_fwd(w.q, w.kv, w.indices, w.sm_scale, w.kv_scale,
                                              outs[k % len(sets)])
        if gathered is not None:
            S.gather_heads(outs[k % len(sets)], dist.world, staging=gathered)

    stream = torch.cuda.Stream(device)
    with torch.cuda.stream(stream):
        for k in range(max(args.warmup, 3)):
            step(k)
    torch.cuda.synchronize()

    # capture the K timed steps in one graph (launch-bound otherwise); the
    # NCCL all-gather of the head-sharded mode is captured with them
    graph = torch.cuda.CUDAGraph()
    use_graph = True
    if use_graph:
        with torch.cuda.graph(graph, stream=stream):
            for k in range(args.steps):
                step(k)
        torch.cuda.synchronize()
        graph.replay()          # untimed replay: warm the graph launch path
        torch.cuda.synchronize()

    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dist.local, enabled=not args.no_clocks) as clk:
        # soak so the sampler sees the clocks under this load
        t_end = time.time() + (0.0 if args.no_clocks else 0.5)
        while time.time() < t_end:
            (graph.replay() if use_graph else [step(k) for k in range(len(sets))])
            torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            e0.record(stream)
            if use_graph:
                graph.replay()
            else:
                for k in range(args.steps):
                    step(k)
            e1.record(stream)
        torch.cuda.synchronize()
        dist.barrier()
    ms_local = e0.elapsed_time(e1)
    ms = dist.max(ms_local, device)
    ms_step = ms / args.steps
    units = w0.T * (dist.world if args.shard == "tokens" else 1)
    value = units / (ms_step / 1e3)

    # roofline for the attention kernel (per launch on this rank)
    alg_bytes = w0.algorithmic_bytes()
    hbm_peak, tf_peak, peak_kind = measured_peaks()
    achieved = alg_bytes / (ms_local / args.steps / 1e3) / 1e9
    roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
            "frac": round(achieved / hbm_peak, 4), "peak_source": peak_kind,
            "traffic": profiled_traffic(args.workload),
            "traffic_source": traffic_source(args.workload),
            "algorithmic_bytes_per_launch": alg_bytes,
            "tensor_tflops": round(w0.flops() / (ms_local / args.steps / 1e3) / 1e12, 1),
            "tensor_frac": round(w0.flops() / (ms_local / args.steps / 1e3) / 1e12 / tf_peak, 4)}
    del graph
    torch.cuda.synchronize()

    # spread (outside the contract's one timed run): 20 replays of a graph of
    # up to 50 steps, each timed, give median and p10 / p90 per step
    spread = None
    if not args.no_spread:
        n_sp = min(50, args.steps)
        g_sp = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_sp, stream=stream):
            for k in range(n_sp):
                step(k)
        torch.cuda.synchronize()
        per = []
        for _ in range(20):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(stream):
                a.record(stream)
                g_sp.replay()
                b.record(stream)
            b.synchronize()
            per.append(a.elapsed_time(b) / n_sp)
        del g_sp
        torch.cuda.synchronize()
        q = np.percentile(per, [10, 50, 90])
        spread = {"median_ms": round(float(q[1]), 5), "p10_ms": round(float(q[0]), 5),
                  "p90_ms": round(float(q[2]), 5), "replays": 20, "steps_per_replay": n_sp,
                  "rank": dist.rank}

    # the bare gather of the same rows on the same sets (the gather roof)
    g_ms = gather_roof_ms(G, sets, stream, min(args.steps, 50) if args.steps > 0 else 1)
    if g_ms is not None:
        kv_bytes = w0.n_valid() * 512 * w0.kv.element_size()
        roof["gather_roof_gbs"] = round(kv_bytes / (g_ms / 1e3) / 1e9, 1)
        roof["gather_roof_ms"] = round(g_ms, 5)
        roof["gather_share"] = round(g_ms / (ms_local / args.steps), 4)

    # end to end through the public API with host buffers
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, G, sets, device, dist)

    cpu = None
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(w0, args.cpu_seconds)

    # extra keys, after every timed loop of the contract: the other configs,
    # the W_UV projection vLLM runs next, the reference's own GPU kernel
    extras = {}
    if not args.no_extras and dist.world == 1 and args.workload == "c2" and not args.heads:
        extras["configs"] = extra_configs(args, G, W, device, stream, hbm_peak)
        extras["w_uv"] = w_uv_leg(stream, device, {
            "c2": ms_local / args.steps,
            "c5": extras["configs"]["c5_bf16"]["ms_per_step"]})
        extras["reference_gpu"] = reference_gpu_leg()
    if not args.no_extras and args.workload == "c2" and not args.heads and args.shard == "tokens":
        extras["head_shard"] = head_shard_leg(S, W, device, stream, dist)

    if dist.rank == 0:
        cfg = attention_config(args, w0, heads_total, dist.world)
        line = {"metric": METRIC if args.workload == "c2" else f"sparse-MLA {UNIT} ({args.workload})",
                "value": round(value, 1), "unit": UNIT, "n_gpus": dist.world, "steps": args.steps,
                "warmup": max(args.warmup, 3), "ms_per_step": round(ms_step, 5),
                "higher_is_better": True,
                "scaling": "weak" if args.shard == "tokens" else "strong",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded, random init)",
                "config": cfg, "roofline": roof, "cpu_baseline": cpu, "e2e": e2e,
                "gpu_launches": args.steps + (args.steps if e2e else 0),
                "clocks": clk.summary(), "spread": spread}
        line.update(extras)
        print(json.dumps(line), flush=True)
    dist.close()


# ---------------------------------------------------------------------------
# the latent KV-cache writer (--op cache_write)
# ---------------------------------------------------------------------------
CACHE_POOL_SLOTS = 524288        # C4's pool: 8192 blocks of 64
CACHE_BLOCK = 64
CW_UNIT = "cache-tokens/s"


def cache_write_sets(args, device, n_sets: int, seed0: int = 300):
    """n_sets independent steps: kv_c [tokens, 512] bf16 and distinct slots."""
    g = torch.Generator(device="cpu")
    sets = []
    for s in range(n_sets):
        g.manual_seed(seed0 + s)
        kv_c = torch.randn((args.tokens, 512), generator=g).to(torch.bfloat16)
        slots = torch.randperm(CACHE_POOL_SLOTS, generator=g)[:args.tokens].to(torch.int64)
        sets.append((kv_c.to(device), slots.to(device)))
    return sets


def cache_write_bytes(tokens: int, fp8: bool) -> int:
    """Algorithmic bytes per launch: the bf16 row read, the cache entry
    written, the slot read."""
    return tokens * (1024 + (512 if fp8 else 1024) + 8)


def cache_write_desc(args, fp8: bool) -> dict:
    return {"workload": f"latent KV-cache write: {args.tokens} new tokens per step into a "
                        f"{CACHE_POOL_SLOTS}-slot paged {'fp8_e4m3' if fp8 else 'bf16'} cache "
                        f"(block {CACHE_BLOCK}), random distinct slots",
            "tokens_per_step": args.tokens, "kv_dtype": "fp8_e4m3" if fp8 else "bf16"}


def time_graph(step, args, dist: Dist, device, stream):
    """Warm-up, then K steps captured in one CUDA graph, timed with CUDA
    events on `stream` between barriers, clocks sampled during the run.
    Returns (ms per step on this rank, ms per step max over ranks, clocks)."""
    with torch.cuda.stream(stream):
        for k in range(max(args.warmup, 3)):
            step(k)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for k in range(args.steps):
            step(k)
    torch.cuda.synchronize()
    graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dist.local, enabled=not args.no_clocks) as clk:
        t_end = time.time() + (0.0 if args.no_clocks else 0.5)
        while time.time() < t_end:
            graph.replay()
            torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            e0.record(stream)
            graph.replay()
            e1.record(stream)
        torch.cuda.synchronize()
        dist.barrier()
    ms_local = e0.elapsed_time(e1) / args.steps
    del graph
    torch.cuda.synchronize()
    return ms_local, dist.max(ms_local * args.steps, device) / args.steps, clk.summary()


def run_cache_write(args, dist: Dist):
    torch.cuda.set_device(dist.local)
    device = torch.device("cuda", dist.local)
    dist.init("nccl")
    import glm53_sparse_mla as G
    fp8 = args.kv == "fp8"
    dtype = "fp8" if fp8 else "auto"
    cache = torch.zeros((CACHE_POOL_SLOTS // CACHE_BLOCK, CACHE_BLOCK, 512),
                        dtype=torch.uint8 if fp8 else torch.bfloat16, device=device)
    scale = torch.tensor([0.05 if fp8 else 1.0], dtype=torch.float32, device=device)
    sets = cache_write_sets(args, device, max(1, args.sets), 300 + 1000 * dist.rank)
    empty_pe = sets[0][0][:, :0]

    def step(k):
        kv_c, slots = sets[k % len(sets)]
        G.concat_and_cache_mla(kv_c, empty_pe, cache, slots, dtype, scale)

    stream = torch.cuda.Stream(device)
    ms_rank, ms_step, clocks = time_graph(step, args, dist, device, stream)
    value = args.tokens * dist.world / (ms_step / 1e3)
    alg = cache_write_bytes(args.tokens, fp8)
    hbm_peak, _, peak_kind = measured_peaks()
    achieved = alg / (ms_rank / 1e3) / 1e9
    m = None
    prof = os.path.join(REPO, "profiles", f"kv_cache_writer_{args.kv}.md")
    if os.path.exists(prof):
        m = re.search(r"traffic_bytes_per_launch:\s*([0-9]+)", open(prof).read())
    roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
            "frac": round(achieved / hbm_peak, 4), "peak_source": peak_kind,
            "traffic": int(m.group(1)) if m else None, "algorithmic_bytes_per_launch": alg}
    e2e = None
    if not args.no_e2e:
        # host buffers: each step copies kv_c and slots in, writes, and reads
        # the written entries' first block back
        hk = [kv.cpu().pin_memory() for kv, _ in sets]
        hs = [sl.cpu().pin_memory() for _, sl in sets]
        dk = [torch.empty_like(kv) for kv, _ in sets]
        ds = [torch.empty_like(sl) for _, sl in sets]
        back = torch.empty(cache[0].shape, dtype=cache.dtype).pin_memory()

        def e2e_step(k):
            j = k % len(sets)
            dk[j].copy_(hk[j], non_blocking=True)
            ds[j].copy_(hs[j], non_blocking=True)
            G.concat_and_cache_mla(dk[j], empty_pe, cache, ds[j], dtype, scale)
            back.copy_(cache[0], non_blocking=True)

        for k in range(max(args.warmup, 3)):
            e2e_step(k)
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record()
        for k in range(args.steps):
            e2e_step(k)
        f1.record()
        torch.cuda.synchronize()
        ms_e = dist.max(f0.elapsed_time(f1), device) / args.steps
        e2e = {"value": round(args.tokens * dist.world / (ms_e / 1e3), 1), "unit": CW_UNIT,
               "h2d_bytes_per_step": args.tokens * (1024 + 8),
               "d2h_bytes_per_step": int(back.numel() * back.element_size()),
               "ms_per_step": round(ms_e, 5),
               "path": "glm53_sparse_mla.concat_and_cache_mla (torch op -> C ABI), pinned host "
                       "buffers; one cache block read back"}
    cpu = None
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        cpu = cache_write_cpu(sets[0], fp8, args.cpu_seconds)
    if dist.rank == 0:
        cfg = cache_write_desc(args, fp8)
        cfg.update({"parallelism": f"dp{dist.world}",
                    "l2": f"{len(sets)} rotating input sets; writes land in random slots of a "
                          f"{cache.numel() * cache.element_size() / 1e6:.0f} MB cache",
                    "timing": "K steps in one CUDA graph, CUDA events, max over ranks"})
        line = {"metric": f"latent KV-cache writes ({args.kv}), {CW_UNIT}", "value": round(value, 1),
                "unit": CW_UNIT, "n_gpus": dist.world, "steps": args.steps,
                "warmup": max(args.warmup, 3), "ms_per_step": round(ms_step, 5),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "bf16->fp8_e4m3" if fp8 else "bf16",
                "data": "synthetic (seeded)", "config": cfg, "roofline": roof,
                "cpu_baseline": cpu, "e2e": e2e,
                "gpu_launches": args.steps + (args.steps if e2e else 0),
                "clocks": clocks}
        print(json.dumps(line), flush=True)
    dist.close()


def cache_write_cpu(one_set, fp8: bool, seconds: float):
    """The oracle's cache write timed on this host over a sample of the step."""
    from oracle import cache_writer_oracle as CW
    kv_c, slots = one_set
    bits = kv_c.cpu().view(torch.uint16).numpy()
    sl = slots.cpu().numpy()
    n = min(len(sl), 1024)
    cache = np.zeros((CACHE_POOL_SLOTS // CACHE_BLOCK, CACHE_BLOCK, 512),
                     np.uint8 if fp8 else np.uint16)
    done, t0 = 0, time.perf_counter()
    while True:
        CW.concat_and_cache_mla(bits[:n], cache, sl[:n], "fp8" if fp8 else "auto", 0.05,
                                inplace=True)
        done += n
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    return {"value": round(done / dt, 2), "unit": CW_UNIT, "cores": 1, "kind": "port",
            "sample": f"{done} tokens in batches of {n}, numpy oracle (restates vLLM's "
                      f"concat_and_cache_mla), {dt:.1f} s"}


# ---------------------------------------------------------------------------
# the indexer's per-row top-k (--op topk)
# ---------------------------------------------------------------------------
TOPK_K = 2048
TK_UNIT = "rows/s"


def topk_sets(args, device, n_sets: int, seed0: int = 500):
    g = torch.Generator(device="cpu")
    out = []
    for s in range(n_sets):
        g.manual_seed(seed0 + s)
        out.append(torch.randn((args.rows, args.ctx), generator=g).to(device))
    return out


def topk_desc(args) -> dict:
    return {"workload": f"indexer top-{TOPK_K} per decode row: {args.rows} rows x {args.ctx} "
                        "fp32 logits (the context), seeded N(0, 1)",
            "rows_per_step": args.rows, "ctx": args.ctx, "topk": TOPK_K}


def paged_sets(device, n_sets: int, seed0: int = 1100):
    """C2-shaped decode batches in vLLM's form: 32 sequences (one request
    each, context 8192 = 128 blocks of 64 over a 2048-block pool), request-local
    top-2048 positions in a 2176-column buffer, as the indexer fills it."""
    out = []
    for s in range(n_sets):
        rng = np.random.default_rng(seed0 + s)
        T, ctx, n_blocks, width = 32, 8192, 2048, 2176
        bt = np.stack([rng.permutation(n_blocks)[:ctx // 64] for _ in range(T)]).astype(np.int32)
        pos = np.full((T, width), -1, np.int32)
        for t in range(T):
            pos[t, :2048] = rng.choice(ctx, 2048, replace=False)
        q = torch.from_numpy(rng.standard_normal((T, 64, 512), dtype=np.float32)).to(torch.bfloat16)
        from glm53_sparse_mla import workloads as W
        kv = W.device_pool(n_blocks * 64, seed0 + s, device)
        out.append((q.to(device), kv, torch.from_numpy(pos).to(device),
                    torch.arange(T, dtype=torch.int32, device=device), torch.from_numpy(bt).to(device)))
    return out


def run_paged(args, dist: Dist):
    """--op paged: the attention in vLLM's index form. The fused path
    (sparse_fwd_paged: request-local positions converted to slots inside the
    kernel's index compaction) against the sequence the reference backend runs
    (its backend.py:341-348, 371-378): narrowing copy of the position buffer,
    vLLM's triton_convert_req_index_to_global_index, then sparse_fwd. Both in
    CUDA graphs over rotating input sets; the line's value is the fused path's."""
    torch.cuda.set_device(dist.local)
    device = torch.device("cuda", dist.local)
    dist.init("nccl")
    import glm53_sparse_mla as G
    sets = paged_sets(device, max(1, args.sets))
    outs = [torch.empty_like(s[0]) for s in sets]
    scale = 512 ** -0.5

    def fused(k):
        q, kv, pos, req, bt = sets[k % len(sets)]
        G.sparse_fwd_paged(q, kv, pos, req, bt, 64, scale, topk=2048, out=outs[k % len(sets)])

    stream = torch.cuda.Stream(device)
    ms_local, ms, clocks = time_graph(fused, args, dist, device, stream)
    unfused_ms = None
    try:
        from vllm.v1.attention.backends.mla.sparse_utils import (
            triton_convert_req_index_to_global_index as convert)
        narrow = [torch.empty(s[2].shape[0], 2048, dtype=torch.int32, device=device) for s in sets]

        def unfused(k):
            q, kv, pos, req, bt = sets[k % len(sets)]
            narrow[k % len(sets)].copy_(pos[:, :2048])
            slots = convert(req, bt, narrow[k % len(sets)], BLOCK_SIZE=64, NUM_TOPK_TOKENS=2048)
            torch.ops.glm53_sparse_mla.sparse_fwd(q, kv, slots, scale, 1.0, outs[k % len(sets)])
        unfused_ms = round(graph_ms(unfused, min(args.steps, 50), stream), 5)
    except Exception as e:  # vLLM or Triton unavailable on this host
        unfused_ms = f"unavailable: {type(e).__name__}: {e}"[:200]
    if dist.rank == 0:
        T = sets[0][0].shape[0]
        line = {"metric": f"sparse-MLA {UNIT}, paged index form (C2 batch)",
                "value": round(T * dist.world / (ms / 1e3), 1), "unit": UNIT,
                "n_gpus": dist.world, "steps": args.steps, "warmup": max(args.warmup, 3),
                "ms_per_step": round(ms, 5), "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded)",
                "config": {"workload": "32 decode sequences x 8192 context, 64 heads, top-2048 "
                                       "request-local positions (2176-column buffer), block 64",
                           "parallelism": f"dp{dist.world}",
                           "timing": "K steps in one CUDA graph, CUDA events, max over ranks"},
                "unfused_ms_per_step": unfused_ms,
                "unfused": "narrowing copy + vLLM triton_convert_req_index_to_global_index + "
                           "sparse_fwd (the reference backend's sequence)",
                "gpu_launches": args.steps, "clocks": clocks}
        print(json.dumps(line), flush=True)
    dist.close()


def run_topk(args, dist: Dist):
    torch.cuda.set_device(dist.local)
    device = torch.device("cuda", dist.local)
    dist.init("nccl")
    import glm53_sparse_mla as G
    sets = topk_sets(args, device, max(1, args.sets), 500 + 1000 * dist.rank)
    seq = torch.full((args.rows,), args.ctx, dtype=torch.int32, device=device)
    out = torch.empty((args.rows, TOPK_K), dtype=torch.int32, device=device)

    def step(k):
        G.top_k_per_row_decode(sets[k % len(sets)], 1, seq, out, args.rows, args.ctx, 1, TOPK_K)

    stream = torch.cuda.Stream(device)
    ms_rank, ms_step, clocks = time_graph(step, args, dist, device, stream)
    value = args.rows * dist.world / (ms_step / 1e3)
    alg = args.rows * (args.ctx * 4 + TOPK_K * 4 + 4)
    hbm_peak, _, peak_kind = measured_peaks()
    achieved = alg / (ms_rank / 1e3) / 1e9
    m = None
    prof = os.path.join(REPO, "profiles", "indexer_topk_decode.md")
    if os.path.exists(prof) and (args.rows, args.ctx) == (32, 8192):
        m = re.search(r"traffic_bytes_per_launch:\s*([0-9]+)", open(prof).read())
    roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
            "frac": round(achieved / hbm_peak, 4), "peak_source": peak_kind,
            "traffic": int(m.group(1)) if m else None, "algorithmic_bytes_per_launch": alg,
            "note": "latency-bound: each row is a chain of dependent selection passes on one SM"}
    # vLLM's compiled op of the same contract, timed the same way, for comparison
    vllm_cmp = None
    try:
        from vllm import _custom_ops as ops

        def vstep(k):
            ops.top_k_per_row_decode(sets[k % len(sets)], 1, seq, out, args.rows, args.ctx, 1,
                                     TOPK_K)
        ms_v, _, _ = time_graph(vstep, args, Dist(1), device, stream)
        vllm_cmp = {"op": "vllm._custom_ops.top_k_per_row_decode", "ms_per_step": round(ms_v, 5)}
    except Exception as exc:   # library code, optional
        vllm_cmp = {"unavailable": repr(exc)[:120]}
    e2e = None
    if not args.no_e2e:
        hl = [x.cpu().pin_memory() for x in sets]
        dl = [torch.empty_like(x) for x in sets]
        back = torch.empty(out.shape, dtype=out.dtype).pin_memory()

        def e2e_step(k):
            j = k % len(sets)
            dl[j].copy_(hl[j], non_blocking=True)
            G.top_k_per_row_decode(dl[j], 1, seq, out, args.rows, args.ctx, 1, TOPK_K)
            back.copy_(out, non_blocking=True)

        for k in range(max(args.warmup, 3)):
            e2e_step(k)
        torch.cuda.synchronize()
        dist.barrier()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record()
        for k in range(args.steps):
            e2e_step(k)
        f1.record()
        torch.cuda.synchronize()
        ms_e = dist.max(f0.elapsed_time(f1), device) / args.steps
        e2e = {"value": round(args.rows * dist.world / (ms_e / 1e3), 1), "unit": TK_UNIT,
               "h2d_bytes_per_step": args.rows * args.ctx * 4,
               "d2h_bytes_per_step": args.rows * TOPK_K * 4, "ms_per_step": round(ms_e, 5),
               "path": "glm53_sparse_mla.top_k_per_row_decode (torch op -> C ABI), pinned host "
                       "buffers"}
    cpu = None
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        cpu = topk_cpu(sets[0].cpu().numpy(), args.ctx, args.cpu_seconds)
    if dist.rank == 0:
        cfg = topk_desc(args)
        cfg.update({"parallelism": f"dp{dist.world}",
                    "l2": f"{len(sets)} rotating logits sets "
                          f"({len(sets) * args.rows * args.ctx * 4 / 1e6:.0f} MB); logits are "
                          "fresh from the indexer in use, so L2-resident inputs are the "
                          "realistic case",
                    "timing": "K steps in one CUDA graph, CUDA events, max over ranks"})
        line = {"metric": f"indexer top-{TOPK_K} {TK_UNIT} (decode, ctx {args.ctx})",
                "value": round(value, 1), "unit": TK_UNIT, "n_gpus": dist.world,
                "steps": args.steps, "warmup": max(args.warmup, 3),
                "ms_per_step": round(ms_step, 5), "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)", "config": cfg,
                "roofline": roof, "cpu_baseline": cpu, "e2e": e2e,
                "library_comparison": vllm_cmp,
                "gpu_launches": args.steps + (args.steps if e2e else 0), "clocks": clocks}
        print(json.dumps(line), flush=True)
    dist.close()


def topk_cpu(logits: np.ndarray, ctx: int, seconds: float):
    """The oracle's top-k timed on this host over a sample of the step."""
    from oracle import topk_oracle as TK
    rows = logits.shape[0]
    done, t0 = 0, time.perf_counter()
    while True:
        r = done % rows
        TK.topk_row(logits[r], 0, ctx, TOPK_K)
        done += 1
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    return {"value": round(done / dt, 2), "unit": TK_UNIT, "cores": 1, "kind": "port",
            "sample": f"{done} rows of the step, numpy oracle (restates vLLM's "
                      f"top_k_per_row_decode), {dt:.1f} s"}


def run_topk_reference(args, dist: Dist):
    if dist.rank != 0:
        return
    sets = topk_sets(args, "cpu", 1)
    cpu = topk_cpu(sets[0].numpy(), args.ctx, max(1.0, min(args.cpu_seconds, 30.0)))
    line = {"impl": "reference", "metric": f"indexer top-{TOPK_K} {TK_UNIT} (decode, ctx {args.ctx})",
            "value": cpu["value"], "unit": TK_UNIT, "n_gpus": dist.world, "steps": args.steps,
            "ms_per_step": round(args.rows / cpu["value"] * 1e3, 5),
            "warmup": max(args.warmup, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
            "config": topk_desc(args), "cpu_baseline": cpu,
            "e2e": {"value": cpu["value"], "unit": TK_UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# the indexer's paged fp8 MQA logits (--op indexer)
# ---------------------------------------------------------------------------
IDX_HEADS = 64
IDX_BLOCK = 64
IX_UNIT = "rows/s"


def indexer_sets(args, device, n_sets: int, seed0: int = 700):
    """n_sets independent decode steps: q, weights, an fp8 indexer cache of
    rows x ctx positions (own blocks per row), block tables, lengths."""
    g = torch.Generator(device="cpu")
    blocks_per_row = (args.ctx + IDX_BLOCK - 1) // IDX_BLOCK
    nb = args.rows * blocks_per_row
    out = []
    for s in range(n_sets):
        g.manual_seed(seed0 + s)
        q = torch.randn((args.rows, 1, IDX_HEADS, 128), generator=g).to(torch.float8_e4m3fn)
        vals = torch.randn((nb, IDX_BLOCK * 128), generator=g).to(torch.float8_e4m3fn).view(torch.uint8)
        sc = (torch.rand((nb, IDX_BLOCK), generator=g) + 0.5).view(torch.uint8)
        cache = torch.cat([vals, sc], 1).contiguous().view(nb, IDX_BLOCK, 1, 132)
        w = torch.randn((args.rows, IDX_HEADS), generator=g)
        bt = torch.randperm(nb, generator=g).to(torch.int32).view(args.rows, blocks_per_row)
        out.append(tuple(x.to(device) for x in (q, cache, w, bt)))
    ctx = torch.full((args.rows,), args.ctx, dtype=torch.int32, device=device)
    return out, ctx


def indexer_bytes(args) -> int:
    """Algorithmic bytes per launch: cache rows and scales read once, queries
    and weights, logits written over max_model_len (= ctx here)."""
    return args.rows * (args.ctx * 132 + IDX_HEADS * 128 + IDX_HEADS * 4 + args.ctx * 4)


def indexer_desc(args) -> dict:
    return {"workload": f"indexer fp8 paged MQA logits: {args.rows} decode rows x {args.ctx} "
                        f"cached positions, {IDX_HEADS} heads x 128, block {IDX_BLOCK}",
            "rows_per_step": args.rows, "ctx": args.ctx, "heads": IDX_HEADS}


def run_indexer(args, dist: Dist):
    torch.cuda.set_device(dist.local)
    device = torch.device("cuda", dist.local)
    dist.init("nccl")
    import glm53_sparse_mla as G
    sets, ctx = indexer_sets(args, device, max(1, args.sets), 700 + 1000 * dist.rank)
    logits = torch.empty((args.rows, args.ctx), dtype=torch.float32, device=device)

    def step(k):
        q, cache, w, bt = sets[k % len(sets)]
        G.fp8_paged_mqa_logits(q, cache, w, ctx, bt, args.ctx, logits=logits)

    stream = torch.cuda.Stream(device)
    ms_rank, ms_step, clocks = time_graph(step, args, dist, device, stream)
    value = args.rows * dist.world / (ms_step / 1e3)
    alg = indexer_bytes(args)
    hbm_peak, tf_peak, peak_kind = measured_peaks()
    achieved = alg / (ms_rank / 1e3) / 1e9
    m = None
    prof = os.path.join(REPO, "profiles", "indexer_logits_decode.md")
    if os.path.exists(prof) and (args.rows, args.ctx) == (32, 8192):
        m = re.search(r"traffic_bytes_per_launch:\s*([0-9]+)", open(prof).read())
    flops = 2 * args.rows * args.ctx * IDX_HEADS * 128
    roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
            "frac": round(achieved / hbm_peak, 4), "peak_source": peak_kind,
            "traffic": int(m.group(1)) if m else None, "algorithmic_bytes_per_launch": alg,
            "tensor_tflops_fp8": round(flops / (ms_rank / 1e3) / 1e12, 1)}
    e2e = None
    if not args.no_e2e:
        hq = [s[0].cpu().pin_memory() for s in sets]
        hw = [s[2].cpu().pin_memory() for s in sets]
        dq = [torch.empty_like(s[0]) for s in sets]
        dw = [torch.empty_like(s[2]) for s in sets]
        back = torch.empty(logits.shape, dtype=logits.dtype).pin_memory()

        def e2e_step(k):
            j = k % len(sets)
            dq[j].copy_(hq[j], non_blocking=True)
            dw[j].copy_(hw[j], non_blocking=True)
            G.fp8_paged_mqa_logits(dq[j], sets[j][1], dw[j], ctx, sets[j][3], args.ctx,
                                   logits=logits)
            back.copy_(logits, non_blocking=True)

        for k in range(max(args.warmup, 3)):
            e2e_step(k)
        torch.cuda.synchronize()
        dist.barrier()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record()
        for k in range(args.steps):
            e2e_step(k)
        f1.record()
        torch.cuda.synchronize()
        ms_e = dist.max(f0.elapsed_time(f1), device) / args.steps
        e2e = {"value": round(args.rows * dist.world / (ms_e / 1e3), 1), "unit": IX_UNIT,
               "h2d_bytes_per_step": args.rows * IDX_HEADS * (128 + 4),
               "d2h_bytes_per_step": args.rows * args.ctx * 4, "ms_per_step": round(ms_e, 5),
               "path": "glm53_sparse_mla.fp8_paged_mqa_logits (torch op -> C ABI), pinned host "
                       "buffers; the cache is resident device state"}
    cpu = None
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        cpu = indexer_cpu(sets[0], args, args.cpu_seconds)
    if dist.rank == 0:
        cfg = indexer_desc(args)
        cfg.update({"parallelism": f"dp{dist.world}",
                    "l2": f"{len(sets)} rotating caches, "
                          f"{len(sets) * args.rows * args.ctx * 132 / 1e6:.0f} MB (>> 126 MB L2)",
                    "timing": "K steps in one CUDA graph, CUDA events, max over ranks"})
        line = {"metric": f"indexer logits {IX_UNIT} (decode, ctx {args.ctx}, {IDX_HEADS} heads)",
                "value": round(value, 1), "unit": IX_UNIT, "n_gpus": dist.world,
                "steps": args.steps, "warmup": max(args.warmup, 3),
                "ms_per_step": round(ms_step, 5), "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "fp8_e4m3", "data": "synthetic (seeded)",
                "config": cfg, "roofline": roof, "cpu_baseline": cpu, "e2e": e2e,
                "gpu_launches": args.steps + (args.steps if e2e else 0), "clocks": clocks}
        print(json.dumps(line), flush=True)
    dist.close()


def indexer_cpu(one_set, args, seconds: float):
    """The oracle's logits timed on this host, one row at a time."""
    from oracle import indexer_logits_oracle as IL
    q, cache, w, bt = (x.cpu() for x in one_set)
    qb = q.view(torch.uint8).numpy()
    kv = cache.view(cache.shape[0], -1).numpy()
    wn, btn = w.numpy(), bt.numpy()
    done, t0 = 0, time.perf_counter()
    while True:
        r = done % args.rows
        IL.paged_mqa_logits(qb[r:r + 1], kv, wn[r:r + 1], np.array([args.ctx]), btn[r:r + 1],
                            args.ctx)
        done += 1
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    return {"value": round(done / dt, 2), "unit": IX_UNIT, "cores": 1, "kind": "port",
            "sample": f"{done} rows of the step, numpy oracle (restates vLLM's "
                      f"fp8_paged_mqa_logits_torch), {dt:.1f} s"}


def run_indexer_reference(args, dist: Dist):
    if dist.rank != 0:
        return
    sets, _ = indexer_sets(args, "cpu", 1)
    cpu = indexer_cpu(sets[0], args, max(1.0, min(args.cpu_seconds, 30.0)))
    line = {"impl": "reference",
            "metric": f"indexer logits {IX_UNIT} (decode, ctx {args.ctx}, {IDX_HEADS} heads)",
            "value": cpu["value"], "unit": IX_UNIT, "n_gpus": dist.world, "steps": args.steps,
            "ms_per_step": round(args.rows / cpu["value"] * 1e3, 5),
            "warmup": max(args.warmup, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
            "config": indexer_desc(args), "cpu_baseline": cpu,
            "e2e": {"value": cpu["value"], "unit": IX_UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# the whole sparse decode step (--op decode_step)
# ---------------------------------------------------------------------------
def decode_step_sets(args, device, n_sets: int, seed0: int = 900):
    """Per set: a paged bf16 latent cache and an fp8 indexer cache sharing one
    block table (rows x ctx positions, block 64), plus the step's inputs: each
    request's new latent row, indexer queries and weights, attention queries."""
    g = torch.Generator(device="cpu")
    bpr = (args.ctx + IDX_BLOCK - 1) // IDX_BLOCK
    nb = args.rows * bpr
    out = []
    for s in range(n_sets):
        g.manual_seed(seed0 + s)
        bt = torch.randperm(nb, generator=g).to(torch.int32).view(args.rows, bpr)
        lat = (torch.randn((nb, IDX_BLOCK, 512), generator=g) * 0.5).to(torch.bfloat16)
        vals = torch.randn((nb, IDX_BLOCK * 128), generator=g).to(torch.float8_e4m3fn).view(torch.uint8)
        sc = (torch.rand((nb, IDX_BLOCK), generator=g) + 0.5).view(torch.uint8)
        icache = torch.cat([vals, sc], 1).contiguous().view(nb, IDX_BLOCK, 1, 132)
        qi = torch.randn((args.rows, 1, IDX_HEADS, 128), generator=g).to(torch.float8_e4m3fn)
        w = torch.randn((args.rows, IDX_HEADS), generator=g)
        q = torch.randn((args.rows, 64, 512), generator=g).to(torch.bfloat16)
        kv_new = torch.randn((args.rows, 512), generator=g).to(torch.bfloat16)
        # the new token of request r sits at position ctx - 1 of its table
        last = args.ctx - 1
        slots = (bt[:, last // IDX_BLOCK].to(torch.int64) * IDX_BLOCK + last % IDX_BLOCK)
        out.append({k: v.to(device) for k, v in dict(
            bt=bt, lat=lat, icache=icache, qi=qi, w=w, q=q, kv_new=kv_new, slots=slots).items()})
    return out


def run_decode_step(args, dist: Dist):
    torch.cuda.set_device(dist.local)
    device = torch.device("cuda", dist.local)
    dist.init("nccl")
    import glm53_sparse_mla as G
    sets = decode_step_sets(args, device, max(1, min(args.sets, 3)), 900 + 1000 * dist.rank)
    ctx = torch.full((args.rows,), args.ctx, dtype=torch.int32, device=device)
    req = torch.arange(args.rows, dtype=torch.int32, device=device)
    logits = torch.empty((args.rows, args.ctx), dtype=torch.float32, device=device)
    pos = torch.empty((args.rows, TOPK_K), dtype=torch.int32, device=device)
    out = torch.empty((args.rows, 64, 512), dtype=torch.bfloat16, device=device)
    one = torch.ones(1, dtype=torch.float32, device=device)

    def step(k):
        d = sets[k % len(sets)]
        G.concat_and_cache_mla(d["kv_new"], d["kv_new"][:, :0], d["lat"], d["slots"], "auto", one)
        G.fp8_paged_mqa_logits(d["qi"], d["icache"], d["w"], ctx, d["bt"], args.ctx, logits=logits)
        G.top_k_per_row_decode(logits, 1, ctx, pos, args.rows, args.ctx, 1, TOPK_K)
        G.sparse_fwd_paged(d["q"], d["lat"].view(-1, 512), pos, req, d["bt"], IDX_BLOCK,
                           512 ** -0.5, out=out)

    stream = torch.cuda.Stream(device)
    ms_rank, ms_step, clocks = time_graph(step, args, dist, device, stream)
    value = args.rows * dist.world / (ms_step / 1e3)
    # the same step with vLLM's compiled top-k in place of this repo's, timed
    # the same way: inside the step a kernel's code is cold at every launch,
    # which a graph of top-k launches alone does not show
    vllm_cmp = None
    if dist.world == 1:
        try:
            from vllm import _custom_ops as ops

            def vstep(k):
                d = sets[k % len(sets)]
                G.concat_and_cache_mla(d["kv_new"], d["kv_new"][:, :0], d["lat"], d["slots"], "auto", one)
                G.fp8_paged_mqa_logits(d["qi"], d["icache"], d["w"], ctx, d["bt"], args.ctx, logits=logits)
                ops.top_k_per_row_decode(logits, 1, ctx, pos, args.rows, args.ctx, 1, TOPK_K)
                G.sparse_fwd_paged(d["q"], d["lat"].view(-1, 512), pos, req, d["bt"], IDX_BLOCK,
                                   512 ** -0.5, out=out)
            ms_v, _, _ = time_graph(vstep, args, Dist(1), device, stream)
            vllm_cmp = {"top_k": "vllm._custom_ops.top_k_per_row_decode", "ms_per_step": round(ms_v, 5)}
        except Exception as exc:   # library code, optional
            vllm_cmp = {"unavailable": repr(exc)[:120]}
    if dist.rank == 0:
        line = {"metric": f"sparse decode step query-tokens/s (cache write + indexer logits + "
                          f"top-{TOPK_K} + attention, ctx {args.ctx}, 64 heads)",
                "value": round(value, 1), "unit": UNIT, "n_gpus": dist.world,
                "steps": args.steps, "warmup": max(args.warmup, 3),
                "ms_per_step": round(ms_step, 5), "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "bf16 attention, fp8 indexer",
                "data": "synthetic (seeded)",
                "config": {"workload": f"{args.rows} decode sequences x {args.ctx} cached tokens: "
                                       "latent cache write (bf16), indexer fp8 paged logits "
                                       f"({IDX_HEADS} heads), top-{TOPK_K}, paged sparse-MLA "
                                       "attention (64 heads) on the top-k positions",
                           "rows": args.rows, "ctx": args.ctx, "parallelism": f"dp{dist.world}",
                           "timing": "K steps in one CUDA graph, CUDA events, max over ranks"},
                "gpu_launches": 4 * args.steps, "clocks": clocks}
        if vllm_cmp is not None:
            line["library_comparison"] = vllm_cmp
        print(json.dumps(line), flush=True)
    dist.close()


def run_e2e(args, G, sets, device, dist: Dist):
    n = len(sets)
    q_h = [w.q.cpu().pin_memory() for w in sets]
    i_h = [w.indices.cpu().pin_memory() for w in sets]
    o_h = [torch.empty(w.q.shape, dtype=torch.bfloat16).pin_memory() for w in sets]
    q_d = [torch.empty_like(w.q) for w in sets]
    i_d = [torch.empty_like(w.indices) for w in sets]
    o_d = [torch.empty_like(w.q) for w in sets]
    steps = args.steps

    # one stream per input set: a step's copy in, op and copy out are ordered
    # on its set's stream, and consecutive steps (other sets) overlap on the
    # copy engines and the SMs, as a serving loop's steps would
    streams = [torch.cuda.Stream(device) for _ in range(n)]
    main = torch.cuda.current_stream(device)

    def step(k):
        j = k % n
        w = sets[j]
        with torch.cuda.stream(streams[j]):
            q_d[j].copy_(q_h[j], non_blocking=True)
            i_d[j].copy_(i_h[j], non_blocking=True)
            G.sparse_fwd(q_d[j], w.kv, i_d[j], w.sm_scale, w.kv_scale, out=o_d[j])
            o_h[j].copy_(o_d[j], non_blocking=True)

    # warm every input set's stream (at least W steps): the op's first call on
    # a stream takes its split-merge workspace from the caching allocator,
    # which then holds it for that stream
    for k in range(max(args.warmup, 3, n)):
        step(k)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dist.barrier()
    torch.cuda.synchronize()
    e0.record(main)
    for s in streams:
        s.wait_stream(main)
    for k in range(steps):
        step(k)
    for s in streams:
        main.wait_stream(s)
    e1.record(main)
    torch.cuda.synchronize()
    dist.barrier()
    ms = dist.max(e0.elapsed_time(e1), device)

    # the same loop with the op left out: the host-copy floor of the step on
    # this box (outside the timed region above)
    def copies(k):
        j = k % n
        with torch.cuda.stream(streams[j]):
            q_d[j].copy_(q_h[j], non_blocking=True)
            i_d[j].copy_(i_h[j], non_blocking=True)
            o_h[j].copy_(o_d[j], non_blocking=True)

    for k in range(max(args.warmup, 3)):
        copies(k)
    torch.cuda.synchronize()
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c0.record(main)
    for s in streams:
        s.wait_stream(main)
    for k in range(steps):
        copies(k)
    for s in streams:
        main.wait_stream(s)
    c1.record(main)
    torch.cuda.synchronize()
    copy_ms = c0.elapsed_time(c1) / steps
    w = sets[0]
    units = w.T * (dist.world if args.shard == "tokens" else 1)
    return {"value": round(units / (ms / steps / 1e3), 1), "unit": UNIT,
            "copy_floor_ms": round(copy_ms, 5),
            "h2d_bytes_per_step": int(w.q.numel() * 2 + w.indices.numel() * 4),
            "d2h_bytes_per_step": int(w.q.numel() * 2),
            "ms_per_step": round(ms / steps, 5),
            "path": "glm53_sparse_mla.sparse_fwd (torch op -> C ABI), pinned host buffers; "
                    "each step's H2D, op and D2H on its input set's stream, consecutive steps "
                    f"overlapped across {n} streams"}


def _oracle_inputs(w, W=None):
    if W is None:
        from glm53_sparse_mla import workloads as W
    kv = W.dequantize_fp8(w.kv, w.kv_scale) if w.kv.dtype == torch.float8_e4m3fn else w.kv
    return (w.q.float().cpu().numpy(), kv.float().cpu().numpy(), w.indices.cpu().numpy())


def cpu_baseline(w, seconds: float, heads: int | None = None):
    """Oracle tokens/s on this host over a bounded sample of the workload."""
    from oracle import sparse_mla_oracle as O
    q, kv, idx = _oracle_inputs(w)
    if heads:
        q = np.ascontiguousarray(q[:, :heads])
    try:
        from threadpoolctl import threadpool_info
        cores = max((i.get("num_threads", 1) for i in threadpool_info()), default=1)
    except Exception:  # pragma: no cover
        cores = os.cpu_count() or 1
    O.sparse_mla_stats(q[:1], kv, idx[:1], w.sm_scale, chunk=1)    # warm
    done, t0 = 0, time.perf_counter()
    while True:
        j = done % w.T
        O.sparse_mla_stats(q[j:j + 1], kv, idx[j:j + 1], w.sm_scale, chunk=1)
        done += 1
        if time.perf_counter() - t0 >= seconds and done >= 1:
            break
    dt = time.perf_counter() - t0
    frac = (heads or w.H) / w.H
    return {"value": round(done * frac / dt, 2), "unit": UNIT, "cores": int(cores),
            "kind": "port",
            "sample": f"{done} query tokens of the same workload, one at a time"
                      f"{'' if not heads else f', {heads} of {w.H} heads (scaled)'}"
                      f", numpy fp32 oracle (restates the reference's tests/reference.py), "
                      f"{dt:.1f} s"}


def _workloads_standalone():
    """workloads.py loaded by file path, without importing the package: the
    package import loads the CUDA extension, which the reference arm must not
    map."""
    import importlib.util
    path = os.path.join(REPO, "vllm-sparse-mla-blackwell_b200", "glm53_sparse_mla", "workloads.py")
    spec = importlib.util.spec_from_file_location("_glm53_workloads_standalone", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod
    spec.loader.exec_module(mod)
    return mod


def run_reference(args, dist: Dist):
    """Reference arm: the reference's CPU implementation of the path (the
    oracle port) on the host cores, rank 0 only; other ranks exit at once.
    Inputs are generated on the host and nothing of this repository's CUDA
    extension is loaded."""
    if dist.rank != 0:
        return
    # torchrun pins OMP threads to 1 per rank; the CPU arm uses every core
    try:
        from threadpoolctl import threadpool_limits
        threadpool_limits(limits=os.cpu_count() or 1)
    except Exception:  # pragma: no cover
        pass
    W = _workloads_standalone()
    w = make_workload(args, W, 100, "cpu", 0)
    from oracle import sparse_mla_oracle as O
    q, kv, idx = _oracle_inputs(w, W)
    # size each step (one query token; a head slice of it if K is large) so
    # the whole run stays within about three minutes
    t0 = time.perf_counter()
    O.sparse_mla_stats(q[:1], kv, idx[:1], w.sm_scale, chunk=1)
    t_tok = max(time.perf_counter() - t0, 1e-4)
    n_total = max(args.steps, 1) + max(args.warmup, 3)
    heads = w.H
    while heads > 1 and n_total * t_tok * heads / w.H > 180.0:
        heads //= 2
    qs = np.ascontiguousarray(q[:, :heads])
    for k in range(max(args.warmup, 3)):
        j = k % w.T
        O.sparse_mla_stats(qs[j:j + 1], kv, idx[j:j + 1], w.sm_scale, chunk=1)
    t0 = time.perf_counter()
    for k in range(args.steps):
        j = k % w.T
        O.sparse_mla_stats(qs[j:j + 1], kv, idx[j:j + 1], w.sm_scale, chunk=1)
    dt = time.perf_counter() - t0
    value = args.steps * (heads / w.H) / dt
    try:
        from threadpoolctl import threadpool_info
        cores = max((i.get("num_threads", 1) for i in threadpool_info()), default=1)
    except Exception:  # pragma: no cover
        cores = os.cpu_count() or 1
    sample = (f"one query token per step ({heads} of {w.H} heads, scaled), numpy fp32 oracle "
              "restating the reference's tests/reference.py")
    heads_total = 64 if args.workload in ("c2", "c5") else (32 if args.workload == "c3" else 16)
    if args.heads:
        heads_total = args.heads
    line = {"impl": "reference", "metric": METRIC if args.workload == "c2" else
            f"sparse-MLA {UNIT} ({args.workload})", "value": round(value, 3), "unit": UNIT,
            "n_gpus": dist.world, "steps": args.steps, "warmup": max(args.warmup, 3),
            "ms_per_step": round(dt / args.steps * 1e3, 4), "higher_is_better": True,
            "scaling": "weak" if args.shard == "tokens" else "strong",
            "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded, random init)",
            "config": attention_config(args, w, heads_total, dist.world),
            "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": int(cores),
                             "kind": "port", "sample": sample},
            "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_cache_write_reference(args, dist: Dist):
    """Reference arm of --op cache_write: the oracle's restatement of vLLM's
    write timed on the host, rank 0 only."""
    if dist.rank != 0:
        return
    fp8 = args.kv == "fp8"
    sets = cache_write_sets(args, "cpu", 1)
    cpu = cache_write_cpu(sets[0], fp8, max(1.0, min(args.cpu_seconds, 30.0)))
    line = {"impl": "reference", "metric": f"latent KV-cache writes ({args.kv}), {CW_UNIT}",
            "value": cpu["value"], "unit": CW_UNIT, "n_gpus": dist.world, "steps": args.steps,
            "ms_per_step": round(args.tokens / cpu["value"] * 1e3, 5),
            "warmup": max(args.warmup, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
            "config": cache_write_desc(args, fp8), "cpu_baseline": cpu,
            "e2e": {"value": cpu["value"], "unit": CW_UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    dist = Dist(args.gpus)
    if args.op == "cache_write":
        if args.impl == "reference":
            run_cache_write_reference(args, dist)
        else:
            run_cache_write(args, dist)
    elif args.op == "decode_step":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the reference has no CPU "
                              "implementation of the indexer or the cache writer; its arms are "
                              "--op attention, cache_write, indexer and topk"}), flush=True)
        else:
            run_decode_step(args, dist)
    elif args.op == "paged":
        if args.impl == "reference":
            run_reference(args, dist)
        else:
            run_paged(args, dist)
    elif args.op == "indexer":
        if args.impl == "reference":
            run_indexer_reference(args, dist)
        else:
            run_indexer(args, dist)
    elif args.op == "topk":
        if args.impl == "reference":
            run_topk_reference(args, dist)
        else:
            run_topk(args, dist)
    elif args.impl == "reference":
        run_reference(args, dist)
    else:
        run_ours(args, dist)


if __name__ == "__main__":
    main()
