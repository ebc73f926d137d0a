"""Generate the golden vectors that pin oracle/sparse_mla_oracle.py.

Run in a checkout that has the reference mounted (it is NOT needed at test
time):

    python tests/golden/make_golden.py /path/to/vllm-sparse-mla-blackwell

It imports the reference's own ground truth, ``sparse_mla_fp32`` from
tests/reference.py of jsmcconn/vllm-sparse-mla-blackwell, runs it on CPU over
seeded inputs from glm53_sparse_mla.workloads (the case matrix at small size,
config C1, and the compaction edge cases) and stores inputs and outputs in
tests/golden/sparse_mla_golden.npz. The inputs themselves are not stored:
they are regenerated bit-exactly from numpy PCG64 seeds by the same
generator, and a SHA-256 of their bytes guards against generator drift.

  <case>/input_sha256             sha256 of q, kv, indices bytes (uint8[32])
  <case>/sm_scale                 float32 scalar
  <case>/out                      float32 [T, H, 512] reference output
  <case>/lse                      float32 [T, H] reference lse (its formula)
"""

from __future__ import annotations

import hashlib
import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "vllm-sparse-mla-blackwell_b200"))

from glm53_sparse_mla import workloads as W  # noqa: E402


def load_reference(ref_root: str):
    path = os.path.join(ref_root, "tests", "reference.py")
    spec = importlib.util.spec_from_file_location("reference_oracle", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.sparse_mla_fp32


def input_digest(c) -> np.ndarray:
    h = hashlib.sha256()
    for t in (c.q, c.kv, c.indices):
        h.update(t.contiguous().view(torch.uint8).numpy().tobytes())
    return np.frombuffer(h.digest(), dtype=np.uint8)


def golden_cases():
    """The inputs the fixtures cover; tests/test_oracle_golden.py calls this too."""
    cases = list(W.case_matrix(heads=4, topk=128, rows=1024, device="cpu", seed=11))
    cases = [c for c in cases if c.name != "tokens_128"]
    cases.append(W.config_c1(device="cpu"))
    edge = W.edge_cases(heads=4, topk=256, rows=1024, device="cpu")
    # the reference oracle indexes rows directly: give it the out-of-range ids
    # already masked, which is what the kernel does with them
    edge.indices = torch.where(edge.indices >= 1024, torch.full_like(edge.indices, -1),
                               edge.indices)
    cases.append(edge)
    return cases


def main(ref_root: str) -> None:
    ref = load_reference(ref_root)
    blob = {}
    for c in golden_cases():
        out, lse = ref(c.q, c.kv, c.indices, c.sm_scale)
        blob[f"{c.name}/input_sha256"] = input_digest(c)
        blob[f"{c.name}/sm_scale"] = np.float32(c.sm_scale)
        blob[f"{c.name}/out"] = out.numpy().astype(np.float32)
        blob[f"{c.name}/lse"] = lse.numpy().astype(np.float32)
        print(f"{c.name:22s} T={c.T:3d} H={c.H:2d} topk={c.topk:4d} "
              f"valid={c.n_valid():6d}")
    dst = os.path.join(HERE, "sparse_mla_golden.npz")
    np.savez_compressed(dst, **blob)
    print("wrote", dst, os.path.getsize(dst), "bytes")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
