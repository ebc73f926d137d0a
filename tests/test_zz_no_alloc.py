"""The no-allocation entry point, glm53_sparse_mla_fwd_noalloc.

It serves callers that cannot allocate device memory when they call
attention (a fixed-size memory pool, an allocator the call site cannot
reach, a runtime that forbids cudaMalloc after start-up): its split-merge
scratch is a 32 MiB array built into the library. These tests call it
through the C ABI and compare it with glm53_sparse_mla_fwd on the same
inputs, within the parity tolerance used everywhere else, on two calls in a
row (the scratch keeps the first call's contents when the second one runs),
and with the CPU oracle directly, and check that a shape needing more scratch than the array holds is refused
before any launch.

The file name makes pytest collect it last.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from conftest import COS_TOL, REL_TOL, parity_metrics
from test_parity_gpu import _check, _oracle

pytestmark = pytest.mark.gpu

import glm53_sparse_mla as G  # noqa: E402
from glm53_sparse_mla import workloads as W  # noqa: E402

_ARGS = [ctypes.c_void_p] * 5 + [ctypes.c_int64] * 6 + [
    ctypes.c_int, ctypes.c_float, ctypes.c_float, ctypes.c_int, ctypes.c_void_p]
ERR_SCRATCH_LIMIT = 11


def _lib():
    lib = ctypes.CDLL(G.library_path())
    for name in ("glm53_sparse_mla_fwd", "glm53_sparse_mla_fwd_noalloc"):
        fn = getattr(lib, name)
        fn.restype = ctypes.c_int
        fn.argtypes = _ARGS
    return lib


def _call(fn, w: W.Workload, splits: int):
    out = torch.full_like(w.q, float("nan"))
    lse = torch.full((w.T, w.H), float("nan"), device=w.q.device)
    kvd = 1 if w.kv.dtype == torch.float8_e4m3fn else 0
    rc = fn(w.q.data_ptr(), w.kv.data_ptr(), w.indices.data_ptr(), out.data_ptr(), lse.data_ptr(),
            w.T, w.H, 512, w.kv.shape[0], 512, w.topk, kvd, w.sm_scale, w.kv_scale, splits,
            torch.cuda.current_stream().cuda_stream)
    return rc, out, lse


def _same(got: torch.Tensor, ref: torch.Tensor, name: str):
    rel, cmin, finite = parity_metrics(got.float().cpu().numpy(), ref.float().cpu().numpy())
    assert finite, name
    assert rel <= REL_TOL and cmin >= COS_TOL, f"{name}: rel={rel:.3e} cos={cmin:.7f}"


def test_noalloc_matches_fwd_on_two_calls_in_a_row():
    lib = _lib()
    first = W.config_c2(device="cuda", seed=21)                       # 64 heads, 4 CTAs per token
    second = next(iter(W.case_matrix(heads=32, topk=2048, rows=8192, device="cuda", seed=22)))
    for w, splits in ((first, 0), (second, 8)):
        rc_ref, ref, ref_lse = _call(lib.glm53_sparse_mla_fwd, w, splits)
        rc, got, lse = _call(lib.glm53_sparse_mla_fwd_noalloc, w, splits)
        torch.cuda.synchronize()
        assert rc_ref == 0 and rc == 0, (rc_ref, rc)
        _same(got, ref, f"{w.name}/splits={splits}")
        # and against the CPU oracle directly, on the second call too, when
        # the scratch still holds the first call's partials
        oref, _ = _oracle(w)
        _check(f"{w.name}/noalloc/splits={splits}", got, oref, w.indices)
        fin = torch.isfinite(ref_lse)
        assert torch.equal(fin, torch.isfinite(lse))
        assert (lse[fin] - ref_lse[fin]).abs().max().item() <= 1e-3


def test_noalloc_refuses_shapes_beyond_its_scratch():
    lib = _lib()
    w = next(iter(W.case_matrix(heads=64, topk=2048, rows=8192, device="cuda", seed=23)))
    # 8 CTAs per token x 64 heads needs T * 8 * 131,072 B of scratch: above 32 MiB once
    # T > 32, so a 64-token batch is refused before anything is launched.
    q = w.q.repeat(64 // w.T + 1, 1, 1)[:64].contiguous()
    idx = w.indices.repeat(64 // w.T + 1, 1)[:64].contiguous()
    big = W.Workload("big", q, w.kv, idx, w.sm_scale)
    rc, out, _ = _call(lib.glm53_sparse_mla_fwd_noalloc, big, 8)
    torch.cuda.synchronize()
    assert rc == ERR_SCRATCH_LIMIT, rc
    assert torch.isnan(out.float()).all(), "a refused call must not write its output"
