"""The fused head gather (glm53_sparse_mla_fwd_heads_gather and the torch op
sparse_fwd_gather_heads) on a B200.

One rank of a head-sharded group writes its heads straight into every
rank's full [T, heads_total, 512] output. On one GPU the "ranks' buffers" are
several local tensors, which exercises the multi-output epilogue of every
merge path without NVLink; with two or more GPUs, HeadShardGather runs over
symmetric memory and each rank's gathered output must equal the 64-head
result computed on one GPU, bit for bit (heads are independent).
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

import glm53_sparse_mla as G  # noqa: E402
from glm53_sparse_mla import sharding as S  # noqa: E402
from glm53_sparse_mla import workloads as W  # noqa: E402

SENTINEL = -7.0


@pytest.mark.parametrize("kv_dtype", ["bf16", "fp8"])
@pytest.mark.parametrize("shape", [("c2", 16, 32), ("c2", 8, 16), ("c1", 16, 0), ("case", 32, 32)])
def test_multi_output_epilogue_matches_plain_op(shape, kv_dtype):
    which, heads, offset = shape
    if which == "c2":
        full = W.config_c2(device="cuda")                 # 4 CTAs per token: L2 merge
    elif which == "c1":
        full = W.config_c1(device="cuda")                 # 1 CTA per token
    else:
        full = next(iter(W.case_matrix(heads=64, topk=2048, rows=8192, device="cuda",
                                       kv_dtype=kv_dtype)))
    if which != "case" and kv_dtype == "fp8":
        full = W.Workload(full.name, full.q, W.quantize_fp8(full.kv.float(), 0.05).contiguous(),
                          full.indices, full.sm_scale, 0.05)
    q = full.q[:, offset:offset + heads].contiguous()
    ref = G.sparse_fwd(q, full.kv, full.indices, full.sm_scale, full.kv_scale)
    T, total = q.shape[0], max(64, offset + heads)
    bufs = [torch.full((T, total, 512), SENTINEL, dtype=torch.bfloat16, device="cuda")
            for _ in range(3)]
    ptrs = [b.data_ptr() for b in bufs]
    for rank in (0, 2):   # own buffer at index `rank`
        torch.ops.glm53_sparse_mla.sparse_fwd_gather_heads(
            q, full.kv, full.indices, full.sm_scale, full.kv_scale, ptrs, rank, offset, bufs[rank])
    torch.cuda.synchronize()
    for b in bufs:
        assert torch.equal(b[:, offset:offset + heads], ref), "gathered heads differ from the op"
        rest = torch.cat([b[:, :offset], b[:, offset + heads:]], dim=1)
        assert (rest == SENTINEL).all(), "heads outside this rank's slice were written"


def test_copy_head_slices_places_one_ranks_heads():
    """glm53_copy_head_slices: this rank's head slice of every token lands in
    the same place of each destination; other heads and the source itself
    are untouched."""
    import ctypes
    lib = ctypes.CDLL(G.library_path())
    f = lib.glm53_copy_head_slices
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                  ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p]
    T, total, off, h = 37, 64, 16, 16
    src = torch.randn(T, total, 512, device="cuda").to(torch.bfloat16)
    dsts = [torch.full((T, total, 512), SENTINEL, dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    keep = src.clone()
    arr = (ctypes.c_void_p * 3)(dsts[0].data_ptr(), src.data_ptr(), dsts[1].data_ptr())
    assert f(arr, 3, src.data_ptr(), T, total, off, h, torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    assert torch.equal(src, keep)
    for d in dsts:
        assert torch.equal(d[:, off:off + h], src[:, off:off + h])
        assert (d[:, :off] == SENTINEL).all() and (d[:, off + h:] == SENTINEL).all()
    assert f(arr, 3, src.data_ptr(), T, total, 56, h, None) == 1      # heads past the buffer


def test_op_rejects_bad_arguments():
    w = W.config_c1(device="cuda")
    buf = torch.empty(w.T, 64, 512, dtype=torch.bfloat16, device="cuda")
    op = torch.ops.glm53_sparse_mla.sparse_fwd_gather_heads
    with pytest.raises(RuntimeError):      # own buffer not at index rank
        op(w.q, w.kv, w.indices, w.sm_scale, 1.0, [buf.data_ptr() + 1024], 0, 0, buf)
    with pytest.raises(RuntimeError):      # heads past the buffer
        op(w.q, w.kv, w.indices, w.sm_scale, 1.0, [buf.data_ptr()], 0, 56, buf)
    with pytest.raises(RuntimeError):      # more than 8 outputs
        op(w.q, w.kv, w.indices, w.sm_scale, 1.0, [buf.data_ptr()] * 9, 0, 0, buf)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, result_path: str):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    import datetime
    torch.distributed.init_process_group("nccl", rank=rank, world_size=world,
                                         timeout=datetime.timedelta(seconds=60),
                                         device_id=torch.device("cuda", rank))
    bad = ["not run"]
    try:
        full = W.config_c2(device="cuda", seed=31)
        q = S.shard_heads(full.q, rank, world)
        bad = []
        for mode, chunk in (("fused", None), ("copy", None), ("copy", 7)):
            # the 64-head op on the same token waves as the gather (the split
            # plan depends on a launch's token count), so equal bit for bit
            step = chunk or full.T
            ref = torch.cat([G.sparse_fwd(full.q[t:t + step], full.kv, full.indices[t:t + step], full.sm_scale)
                             for t in range(0, full.T, step)])
            gather = S.HeadShardGather(full.T, 64, mode=mode, chunk_tokens=chunk)
            for it in range(2):             # twice: the buffer is reused
                out = gather(q, full.kv, full.indices, full.sm_scale)
                torch.cuda.synchronize()
                if not torch.equal(out, ref):
                    d = (out.float() - ref.float()).abs().max().item()
                    bad.append(f"{mode}/chunk={chunk}/call{it}: max|diff| {d:.3e}")
            torch.distributed.barrier()
            del gather
    finally:
        with open(f"{result_path}.{rank}", "w") as f:
            f.write("ok" if not bad else "; ".join(bad))
        torch.distributed.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_head_shard_gather_over_symmetric_memory(tmp_path):
    world = 2
    path = str(tmp_path / "result")
    mp.start_processes(_rank_main, args=(world, _free_port(), path), nprocs=world,
                       start_method="spawn", join=True)
    for r in range(world):
        got = open(f"{path}.{r}").read()
        assert got == "ok", f"rank {r}: gathered output differs: {got}"
