"""Multi-rank host logic on CPU: world_size-2 gloo process groups.

Each rank runs the CPU oracle on its shard (a stand-in for the kernel, which
needs a GPU) and the shards are reassembled with the package's collective
helper. Head sharding must reproduce the full 64-head result exactly, since
heads are independent; token sharding must cover every token once.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from glm53_sparse_mla import sharding as S
from glm53_sparse_mla import workloads as W
from oracle import sparse_mla_oracle as O


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_out(q: torch.Tensor, w: W.Workload) -> np.ndarray:
    out, _, _ = O.sparse_mla_stats(q.float().numpy(), w.kv.float().numpy(),
                                   w.indices.numpy(), w.sm_scale)
    return out


def _worker(rank: int, world: int, port: int, mode: str, q_path: str):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = next(iter(W.case_matrix(heads=16, topk=128, rows=1024, device="cpu")))
        q = torch.cat([w.q, w.q.flip(1) * 0.5], dim=1)          # 32 heads
        if mode == "heads":
            mine = S.shard_heads(q, rank, world)
            out = torch.from_numpy(_oracle_out(mine, w))
            full = S.gather_heads(out, world)
        else:
            t0, n = S.token_range(rank, world, q.shape[0])
            sub = W.Workload(w.name, q[t0:t0 + n], w.kv, w.indices[t0:t0 + n], w.sm_scale)
            out = torch.from_numpy(_oracle_out(sub.q, sub))
            counts = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
            torch.distributed.all_gather(counts, torch.tensor([n]))
            pad = torch.zeros(max(int(c) for c in counts), *out.shape[1:])
            pad[:n] = out
            parts = [torch.empty_like(pad) for _ in range(world)]
            torch.distributed.all_gather(parts, pad)
            full = torch.cat([p[:int(c)] for p, c in zip(parts, counts)])
        if rank == 0:
            torch.save({"full": full, "ref": torch.from_numpy(_oracle_out(q, w))}, q_path)
    finally:
        torch.distributed.destroy_process_group()


@pytest.mark.parametrize("mode", ["heads", "tokens"])
def test_two_rank_shards_reassemble(tmp_path, mode):
    path = str(tmp_path / "res.pt")
    mp.start_processes(_worker, args=(2, _free_port(), mode, path), nprocs=2,
                       start_method="spawn", join=True)
    res = torch.load(path)
    assert res["full"].shape == res["ref"].shape
    assert torch.equal(res["full"], res["ref"]), mode


def test_ranges():
    assert [S.head_range(r, 4, 64) for r in range(4)] == [(0, 16), (16, 16), (32, 16), (48, 16)]
    assert S.head_range(0, 1, 64) == (0, 64)
    with pytest.raises(ValueError):
        S.head_range(0, 16, 64)          # 4 heads per rank: not served
    with pytest.raises(ValueError):
        S.head_range(2, 2, 64)
    spans = [S.token_range(r, 3, 10) for r in range(3)]
    assert spans == [(0, 4), (4, 3), (7, 3)]
    assert S.token_range(3, 4, 2) == (2, 0)


def test_peer_pointer_order():
    assert S.peer_pointer_order([4096, 8192], 1) == [4096, 8192]
    with pytest.raises(ValueError):
        S.peer_pointer_order([], 0)
    with pytest.raises(ValueError):
        S.peer_pointer_order([16] * 9, 0)
    with pytest.raises(ValueError):
        S.peer_pointer_order([4096, 8192], 2)
    with pytest.raises(ValueError):
        S.peer_pointer_order([4096, 8200], 0)          # not 16-byte aligned
