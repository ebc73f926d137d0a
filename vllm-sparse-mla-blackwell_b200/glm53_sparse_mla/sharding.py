"""Multi-GPU layouts for the sparse-MLA op: one process per GPU, no collective
on the attention data path.

Two ways to spread a batch over ``world`` ranks:

* **head sharding** (vLLM tensor parallelism): rank r serves heads
  ``[r * H / world, (r + 1) * H / world)`` of every token, with the index
  list and the latent KV pool replicated (the pool is one shared latent head,
  as vLLM TP replicates the MLA cache). Heads are independent, so a shard's
  output is exactly the matching slice of the full result;
  :func:`gather_heads` reassembles ``[T, H, 512]`` with one all-gather.
* **token sharding** (data-parallel attention): rank r serves a contiguous
  range of query tokens with all heads.

The attention kernel never communicates; the only collective is the optional
output all-gather (NCCL on GPUs, gloo in the CPU tests).
"""

from __future__ import annotations

import torch

from . import SUPPORTED_HEADS_PER_RANK

__all__ = ["head_range", "token_range", "shard_heads", "gather_heads"]


def head_range(rank: int, world: int, heads_total: int) -> tuple[int, int]:
    """(first head, head count) of ``rank``; the count must be one the kernel
    serves (8, 16, 32 or 64 heads per rank)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    if heads_total % world:
        raise ValueError(f"{heads_total} heads do not split evenly over {world} ranks")
    per = heads_total // world
    if per not in SUPPORTED_HEADS_PER_RANK:
        raise ValueError(f"{per} heads per rank; supported: {SUPPORTED_HEADS_PER_RANK}")
    return rank * per, per


def token_range(rank: int, world: int, tokens: int) -> tuple[int, int]:
    """(first token, token count) of ``rank``: contiguous, sizes differ by at
    most one, trailing ranks may be empty."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    base, extra = divmod(tokens, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def shard_heads(q: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """This rank's contiguous ``[T, H / world, 512]`` slice of ``q``."""
    h0, n = head_range(rank, world, q.shape[1])
    return q[:, h0:h0 + n].contiguous()


def gather_heads(out_shard: torch.Tensor, world: int, group=None,
                 staging: torch.Tensor | None = None) -> torch.Tensor:
    """All-gather per-rank ``[T, h, 512]`` outputs into ``[T, world * h, 512]``
    (rank order = head order). ``staging`` (``[world, T, h, 512]``) may be
    passed to keep the collective allocation-free under CUDA-graph capture."""
    if world == 1:
        return out_shard
    T, h, d = out_shard.shape
    if staging is None:
        staging = torch.empty(world, T, h, d, dtype=out_shard.dtype, device=out_shard.device)
    if torch.distributed.get_backend(group) == "gloo":
        torch.distributed.all_gather(list(staging.unbind(0)), out_shard.contiguous(), group=group)
    else:
        torch.distributed.all_gather_into_tensor(staging, out_shard.contiguous(), group=group)
    return staging.permute(1, 0, 2, 3).reshape(T, world * h, d)
