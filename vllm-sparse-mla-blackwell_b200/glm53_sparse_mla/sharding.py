"""Multi-GPU layouts for the sparse-MLA op: one process per GPU, no collective
on the attention data path.

Two ways to spread a batch over ``world`` ranks:

* **head sharding** (vLLM tensor parallelism): rank r serves heads
  ``[r * H / world, (r + 1) * H / world)`` of every token, with the index
  list and the latent KV pool replicated (the pool is one shared latent head,
  as vLLM TP replicates the MLA cache). Heads are independent, so a shard's
  output is exactly the matching slice of the full result;
  :func:`gather_heads` reassembles ``[T, H, 512]`` with one all-gather, and
  :class:`HeadShardGather` does without it: the kernel stores each rank's
  heads straight into every rank's full output (symmetric memory over
  NVLink), so the exchange overlaps the attention itself.
* **token sharding** (data-parallel attention): rank r serves a contiguous
  range of query tokens with all heads.

Attention itself needs no collective; the only exchange is the optional
output gather (NCCL all-gather, gloo in the CPU tests, or the fused peer
stores of :class:`HeadShardGather`).
"""

from __future__ import annotations

import os

import torch

from . import SUPPORTED_HEADS_PER_RANK

__all__ = ["head_range", "token_range", "shard_heads", "gather_heads", "HeadShardGather",
           "peer_pointer_order"]


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


def peer_pointer_order(buffer_ptrs, rank: int) -> list[int]:
    """Output pointers for the fused gather, in rank order (rank i's buffer
    at index i, this rank's own at index ``rank``): at most 8 ranks."""
    ptrs = [int(x) for x in buffer_ptrs]
    if not 1 <= len(ptrs) <= 8:
        raise ValueError(f"the fused head gather spans 1 to 8 ranks, got {len(ptrs)}")
    if not 0 <= rank < len(ptrs):
        raise ValueError(f"rank {rank} outside {len(ptrs)} buffers")
    if any(p == 0 or p % 16 for p in ptrs):
        raise ValueError("every output buffer must be a non-null 16-byte aligned device pointer")
    return ptrs


class HeadShardGather:
    """Head-sharded attention with the output gather fused into the kernel.

    Every rank holds a ``[tokens, heads_total, 512]`` bf16 buffer in symmetric
    memory (``torch.distributed._symmetric_memory``), mapped into every other
    rank's address space. A call runs this rank's heads through
    ``torch.ops.glm53_sparse_mla.sparse_fwd_gather_heads``: the epilogue of the
    attention kernel stores each output element into all ranks' buffers at
    this rank's head offset (plain peer stores over NVLink, no multicast), so
    the exchange overlaps the kernel's remaining work and no all-gather or
    reorder copy follows. A symmetric-memory barrier on the same stream then
    orders every rank's stores before anyone reads; the call returns this
    rank's gathered buffer. The buffer is reused by the next call.

    ``mode="copy"`` exchanges the outputs with the copy engines instead: the
    batch runs as one attention launch per wave of ``chunk_tokens`` tokens
    (default: the SM count) into this rank's own buffer, and after each launch
    a side stream pushes that chunk's head slice into every peer's buffer
    (``glm53_copy_head_slices``: 2-D copies that read only local memory), so
    a wave's exchange overlaps the next wave's compute and no SM stalls on
    NVLink stores.

    Collective: every rank of ``group`` constructs it and calls it in the
    same order.
    """

    def __init__(self, tokens: int, heads_total: int, group=None, device=None,
                 mode: str = "fused", chunk_tokens: int | None = None):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem

        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        self.head_offset, self.heads = head_range(self.rank, self.world, heads_total)
        self.tokens, self.heads_total = tokens, heads_total
        device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        # plain peer stores are all the gather uses; keep the buffer off any
        # NVLink multicast object
        os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
        self.buf = symm_mem.empty(tokens, heads_total, 512, dtype=torch.bfloat16, device=device)
        self.handle = symm_mem.rendezvous(self.buf, self.group.group_name)
        self.ptrs = peer_pointer_order(self.handle.buffer_ptrs, self.rank)
        if mode not in ("fused", "copy"):
            raise ValueError(f"mode must be 'fused' or 'copy', got {mode!r}")
        self.mode = mode
        if mode == "copy":
            import ctypes

            from . import library_path
            self._lib = ctypes.CDLL(library_path())
            self._lib.glm53_copy_head_slices.restype = ctypes.c_int
            self._lib.glm53_copy_head_slices.argtypes = [
                ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p]
            self._copy_stream = torch.cuda.Stream(device)
            sms = torch.cuda.get_device_properties(device).multi_processor_count
            self.chunk = int(chunk_tokens or sms)
            self._row_bytes = heads_total * 512 * 2

    def __call__(self, q_shard: torch.Tensor, kv: torch.Tensor, indices: torch.Tensor,
                 sm_scale: float, kv_scale: float = 1.0, barrier: bool = True) -> torch.Tensor:
        if q_shard.shape[0] != self.tokens or q_shard.shape[1] != self.heads:
            raise ValueError(f"q shard must be [{self.tokens}, {self.heads}, 512], got "
                             f"{tuple(q_shard.shape)}")
        if self.mode == "fused":
            torch.ops.glm53_sparse_mla.sparse_fwd_gather_heads(
                q_shard, kv, indices, float(sm_scale), float(kv_scale), self.ptrs, self.rank,
                self.head_offset, self.buf)
        else:
            self._chunked(q_shard, kv, indices, float(sm_scale), float(kv_scale))
        if barrier:
            self.handle.barrier(channel=0, timeout_ms=10000)
        return self.buf

    def _chunked(self, q_shard, kv, indices, sm_scale, kv_scale):
        import ctypes

        main = torch.cuda.current_stream()
        side = self._copy_stream
        side.wait_stream(main)              # earlier readers of the buffers are done
        dsts = (ctypes.c_void_p * len(self.ptrs))()
        for t0 in range(0, self.tokens, self.chunk):
            t1 = min(self.tokens, t0 + self.chunk)
            out = self.buf[t0:t1]
            torch.ops.glm53_sparse_mla.sparse_fwd_gather_heads(
                q_shard[t0:t1], kv, indices[t0:t1], sm_scale, kv_scale, [out.data_ptr()], 0,
                self.head_offset, out)
            ev = torch.cuda.Event()
            ev.record(main)
            side.wait_event(ev)
            for i, ptr in enumerate(self.ptrs):
                dsts[i] = ptr + t0 * self._row_bytes
            rc = self._lib.glm53_copy_head_slices(
                dsts, len(self.ptrs), out.data_ptr(), t1 - t0, self.heads_total,
                self.head_offset, self.heads, side.cuda_stream)
            if rc != 0:
                raise RuntimeError(f"glm53_copy_head_slices failed with status {rc}")
        main.wait_stream(side)
