"""Sparse MLA (NoPE) attention for B200 (sm_100a).

Exposes ``torch.ops.glm53_sparse_mla.sparse_fwd`` with the schema of the
reference extension, so the vLLM backend in :mod:`glm53_sparse_mla.backend`
and any other caller bind unchanged, plus ``sparse_fwd_lse`` which also returns
the log2-space log-sum-exp. The op is a thin binding over the C ABI declared in
``include/glm53_sparse_mla.h`` (``libglm53_sparse_mla.so``); the kernel is a
hand-written tcgen05/TMEM kernel for sm_100a. There is no CPU or fallback path:
without the compiled extension the import fails.

Mirrors the reference facade (glm53_sparse_mla/__init__.py:14-85): same
constants, same ``sparse_fwd`` signature and return value, same fake kernel
for ``torch.compile``.
"""

from __future__ import annotations

import os

import torch

__all__ = [
    "sparse_fwd",
    "sparse_fwd_with_lse",
    "sparse_fwd_paged",
    "concat_and_cache_mla",
    "top_k_per_row_decode",
    "top_k_per_row_prefill",
    "fp8_paged_mqa_logits",
    "fp8_fp4_paged_mqa_logits",
    "HEADS_PER_RANK",
    "SUPPORTED_HEADS_PER_RANK",
    "KV_LORA_RANK",
    "library_path",
]

# A 64-head model fits on one B200: TP=1 is the default deployment.
HEADS_PER_RANK = 64
# 8 / 16 / 32 / 64 heads per rank, i.e. TP=8 / 4 / 2 / 1 on a 64-head model.
SUPPORTED_HEADS_PER_RANK = (8, 16, 32, 64)
KV_LORA_RANK = 512  # head_size, since qk_rope_head_dim == 0 (NoPE)

_HERE = os.path.dirname(os.path.abspath(__file__))


def library_path() -> str:
    """Path of the C-ABI shared library (libglm53_sparse_mla.so)."""
    return os.path.join(_HERE, "libglm53_sparse_mla.so")


def _load() -> None:
    """Register the CUDA ops.

    The op library is TORCH_LIBRARY-only (no PyInit), so it is loaded with
    ``torch.ops.load_library``. When it is missing but the sources are present
    (a development checkout) it is built in place first; a deployed package
    without its compiled extension raises ImportError instead.
    """
    if hasattr(torch.ops, "glm53_sparse_mla") and hasattr(
        torch.ops.glm53_sparse_mla, "sparse_fwd"
    ):
        return
    op_lib = os.path.join(_HERE, "_C.so")
    if not (os.path.exists(op_lib) and os.path.exists(library_path())):
        if not os.path.exists(os.path.join(os.path.dirname(_HERE), "csrc")):
            raise ImportError(
                "glm53_sparse_mla: no compiled _C.so / libglm53_sparse_mla.so next to "
                "the package and no csrc/ to build from. The build did not ship its "
                "extension."
            )
        from .build import build

        build()
    torch.ops.load_library(op_lib)


_load()


def sparse_fwd(q, kv, indices, sm_scale, kv_scale=1.0, out=None):
    """Gathered sparse MLA over the top-k indices.

    q       [T, H, 512]  bfloat16, H in SUPPORTED_HEADS_PER_RANK
    kv      [R, 512]     bfloat16 or float8_e4m3fn; a flat row view of the paged
                         cache serving as both K and V (absorbed MLA). kv_scale
                         is vLLM's per-tensor cache scale (ignored for bf16).
    indices [T, topk]    int32 physical row ids, -1 is the mask sentinel
    returns [T, H, 512]  bfloat16 (``out`` if given, written in place)

    Causality is not applied here; the indexer owns it. A token whose indices
    are all masked returns exactly zero (never NaN).
    """
    if out is None:
        out = torch.empty_like(q)
    torch.ops.glm53_sparse_mla.sparse_fwd(q, kv, indices, float(sm_scale), float(kv_scale), out)
    return out


def sparse_fwd_with_lse(q, kv, indices, sm_scale, kv_scale=1.0, out=None, lse=None):
    """As :func:`sparse_fwd`, also returning ``lse [T, H]`` float32.

    ``lse = log2(sum_i exp(sm_scale * q . kv_i))`` over the valid indices, i.e.
    the natural-log LSE times log2(e); -inf for a fully masked (token, head).
    """
    if out is None:
        out = torch.empty_like(q)
    if lse is None:
        lse = torch.empty(q.shape[0], q.shape[1], dtype=torch.float32, device=q.device)
    torch.ops.glm53_sparse_mla.sparse_fwd_lse(
        q, kv, indices, float(sm_scale), float(kv_scale), out, lse
    )
    return out, lse


def sparse_fwd_paged(q, kv, topk_positions, req_id_per_token, block_table, block_size,
                     sm_scale, kv_scale=1.0, topk=None, out=None, lse=None,
                     block_stride_rows=0):
    """Sparse MLA on vLLM's request-local top-k positions.

    topk_positions [T, >= topk] int32   token positions within each request
                                        (-1 masked); only the first ``topk``
                                        columns are read (default: all)
    req_id_per_token [T] int32          request of each query token
    block_table [requests, max_blocks]  int32 physical block ids
    block_size                          tokens per cache block

    The kernel maps position p of request r to the slot
    ``block_table[r, p // block_size] * block_stride_rows + p % block_size``
    (``block_stride_rows`` = ``block_size`` for contiguous pages, the default)
    while it compacts the index list, as vLLM's index converter would, so
    neither that converter nor a narrowing copy of the positions is needed.
    Returns ``out`` (and fills ``lse`` [T, H] float32, log2 base, if given).
    """
    if out is None:
        out = torch.empty_like(q)
    k = int(topk) if topk is not None else int(topk_positions.shape[1])
    torch.ops.glm53_sparse_mla.sparse_fwd_paged(
        q, kv, topk_positions, req_id_per_token, block_table, int(block_size), k,
        float(sm_scale), float(kv_scale), out, lse, int(block_stride_rows))
    return out


def concat_and_cache_mla(kv_c, k_pe, kv_cache, slot_mapping, kv_cache_dtype, scale):
    """Write new tokens' latent rows into the paged cache the op reads.

    kv_c [N, 512] bf16 (rows may be strided), k_pe [N, 0] (NoPE), kv_cache
    [num_blocks, block_size, 512] (bf16 for ``"auto"``; uint8 or
    float8_e4m3fn for ``"fp8"`` / ``"fp8_e4m3"``), slot_mapping [T] int64
    (T <= N; slot < 0 = padded token, skipped), scale: float32 CUDA tensor,
    the per-tensor fp8 scale (element = e4m3(x / scale), saturating).

    Same argument list and meaning as vLLM's ``ops.concat_and_cache_mla``
    (vllm 0.22.0 vllm/_custom_ops.py:2613-2623), which the reference leaves
    vLLM to call; here it runs this package's sm_100a kernel.
    """
    torch.ops.glm53_sparse_mla.concat_and_cache_mla(kv_c, k_pe, kv_cache, slot_mapping,
                                                    str(kv_cache_dtype), scale)


def top_k_per_row_decode(logits, next_n, seq_lens, raw_topk_indices, num_rows, stride0, stride1,
                         topk_tokens):
    """Top-k positions of each decode row of the indexer's logits.

    Row r covers ``logits[r, :end)`` with ``end = seq_lens[r // next_n] -
    next_n + r % next_n + 1`` (1-D seq_lens) or ``seq_lens.flatten()[r]``
    (2-D [B, next_n]); ``raw_topk_indices[r, :topk_tokens]`` receives
    0..end-1 then -1 when end <= topk_tokens, else the positions of the
    topk_tokens largest logits in no particular order. Same arguments as
    vLLM's ``ops.top_k_per_row_decode`` (vllm 0.22.0
    vllm/_custom_ops.py:2821-2840).
    """
    torch.ops.glm53_sparse_mla.top_k_per_row_decode(
        logits, int(next_n), seq_lens, raw_topk_indices, int(num_rows), int(stride0),
        int(stride1), int(topk_tokens))


def top_k_per_row_prefill(logits, cu_seqlen_ks, cu_seqlen_ke, raw_topk_indices, num_rows,
                          stride0, stride1, topk_tokens):
    """Top-k positions of each prefill row: row r covers
    ``logits[r, cu_seqlen_ks[r]:cu_seqlen_ke[r])`` and its positions are
    written relative to cu_seqlen_ks[r]. Same arguments as vLLM's
    ``ops.top_k_per_row_prefill`` (vllm 0.22.0 vllm/_custom_ops.py:2799-2818).
    """
    torch.ops.glm53_sparse_mla.top_k_per_row_prefill(
        logits, cu_seqlen_ks, cu_seqlen_ke, raw_topk_indices, int(num_rows), int(stride0),
        int(stride1), int(topk_tokens))


def fp8_paged_mqa_logits(q, kv_cache, weights, context_lens, block_tables, max_model_len,
                         clean_logits=True, logits=None):
    """The sparse-attention indexer's scores over its paged fp8 cache.

    q [B, next_n, H, 128] fp8_e4m3 (H 32 or 64, next_n 1, 2 or 4); kv_cache
    [num_blocks, block_size, (1,) 132] uint8 (each block: block_size rows of
    128 e4m3 values, then block_size fp32 scales); weights [B * next_n, H]
    fp32; context_lens [B] (token j of request i sees positions
    < context_lens[i] - next_n + j + 1) or [B, next_n] (per token);
    block_tables [B, max_blocks] int32. Returns logits [B * next_n,
    max_model_len] fp32: scale[p] * sum_h relu(q[h] . k[p]) * w[h] on visible
    positions, -inf elsewhere with ``clean_logits`` (untouched without it).
    """
    if logits is None:
        logits = torch.empty((q.shape[0] * q.shape[1], int(max_model_len)), dtype=torch.float32,
                             device=q.device)
    torch.ops.glm53_sparse_mla.fp8_paged_mqa_logits(q, kv_cache, weights, context_lens,
                                                    block_tables, int(max_model_len),
                                                    bool(clean_logits), logits)
    return logits


def fp8_fp4_paged_mqa_logits(q, kv_cache, weights, context_lens, block_tables,
                             schedule_metadata, max_model_len, clean_logits):
    """Drop-in for vLLM's ``vllm.utils.deep_gemm.fp8_fp4_paged_mqa_logits``
    (vllm 0.22.0 vllm/utils/deep_gemm.py:407-456) on the fp8 path: ``q`` is
    the ``(values, None)`` pair; ``schedule_metadata`` (DeepGEMM's SM
    schedule) is not needed and ignored."""
    values, q_scale = q if isinstance(q, tuple) else (q, None)
    if q_scale is not None:
        raise NotImplementedError("glm53_sparse_mla: the MXFP4 indexer cache is not supported")
    return fp8_paged_mqa_logits(values, kv_cache, weights, context_lens, block_tables,
                                max_model_len, clean_logits)


# Shape-only meta kernels so torch.compile can trace through the ops.
@torch.library.register_fake("glm53_sparse_mla::sparse_fwd")
def _sparse_fwd_fake(q, kv, indices, sm_scale, kv_scale, out):
    torch._check(q.dim() == 3 and kv.dim() == 2 and indices.dim() == 2)
    torch._check(out.shape == q.shape)
    return None


@torch.library.register_fake("glm53_sparse_mla::sparse_fwd_lse")
def _sparse_fwd_lse_fake(q, kv, indices, sm_scale, kv_scale, out, lse):
    torch._check(q.dim() == 3 and kv.dim() == 2 and indices.dim() == 2)
    torch._check(out.shape == q.shape)
    torch._check(lse.dim() == 2 and lse.shape[0] == q.shape[0] and lse.shape[1] == q.shape[1])
    return None


@torch.library.register_fake("glm53_sparse_mla::sparse_fwd_paged")
def _sparse_fwd_paged_fake(q, kv, topk_positions, req_id_per_token, block_table, block_size,
                           topk, sm_scale, kv_scale, out, lse=None, block_stride_rows=0):
    torch._check(q.dim() == 3 and kv.dim() == 2 and topk_positions.dim() == 2)
    torch._check(out.shape == q.shape)
    return None


@torch.library.register_fake("glm53_sparse_mla::concat_and_cache_mla")
def _concat_and_cache_mla_fake(kv_c, k_pe, kv_cache, slot_mapping, kv_cache_dtype, scale):
    torch._check(kv_c.dim() == 2 and kv_cache.dim() == 3 and slot_mapping.dim() == 1)
    return None


@torch.library.register_fake("glm53_sparse_mla::top_k_per_row_decode")
def _top_k_per_row_decode_fake(logits, next_n, seq_lens, raw_topk_indices, num_rows, stride0,
                               stride1, topk_tokens):
    torch._check(raw_topk_indices.dim() == 2)
    return None


@torch.library.register_fake("glm53_sparse_mla::top_k_per_row_prefill")
def _top_k_per_row_prefill_fake(logits, cu_seqlen_ks, cu_seqlen_ke, raw_topk_indices, num_rows,
                                stride0, stride1, topk_tokens):
    torch._check(raw_topk_indices.dim() == 2)
    return None


@torch.library.register_fake("glm53_sparse_mla::fp8_paged_mqa_logits")
def _fp8_paged_mqa_logits_fake(q, kv_cache, weights, context_lens, block_tables, max_model_len,
                               clean_logits, logits):
    torch._check(q.dim() == 4 and logits.dim() == 2)
    return None


@torch.library.register_fake("glm53_sparse_mla::sparse_fwd_gather_heads")
def _sparse_fwd_gather_heads_fake(q, kv, indices, sm_scale, kv_scale, out_ptrs, rank, head_offset,
                                  out):
    torch._check(q.dim() == 3 and kv.dim() == 2 and indices.dim() == 2 and out.dim() == 3)
    torch._check(out.shape[0] == q.shape[0] and out.shape[2] == q.shape[2])
    return None
