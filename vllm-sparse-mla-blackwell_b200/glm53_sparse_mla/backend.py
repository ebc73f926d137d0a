# SPDX-License-Identifier: Apache-2.0
"""vLLM attention backend for NoPE sparse MLA on B200 (sm_100).

Same classes, methods and behaviour as the reference plugin's backend
(glm53_sparse_mla/backend.py:98-449 of jsmcconn/vllm-sparse-mla-blackwell):

* head size = kv_lora_rank = 512 (qk_rope_head_dim == 0), so no rope block,
  no ``fp8_ds_mla`` packing and no fabricated zero pe;
* every token, prefill included, goes through the top-k sparse MQA path, which
  the builder expresses by reporting all tokens as decode tokens (the shared
  MLA layer then never enters its dense-MHA branch);
* bf16 or plain fp8_e4m3 KV with vLLM's per-tensor scale;
* ``AttentionCGSupport.UNIFORM_BATCH``: the op does no host sync, takes its
  split-merge workspace from the caching allocator on the current stream, and
  its launch geometry depends only on shapes.

What differs, because the kernel is built for sm_100a only:

* ``supports_compute_capability`` accepts major 10 (the reference: 12).
* ``register`` overrides the sparse-MLA slot vLLM lists for capability 10,
  ``FLASHINFER_MLA_SPARSE`` by default (the reference overrode
  ``FLASHINFER_MLA_SPARSE_SM120``, which vLLM only lists for 12.x); the
  ``VLLM_GLM53_BACKEND_SLOT`` environment variable names another slot.
* 64 heads per rank are supported (``SUPPORTED_HEADS_PER_RANK``).
* ``forward_mqa`` hands the indexer's request-local positions, the block table
  and ``req_id_per_token`` to the kernel (``sparse_fwd_paged``), which converts
  them to slots while compacting the index list; the reference ran vLLM's
  Triton converter and a narrowing copy first (its backend.py:341-348,
  371-378).
* With decode context parallelism (``dcp_world_size > 1``) ``forward_mqa``
  returns the natural-log LSE vLLM merges the ranks' outputs with; the
  reference returned None (its backend.py:395).
* ``do_kv_cache_update`` writes the latent cache with this package's sm_100a
  writer (``concat_and_cache_mla``); the reference inherited vLLM's, which
  calls vLLM's compiled op of that name.

Gate: ``VLLM_GLM53_CUDA_SPARSE_MLA=1``; unset, importing this module changes
nothing.
"""

from __future__ import annotations

import math
import os
from dataclasses import dataclass
from typing import TYPE_CHECKING, ClassVar

import numpy as np
import torch

from vllm.config import VllmConfig
from vllm.config.cache import CacheDType
from vllm.logger import init_logger
from vllm.v1.attention.backend import (
    AttentionBackend,
    AttentionCGSupport,
    AttentionLayer,
    AttentionMetadata,
    AttentionMetadataBuilder,
    CommonAttentionMetadata,
    MLAAttentionImpl,
)
from vllm.v1.kv_cache_interface import AttentionSpec

try:  # newer vLLM: row view that knows about interleaved layer pages
    from vllm.v1.attention.backends.mla.sparse_utils import flat_kv_row_view
except ImportError:
    flat_kv_row_view = None

import glm53_sparse_mla  # noqa: E402  registers torch.ops.glm53_sparse_mla.*

if TYPE_CHECKING:
    from vllm.model_executor.models.deepseek_v2 import Indexer
    from vllm.platforms.interface import DeviceCapability

logger = init_logger(__name__)

KV_LORA_RANK = glm53_sparse_mla.KV_LORA_RANK            # 512
SUPPORTED_HEADS_PER_RANK = glm53_sparse_mla.SUPPORTED_HEADS_PER_RANK
DEFAULT_SLOT = "FLASHINFER_MLA_SPARSE"


def _slot_name() -> str:
    return os.environ.get("VLLM_GLM53_BACKEND_SLOT", DEFAULT_SLOT)


class Glm53SparseMLABackend(AttentionBackend):
    supported_dtypes: ClassVar[list[torch.dtype]] = [torch.bfloat16]
    supported_kv_cache_dtypes: ClassVar[list[CacheDType]] = [
        "auto", "bfloat16", "fp8", "fp8_e4m3",
    ]

    @staticmethod
    def get_name() -> str:
        # The name of the slot this class was registered into, so the selector,
        # vLLM's kv-dtype handling and the logs agree.
        return _slot_name()

    @staticmethod
    def get_metadata_cls() -> type["Glm53SparseMLAMetadata"]:
        return Glm53SparseMLAMetadata

    @staticmethod
    def get_builder_cls() -> type["Glm53SparseMLAMetadataBuilder"]:
        return Glm53SparseMLAMetadataBuilder

    @staticmethod
    def get_impl_cls() -> type["Glm53SparseMLAImpl"]:
        return Glm53SparseMLAImpl

    @classmethod
    def is_mla(cls) -> bool:
        return True

    @classmethod
    def is_sparse(cls) -> bool:
        return True

    @staticmethod
    def get_kv_cache_shape(
        num_blocks: int,
        block_size: int,
        num_kv_heads: int,
        head_size: int,
        cache_dtype_str: str = "auto",
    ) -> tuple[int, ...]:
        # one latent head: [num_blocks, block_size, 512]
        return (num_blocks, block_size, head_size)

    @classmethod
    def get_supported_head_sizes(cls) -> list[int]:
        return [KV_LORA_RANK]

    @classmethod
    def supports_compute_capability(cls, capability: "DeviceCapability") -> bool:
        return capability.major == 10

    @classmethod
    def supports_combination(
        cls,
        head_size: int,
        dtype: torch.dtype,
        kv_cache_dtype: "CacheDType | None",
        block_size: int | None,
        use_mla: bool,
        has_sink: bool,
        use_sparse: bool,
        use_mm_prefix: bool,
        device_capability: "DeviceCapability",
    ) -> str | None:
        if not (use_mla and use_sparse):
            return "glm53 sparse MLA requires sparse MLA attention"
        if head_size != KV_LORA_RANK:
            return (f"glm53 sparse MLA is a NoPE kernel: head_size must be {KV_LORA_RANK} "
                    f"(qk_rope_head_dim == 0), got {head_size}")
        if has_sink:
            return "glm53 sparse MLA does not support attention sinks"
        return None


@dataclass
class Glm53SparseMLAMetadata(AttentionMetadata):
    num_reqs: int
    max_query_len: int
    max_seq_len: int

    num_actual_tokens: int
    query_start_loc: torch.Tensor
    slot_mapping: torch.Tensor

    block_table: torch.Tensor
    req_id_per_token: torch.Tensor

    block_size: int = 1
    topk_tokens: int = 2048

    # Read by the shared MLA layer to split MQA from dense-MHA tokens; with all
    # tokens counted as decode tokens the dense branch is never taken.
    num_decodes: int = 0
    num_prefills: int = 0
    num_decode_tokens: int = 0


@dataclass
class Glm53SparseMLAMetadataBuilder(AttentionMetadataBuilder[Glm53SparseMLAMetadata]):
    # Uniform query lengths (1, or 1 + speculative tokens) capture cleanly;
    # mixed prefill/decode batches vary the length and are run eagerly.
    _cudagraph_support: ClassVar[AttentionCGSupport] = AttentionCGSupport.UNIFORM_BATCH

    def __init__(
        self,
        kv_cache_spec: AttentionSpec,
        layer_names: list[str],
        vllm_config: VllmConfig,
        device: torch.device,
    ):
        self.kv_cache_spec = kv_cache_spec
        self.model_config = vllm_config.model_config
        self.device = device
        self.topk_tokens = vllm_config.model_config.hf_config.index_topk
        # persistent, so captured graphs keep reading the same storage
        self.req_id_per_token_buffer = torch.empty(
            (vllm_config.scheduler_config.max_num_batched_tokens,),
            dtype=torch.int32, device=device)

    def build(
        self,
        common_prefix_len: int,
        common_attn_metadata: CommonAttentionMetadata,
        fast_build: bool = False,
    ) -> Glm53SparseMLAMetadata:
        cm = common_attn_metadata
        n_tok = cm.num_actual_tokens
        starts = np.asarray(cm.query_start_loc_cpu, dtype=np.int64)
        per_req = np.diff(starts)
        req_ids = np.repeat(np.arange(per_req.size, dtype=np.int32), per_req)
        self.req_id_per_token_buffer.fill_(0)
        self.req_id_per_token_buffer[: req_ids.size].copy_(torch.from_numpy(req_ids),
                                                           non_blocking=True)
        return Glm53SparseMLAMetadata(
            num_reqs=cm.num_reqs,
            max_query_len=cm.max_query_len,
            max_seq_len=cm.max_seq_len,
            num_actual_tokens=n_tok,
            query_start_loc=cm.query_start_loc,
            slot_mapping=cm.slot_mapping,
            block_table=cm.block_table_tensor,
            req_id_per_token=self.req_id_per_token_buffer[:n_tok],
            block_size=self.kv_cache_spec.block_size,
            topk_tokens=self.topk_tokens,
            num_decodes=cm.num_reqs,
            num_prefills=0,
            num_decode_tokens=n_tok,
        )


class Glm53SparseMLAImpl(MLAAttentionImpl[Glm53SparseMLAMetadata]):
    is_sparse = True
    supports_dense_mha_prefill = False

    def __init__(
        self,
        num_heads: int,
        head_size: int,
        scale: float,
        num_kv_heads: int,
        alibi_slopes: list[float] | None,
        sliding_window: int | None,
        kv_cache_dtype: str,
        logits_soft_cap: float | None,
        attn_type: str,
        kv_sharing_target_layer_name: str | None,
        topk_indices_buffer: torch.Tensor | None = None,
        indexer: "Indexer | None" = None,
        **mla_args,
    ) -> None:
        if any([alibi_slopes, sliding_window, logits_soft_cap]):
            raise NotImplementedError(
                "glm53 sparse MLA does not support alibi_slopes / sliding_window / "
                "logits_soft_cap")
        self.num_heads = num_heads
        self.head_size = head_size
        self.scale = float(scale)
        self.num_kv_heads = num_kv_heads
        self.kv_cache_dtype = kv_cache_dtype
        self.kv_lora_rank: int = mla_args["kv_lora_rank"]
        self.softmax_scale = scale
        if num_heads not in SUPPORTED_HEADS_PER_RANK:
            raise NotImplementedError(
                f"glm53 sparse MLA supports {sorted(SUPPORTED_HEADS_PER_RANK)} heads per rank "
                f"(TP=8/4/2/1 on a 64-head model); got {num_heads}")
        # normal layers share the indexer's buffer; skip layers pass it directly
        self.topk_indices_buffer: torch.Tensor | None = (
            indexer.topk_indices_buffer if indexer is not None else topk_indices_buffer)

    def _kv_rows(self, kv_cache: torch.Tensor, attn_metadata: Glm53SparseMLAMetadata):
        """Flat [R, 512] view of the paged cache and the row distance between
        consecutive blocks (block_size for contiguous pages)."""
        head_dim = kv_cache.shape[-1]
        if flat_kv_row_view is not None:
            rows, stride_rows = flat_kv_row_view(kv_cache, attn_metadata.block_size)
            return rows, int(stride_rows)
        # Without flat_kv_row_view the pages must be contiguous for block *
        # block_size + offset to be a flat row.
        stride0 = kv_cache.stride(0)
        assert stride0 == attn_metadata.block_size * head_dim, (
            f"paged KV block stride {stride0} != block_size * head_dim "
            f"({attn_metadata.block_size} * {head_dim}); a flat row view of this "
            f"layout needs vLLM's flat_kv_row_view")
        return kv_cache.view(-1, head_dim), int(attn_metadata.block_size)

    @staticmethod
    def _kv_scale(layer, kv_rows: torch.Tensor) -> float:
        if kv_rows.dtype == torch.bfloat16:
            return 1.0
        s = getattr(layer, "_k_scale_float", None)
        if s is None:
            s = getattr(layer, "_k_scale", None)
        if s is None:
            return 1.0
        return float(s.item()) if torch.is_tensor(s) else float(s)

    def do_kv_cache_update(self, kv_c_normed: torch.Tensor, k_pe: torch.Tensor,
                           kv_cache: torch.Tensor, slot_mapping: torch.Tensor,
                           kv_cache_dtype: str, k_scale: torch.Tensor) -> None:
        """Write the step's new latent rows into the paged cache with this
        package's sm_100a writer: the same write, with the same arguments, as
        MLAAttentionImpl's default, which calls vLLM's concat_and_cache_mla
        (vllm 0.22.0 vllm/v1/attention/backend.py:990-1010); bf16 for
        ``auto``, plain e4m3(x / k_scale) for ``fp8`` / ``fp8_e4m3``."""
        if kv_cache.numel() == 0:
            return
        if k_pe.dim() == 3:
            k_pe = k_pe.squeeze(1)
        glm53_sparse_mla.concat_and_cache_mla(kv_c_normed, k_pe, kv_cache, slot_mapping.flatten(),
                                              kv_cache_dtype, k_scale)

    def forward_mha(self, q, kv_c_normed, k_pe, kv_c_and_k_pe_cache, attn_metadata, k_scale,
                    output) -> None:
        # The builder reports every token as a decode token, so the shared MLA
        # layer never takes its dense-MHA branch; vLLM versions that declare
        # this method abstract still need it defined.
        raise NotImplementedError("glm53 sparse MLA runs every token through forward_mqa")

    def forward_mqa(
        self,
        q: torch.Tensor | tuple[torch.Tensor, torch.Tensor],
        kv_c_and_k_pe_cache: torch.Tensor,
        attn_metadata: Glm53SparseMLAMetadata,
        layer: AttentionLayer,
    ) -> tuple[torch.Tensor, torch.Tensor | None]:
        if self.kv_cache_dtype == "fp8_ds_mla":
            raise NotImplementedError(
                "glm53 sparse MLA uses a plain 512-wide cache; fp8_ds_mla packs a 64-wide "
                "rope block this NoPE model does not have")
        if isinstance(q, tuple):  # pe half is empty for NoPE
            q = torch.cat(q, dim=-1)
        n_tok = q.shape[0]
        assert self.topk_indices_buffer is not None
        positions = self.topk_indices_buffer[:n_tok]
        # The indexer's request-local positions go to the kernel as they are:
        # it converts them to slots through the block table while compacting
        # them (the conversion vLLM's index converter would launch separately)
        # and reads only the first topk columns of each row at the buffer's
        # row stride, so the extra columns the indexer emits (topk rounded up
        # to 128) need no narrowing copy.
        topk = min(int(attn_metadata.topk_tokens), positions.shape[1])
        kv_rows, stride_rows = self._kv_rows(kv_c_and_k_pe_cache, attn_metadata)
        out = q.new_empty((n_tok, self.num_heads, self.kv_lora_rank))
        # Decode context parallelism merges the ranks' partial results by their
        # log-sum-exp, which vLLM takes in natural-log base.
        lse = None
        if getattr(self, "dcp_world_size", 1) > 1:
            lse = torch.empty((n_tok, self.num_heads), dtype=torch.float32, device=q.device)
        glm53_sparse_mla.sparse_fwd_paged(
            q, kv_rows, positions, attn_metadata.req_id_per_token, attn_metadata.block_table,
            attn_metadata.block_size, self.softmax_scale, self._kv_scale(layer, kv_rows),
            topk=topk, out=out, lse=lse, block_stride_rows=stride_rows)
        if lse is not None:
            lse.mul_(math.log(2.0))   # the kernel returns log2
        return out, lse


def _allow_plain_fp8_kv() -> None:
    """Keep ``--kv-cache-dtype fp8`` as a plain 512-wide fp8 cache.

    vLLM snapshots that rewrite fp8 into the packed ``fp8_ds_mla`` record by
    backend name (``_canonicalize_sparse_mla_kv_cache_dtype``) are patched to
    leave this backend's dtype alone; the packed record's writer asserts a
    64-wide rope block that a NoPE model does not have. vLLM versions without
    that hook (0.22 rewrites only for FLASHMLA_SPARSE) need nothing.
    """
    from vllm.model_executor.layers.attention import mla_attention as mla

    original = getattr(mla, "_canonicalize_sparse_mla_kv_cache_dtype", None)
    if original is None or getattr(mla, "_glm53_kv_canon_patched", False):
        return

    def patched(attn_backend, kv_cache_dtype):
        if attn_backend.get_impl_cls() is Glm53SparseMLAImpl:
            return kv_cache_dtype
        return original(attn_backend, kv_cache_dtype)

    mla._canonicalize_sparse_mla_kv_cache_dtype = patched
    mla._glm53_kv_canon_patched = True
    logger.info("glm53: plain fp8 KV allowed (no fp8_ds_mla rewrite)")


def register() -> bool:
    """vllm.general_plugins entry point; a no-op unless the env gate is set."""
    if os.environ.get("VLLM_GLM53_CUDA_SPARSE_MLA", "") not in ("1", "true", "TRUE"):
        return False
    from vllm.v1.attention.backends.registry import AttentionBackendEnum, register_backend

    slot = _slot_name()
    if not hasattr(AttentionBackendEnum, slot):
        raise ValueError(f"glm53_sparse_mla: this vLLM has no attention backend slot {slot!r}")
    register_backend(getattr(AttentionBackendEnum, slot),
                     "glm53_sparse_mla.backend.Glm53SparseMLABackend")
    _allow_plain_fp8_kv()
    logger.info("glm53_sparse_mla: overrode %s with the NoPE sm_100a sparse-MLA backend "
                "(head_size=%d, bf16/fp8 KV)", slot, KV_LORA_RANK)
    return True
