"""CPU oracle for the sparse-attention indexer's paged fp8 MQA logits --
TEST INFRASTRUCTURE ONLY.

Only tests/ and bench.py's CPU legs may import this module, and only as the
checker (or as the timed CPU reference in bench.py). The product path never
calls it.

The reference's backend reads the top-k positions vLLM's indexer leaves in
``topk_indices_buffer`` (glm53_sparse_mla/backend.py:310-314 of jsmcconn/vllm-
sparse-mla-blackwell). On the decode path the indexer scores every cached
token with ``fp8_fp4_paged_mqa_logits`` (vllm 0.22.0
vllm/model_executor/layers/sparse_attn_indexer.py:324-333, DeepGEMM's kernel,
vllm/utils/deep_gemm.py:407-456) and then takes the per-row top-k. vLLM's own
torch restatement of the scorer is ``fp8_paged_mqa_logits_torch``
(vllm/v1/attention/ops/rocm_aiter_mla_sparse.py:256-356). vLLM and DeepGEMM
are dependencies of the reference, not part of it. The rule restated here:

  * the indexer cache is paged, block b holding block_size fp8_e4m3 rows of
    D = 128 values followed by block_size fp32 scales (the layout vLLM's
    indexer cache writer produces: rocm_aiter_mla_sparse.py:112-118);
  * query token j of request i (next_n tokens per request, rows
    i * next_n + j) sees cache positions p < context_lens[i] - next_n + j + 1;
  * logit = scale[p] * sum_h relu(q[i, j, h, :] . k[p, :]) * weights[row, h],
    with q and k as their exact e4m3 values;
  * positions a row does not see are -inf (the ``clean_logits`` form).

Parity pin: tests/test_indexer_logits_cpu.py checks this module against
vLLM's torch restatement (its next_n == 1 form; with next_n > 1 that code
reads the cache bytes per token instead of per block, which contradicts the
block layout above, so rows of a next_n > 1 request are pinned as next_n == 1
rows with the per-token context length).
"""

from __future__ import annotations

import numpy as np

from .sparse_mla_oracle import e4m3_to_f32

D = 128


def row_lengths(context_lens, next_n: int) -> np.ndarray:
    """Visible positions of each row (request i, token j)."""
    c = np.asarray(context_lens, dtype=np.int64).reshape(-1)
    j = np.arange(next_n)
    return (c[:, None] - next_n + j[None, :] + 1).reshape(-1)


def paged_mqa_logits(q_bits: np.ndarray, kv_blocks: np.ndarray, weights: np.ndarray,
                     context_lens, block_table, max_model_len: int) -> np.ndarray:
    """q_bits [B, next_n, H, 128] uint8 (e4m3); kv_blocks [num_blocks,
    block_size * 132] uint8; weights [B * next_n, H] fp32. Returns
    [B * next_n, max_model_len] fp32 logits, -inf where not visible."""
    B, next_n, H, d = q_bits.shape
    assert d == D
    nb, block_bytes = kv_blocks.shape
    bs = block_bytes // (D + 4)
    assert bs * (D + 4) == block_bytes
    q = e4m3_to_f32(q_bits).astype(np.float32)
    w = np.asarray(weights, dtype=np.float32)
    lens = row_lengths(context_lens, next_n)
    bt = np.asarray(block_table, dtype=np.int64)
    out = np.full((B * next_n, max_model_len), -np.inf, np.float32)
    for i in range(B):
        L = int(lens[i * next_n:(i + 1) * next_n].max())
        if L <= 0:
            continue
        pages = (L + bs - 1) // bs
        blk = kv_blocks[bt[i, :pages]]                              # only this request's blocks
        k = e4m3_to_f32(blk[:, :bs * D]).reshape(pages * bs, D)[:L]
        sc = np.ascontiguousarray(blk[:, bs * D:]).view(np.float32).reshape(pages * bs)[:L]
        for j in range(next_n):
            r = i * next_n + j
            Lj = int(lens[r])
            if Lj <= 0:
                continue
            s = np.maximum(k[:Lj] @ q[i, j].T, np.float32(0.0))     # [Lj, H]
            out[r, :Lj] = (s @ w[r]) * sc[:Lj]
    return out
