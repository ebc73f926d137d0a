"""CPU oracle for the indexer's per-row top-k -- TEST INFRASTRUCTURE ONLY.

Only tests/ and bench.py's CPU legs may import this module, and only as the
checker (or as the timed CPU reference in bench.py). The product path never
calls it.

The reference's backend reads the request-local top-k positions vLLM's
sparse-attention indexer leaves in ``topk_indices_buffer``
(glm53_sparse_mla/backend.py:310-314 of jsmcconn/vllm-sparse-mla-blackwell).
The last step of that producer is vLLM 0.22.0's top_k_per_row_decode /
top_k_per_row_prefill (vllm/_custom_ops.py:2799-2840, called at
vllm/model_executor/layers/sparse_attn_indexer.py:247-256, 351-360); vLLM's
own torch restatement of it is ``_topk_indices_torch``
(vllm/v1/attention/ops/rocm_aiter_mla_sparse.py:572-600). vLLM is a
dependency of the reference, not part of it. The rule restated here:

  * row r covers logits[r, start:end): decode start = 0, end =
    seq_lens[r // next_n] - next_n + r % next_n + 1; prefill start/end given;
  * len = end - start <= k: positions 0..len-1, then -1 up to k;
  * otherwise the positions (relative to start) of the k largest values; the
    order of the output and which of several values equal to the k-th largest
    are taken are unspecified, so ``topk_row`` returns one canonical choice
    (value descending, position ascending) and ``check_row`` accepts any
    selection whose values form the same multiset;
  * values compare by IEEE order with +NaN above +inf (the order of the
    32-bit key below).

Parity pin: tests/test_topk_cpu.py checks this module against vLLM's
``_topk_indices_torch``; tests/test_topk_gpu.py checks the kernel against
this module and against vLLM's compiled ops.
"""

from __future__ import annotations

import numpy as np


def order_key(x: np.ndarray) -> np.ndarray:
    """fp32 -> uint32 whose unsigned order is IEEE order (+NaN on top)."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    neg = (b & np.uint32(0x80000000)) != 0
    return np.where(neg, ~b, b | np.uint32(0x80000000)).astype(np.uint32)


def decode_row_ends(seq_lens, next_n: int, num_rows: int) -> np.ndarray:
    """Row ends of the decode form: 1-D seq_lens by the next_n rule, 2-D
    [B, next_n] seq_lens as per-row lengths."""
    s = np.asarray(seq_lens, dtype=np.int64)
    if s.ndim == 2 and s.shape[1] > 1:
        return s.reshape(-1)[:num_rows]
    s = s.reshape(-1)
    r = np.arange(num_rows)
    return s[r // next_n] - next_n + r % next_n + 1


def topk_row(row: np.ndarray, start: int, end: int, k: int) -> np.ndarray:
    length = max(0, int(end) - int(start))
    out = np.full(k, -1, np.int32)
    if length <= k:
        out[:length] = np.arange(length, dtype=np.int32)
        return out
    keys = order_key(row[start:end]).astype(np.int64)
    order = np.lexsort((np.arange(length), -keys))       # value desc, position asc
    out[:] = order[:k].astype(np.int32)
    return out


def topk_rows(logits: np.ndarray, starts, ends, k: int) -> np.ndarray:
    logits = np.asarray(logits, dtype=np.float32)
    return np.stack([topk_row(logits[r], starts[r], ends[r], k) for r in range(len(ends))]) \
        if len(ends) else np.zeros((0, k), np.int32)


def check_row(got: np.ndarray, row: np.ndarray, start: int, end: int, k: int) -> str | None:
    """None when ``got`` (k ints) is a valid top-k of row[start:end], else why not."""
    length = max(0, int(end) - int(start))
    got = np.asarray(got, dtype=np.int64)
    if length <= k:
        want = np.full(k, -1, np.int64)
        want[:length] = np.arange(length)
        return None if np.array_equal(got, want) else "short row: expected 0..len-1 then -1"
    if got.min() < 0 or got.max() >= length:
        return "position out of range"
    if np.unique(got).size != k:
        return "repeated position"
    keys = order_key(row[start:end])
    want = np.sort(keys[topk_row(row, start, end, k)])
    if not np.array_equal(np.sort(keys[got]), want):
        return "selected values differ from the k largest"
    return None
