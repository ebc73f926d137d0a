"""CPU oracle for the sparse-MLA path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
import this module, and only as the checker (or, in bench.py, as the timed
reference CPU implementation). The product path never calls it.

This is a numpy fp32 restatement of the reference's ground truth,
tests/reference.py:21-74 of jsmcconn/vllm-sparse-mla-blackwell:

  * clamp, then gather: index < 0 reads row 0 but is masked   (reference.py:47-49)
  * scores s = (q . kv_row) * sm_scale, then mask to -inf        (reference.py:52-53)
  * a fully masked row gets a finite shift of 0                  (reference.py:55-57)
  * p = exp(s - m) on valid rows, 0 elsewhere; sumexp = sum(p)   (reference.py:58-61)
  * out = (p @ rows) / sumexp, exactly 0 where sumexp == 0       (reference.py:62-69)
  * lse as the reference file writes it                          (reference.py:71-73)

Parity pin: tests/test_oracle_golden.py checks this module against vectors
produced by the reference's own sparse_mla_fp32 (tests/golden/make_golden.py).

LSE note. The reference file computes ``log2(sumexp) + m * sm_scale * log2e``
with ``m`` the max of the *already scaled* scores, so its LSE applies sm_scale
to the max term twice; it equals the log2 log-sum-exp only when sm_scale == 1.
``lse_reference`` reproduces that formula bit-for-bit (for pinning);
``lse_log2`` is the quantity the kernel returns, log2(sum_i exp(s_i)) =
log2(sumexp) + m * log2e, -inf for a fully masked row.
"""

from __future__ import annotations

import numpy as np

LOG2E_REF = 1.44269504          # constant used by the reference file
LOG2E = 1.4426950408889634


def _one_chunk(qf: np.ndarray, kvf: np.ndarray, idx: np.ndarray, sm_scale: float):
    valid = idx >= 0                                   # [t, K]
    rows = np.maximum(idx, 0).astype(np.int64)
    gathered = kvf[rows]                               # [t, K, D]
    s = np.matmul(qf, gathered.transpose(0, 2, 1)) * np.float32(sm_scale)   # [t, H, K]
    s = np.where(valid[:, None, :], s, np.float32(-np.inf))
    m = s.max(axis=-1)                                 # [t, H]
    m_safe = np.where(np.isfinite(m), m, np.float32(0.0)).astype(np.float32)
    with np.errstate(invalid="ignore", over="ignore"):
        p = np.exp(s - m_safe[..., None])
    p = np.where(valid[:, None, :], p, np.float32(0.0)).astype(np.float32)
    sumexp = p.sum(axis=-1, dtype=np.float32)          # [t, H]
    out = np.matmul(p, gathered)                       # [t, H, D]
    safe = sumexp > 0
    out = np.where(safe[..., None], out / np.maximum(sumexp, np.float32(1e-30))[..., None],
                   np.float32(0.0)).astype(np.float32)
    return out, m_safe, sumexp, safe


def sparse_mla_stats(q, kv, indices, sm_scale, chunk: int = 8):
    """Returns (out [T,H,D], m_safe [T,H], sumexp [T,H]) in float32.

    q, kv: float arrays holding the bf16 (or dequantised fp8) values; indices:
    integer [T, K]. ``m_safe`` is the max scaled score (0 on a fully masked row).
    """
    qf = np.ascontiguousarray(q, dtype=np.float32)
    kvf = np.ascontiguousarray(kv, dtype=np.float32)
    idx = np.asarray(indices)
    T, H, D = qf.shape
    assert kvf.shape[1] == D and idx.shape[0] == T
    outs, ms, ss = [], [], []
    step = chunk if chunk else max(T, 1)
    for i in range(0, T, step):
        o, m, s, _ = _one_chunk(qf[i:i + step], kvf, idx[i:i + step], sm_scale)
        outs.append(o)
        ms.append(m)
        ss.append(s)
    if not outs:
        z = np.zeros((0, H), np.float32)
        return np.zeros((0, H, D), np.float32), z, z
    return np.concatenate(outs), np.concatenate(ms), np.concatenate(ss)


def lse_reference(m_safe, sumexp, sm_scale):
    """The reference file's LSE formula (tests/reference.py:71-73), verbatim in meaning."""
    safe = sumexp > 0
    with np.errstate(divide="ignore"):
        v = np.log2(np.maximum(sumexp, np.float32(1e-30))) + m_safe * np.float32(sm_scale * LOG2E_REF)
    return np.where(safe, v, np.float32(-np.inf)).astype(np.float32)


def lse_log2(m_safe, sumexp):
    """log2-space log-sum-exp of the scaled scores; -inf on a fully masked row."""
    safe = sumexp > 0
    with np.errstate(divide="ignore"):
        v = np.log2(np.maximum(sumexp, np.float32(1e-30))) + m_safe * np.float32(LOG2E)
    return np.where(safe, v, np.float32(-np.inf)).astype(np.float32)


def sparse_mla_fp32(q, kv, indices, sm_scale, chunk: int = 8):
    """Same contract as the reference's sparse_mla_fp32: returns (out, lse)."""
    out, m, s = sparse_mla_stats(q, kv, indices, sm_scale, chunk)
    return out, lse_reference(m, s, sm_scale)


# ---------------------------------------------------------------------------
# bf16 / fp8 value helpers (numpy has neither type)
# ---------------------------------------------------------------------------
def bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns (uint16), round to nearest even."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounded = u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))
    return (rounded >> np.uint32(16)).astype(np.uint16)


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    return bf16_to_f32(bf16_bits(x))


def e4m3_to_f32(bits: np.ndarray) -> np.ndarray:
    """float8_e4m3fn bit patterns (uint8) -> float32 (exact)."""
    b = np.asarray(bits, dtype=np.uint8).astype(np.int32)
    sign = np.where(b & 0x80, -1.0, 1.0)
    exp = (b >> 3) & 0xF
    man = b & 0x7
    normal = sign * (1.0 + man / 8.0) * np.exp2(exp - 7.0)
    sub = sign * (man / 8.0) * np.exp2(-6.0)
    v = np.where(exp == 0, sub, normal)
    v = np.where((exp == 0xF) & (man == 0x7), np.nan, v)
    return v.astype(np.float32)


def dequant_fp8(bits: np.ndarray, scale: float) -> np.ndarray:
    """bf16(float(e4m3) * scale), the value the kernel places in shared memory."""
    return bf16_round(e4m3_to_f32(bits) * np.float32(scale))


def convert_req_index_to_global(req_id, block_table, token_indices, block_size: int,
                                block_stride_rows: int | None = None):
    """Request-local top-k positions -> physical cache slots.

    Restates the index converter the reference's backend calls before the op
    (glm53_sparse_mla/backend.py:371-378 of the reference): vLLM 0.22.0's
    ``triton_convert_req_index_to_global_index`` without a prefill workspace
    (vllm/v1/attention/backends/mla/sparse_utils.py:11-84). vLLM is a
    dependency of the reference, not part of it; this restates its published
    rule:

        out[t, k] = block_table[req_id[t], pos // block_size] * block_stride
                    + pos % block_size,        pos = token_indices[t, k]

    and -1 where pos < 0 or pos // block_size is not a valid block column
    (0 <= block < block_table.shape[1]). ``block_stride_rows`` defaults to
    ``block_size`` (contiguous pages), the only form that converter emits.
    """
    req_id = np.asarray(req_id, dtype=np.int64)
    bt = np.asarray(block_table, dtype=np.int64)
    pos = np.asarray(token_indices, dtype=np.int64)
    stride = block_size if block_stride_rows is None else block_stride_rows
    blk = np.floor_divide(pos, block_size)
    off = pos - blk * block_size
    ok = (pos >= 0) & (blk >= 0) & (blk < bt.shape[1])
    rows = bt[req_id[:, None], np.where(ok, blk, 0)]
    out = np.where(ok, rows * stride + off, -1)
    return out.astype(np.int32)
