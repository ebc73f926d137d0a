"""The indexer's per-row top-k without a GPU.

* the oracle (oracle/topk_oracle.py) against vLLM's torch restatement of its
  top-k ops, ``_topk_indices_torch`` (vllm 0.22.0
  vllm/v1/attention/ops/rocm_aiter_mla_sparse.py:572-600), on rows masked to
  -inf outside their range as vLLM's torch logits are: decode (next_n 1, 2, 4)
  and prefill (row starts and ends), rows shorter and longer than k;
* the oracle's key order (IEEE with +NaN on top) and its row checker;
* glm53_topk_per_row validates its arguments before any CUDA call;
* the torch ops carry vLLM's schemas and have fake kernels.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import topk_oracle as TK

import glm53_sparse_mla as G  # noqa: E402

OK, E_RANK, E_TOPK, E_ALIGN = 0, 1, 4, 6


def _vllm_topk():
    try:
        from vllm.v1.attention.ops.rocm_aiter_mla_sparse import _topk_indices_torch
    except Exception as exc:   # pragma: no cover - vLLM is in this image
        pytest.skip(f"vLLM torch top-k restatement unavailable: {exc}")
    return _topk_indices_torch


def _masked(rng, rows, width, starts, ends):
    x = rng.standard_normal((rows, width)).astype(np.float32)
    col = np.arange(width)
    mask = (col[None, :] < np.asarray(starts)[:, None]) | (col[None, :] >= np.asarray(ends)[:, None])
    return np.where(mask, np.float32(-np.inf), x)


@pytest.mark.parametrize("next_n", [1, 2, 4])
@pytest.mark.parametrize("k", [16, 64])
def test_decode_matches_vllm_restatement(next_n, k):
    topk_torch = _vllm_topk()
    rng = np.random.default_rng(next_n * 100 + k)
    B, width = 6, 300
    seq = rng.integers(1, width, B).astype(np.int32)
    seq[0] = k // 2 + next_n       # a short row
    ends = TK.decode_row_ends(seq, next_n, B * next_n)
    starts = np.zeros_like(ends)
    logits = _masked(rng, B * next_n, width, starts, ends)
    theirs = topk_torch(torch.from_numpy(logits), k).numpy()
    ours = TK.topk_rows(logits, starts, ends, k)
    for r in range(B * next_n):
        assert set(theirs[r][theirs[r] >= 0]) == set(ours[r][ours[r] >= 0]), r
        assert TK.check_row(ours[r], logits[r], 0, ends[r], k) is None


def test_prefill_matches_vllm_restatement():
    topk_torch = _vllm_topk()
    rng = np.random.default_rng(3)
    rows, width, k = 40, 500, 32
    starts = rng.integers(0, 200, rows).astype(np.int32)
    ends = (starts + rng.integers(1, 300, rows)).astype(np.int32)
    logits = _masked(rng, rows, width, starts, ends)
    theirs = topk_torch(torch.from_numpy(logits), k, row_starts=torch.from_numpy(starts)).numpy()
    ours = TK.topk_rows(logits, starts, ends, k)
    for r in range(rows):
        assert set(theirs[r][theirs[r] >= 0]) == set(ours[r][ours[r] >= 0]), r
        assert TK.check_row(ours[r], logits[r], starts[r], ends[r], k) is None


def test_key_order_and_checker():
    v = np.array([-np.inf, -1e30, -1.0, -0.0, 0.0, 1e-40, 1.0, np.inf, np.nan], np.float32)
    keys = TK.order_key(v)
    assert np.all(np.diff(keys.astype(np.int64)) > 0)
    row = np.array([3, 1, 4, 1, 5, 9, 2, 6], np.float32)
    assert TK.check_row(np.array([5, 7, 4]), row, 0, 8, 3) is None
    assert TK.check_row(np.array([5, 7, 2]), row, 0, 8, 3) is not None      # 4 < 5
    assert TK.check_row(np.array([5, 5, 7]), row, 0, 8, 3) is not None      # repeated
    assert TK.check_row(np.array([0, 1, -1, -1]), row, 0, 2, 4) is None     # short row
    ties = np.zeros(10, np.float32)
    assert TK.check_row(np.array([9, 3, 0]), ties, 0, 10, 3) is None        # any tie choice


@pytest.fixture(scope="module")
def lib():
    lib = ctypes.CDLL(G.library_path())
    lib.glm53_topk_per_row.argtypes = [
        ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
        ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
        ctypes.c_int, ctypes.c_void_p]
    return lib


def test_c_abi_validates_before_cuda(lib):
    f = lib.glm53_topk_per_row
    A = 0x10000
    # (logits, rows, stride0, stride1, seq_lens, next_n, starts, ends, out, out_stride, k, stream)
    assert f(A, 0, 4096, 1, A, 1, None, None, A, 2048, 2048, None) == OK      # no rows
    assert f(A, 4, 4096, 1, A, 1, None, None, A, 2048, 0, None) == E_TOPK
    assert f(A, 4, 4096, 1, A, 1, None, None, A, 20000, 20000, None) == E_TOPK
    assert f(A, 4, 4096, 2, A, 1, None, None, A, 2048, 2048, None) == E_RANK  # strided columns
    assert f(A, 4, 4096, 1, A, 1, A, A, A, 2048, 2048, None) == E_RANK        # both forms
    assert f(A, 4, 4096, 1, None, 1, A, None, A, 2048, 2048, None) == E_RANK  # prefill needs both
    assert f(A, 4, 4096, 1, A, 0, None, None, A, 2048, 2048, None) == E_RANK  # next_n 0
    assert f(A, 4, 4096, 1, A, 1, None, None, A, 1024, 2048, None) == E_RANK  # out too narrow
    assert f(A + 2, 4, 4096, 1, A, 1, None, None, A, 2048, 2048, None) == E_ALIGN


def test_op_schemas_and_fakes():
    d = str(torch.ops.glm53_sparse_mla.top_k_per_row_decode.default._schema)
    assert d == ("glm53_sparse_mla::top_k_per_row_decode(Tensor logits, int next_n, Tensor "
                 "seq_lens, Tensor(a!) raw_topk_indices, int num_rows, int stride0, int stride1, "
                 "int topk_tokens) -> ()")
    p = str(torch.ops.glm53_sparse_mla.top_k_per_row_prefill.default._schema)
    assert p == ("glm53_sparse_mla::top_k_per_row_prefill(Tensor logits, Tensor cu_seqlen_ks, "
                 "Tensor cu_seqlen_ke, Tensor(a!) raw_topk_indices, int num_rows, int stride0, "
                 "int stride1, int topk_tokens) -> ()")
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        lg = torch.empty((4, 64))
        out = torch.empty((4, 16), dtype=torch.int32)
        torch.ops.glm53_sparse_mla.top_k_per_row_decode(lg, 1, torch.empty(4, dtype=torch.int32),
                                                        out, 4, 64, 1, 16)
