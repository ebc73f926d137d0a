"""The indexer's paged fp8 MQA logits without a GPU.

* the oracle (oracle/indexer_logits_oracle.py) against vLLM's torch
  restatement ``fp8_paged_mqa_logits_torch`` (vllm 0.22.0
  vllm/v1/attention/ops/rocm_aiter_mla_sparse.py:256-356), next_n == 1, over
  context lengths from 1 to the full table and a block size of 64 and 16;
* rows of a next_n > 1 request equal next_n == 1 rows with the per-token
  visible length;
* glm53_indexer_logits validates its arguments before any CUDA call;
* the torch op has its schema and a fake kernel.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import indexer_logits_oracle as IL

import glm53_sparse_mla as G  # noqa: E402

OK, E_RANK, E_DIM, E_HEADS, E_ALIGN = 0, 1, 2, 3, 6


def make_case(rng, B, next_n, H, bs, nb, max_blocks):
    q = torch.from_numpy(rng.standard_normal((B, next_n, H, 128)).astype(np.float32)) \
        .to(torch.float8_e4m3fn)
    vals = torch.from_numpy(rng.standard_normal((nb, bs * 128)).astype(np.float32)) \
        .to(torch.float8_e4m3fn).view(torch.uint8)
    sc = torch.from_numpy(rng.uniform(0.25, 2.0, (nb, bs)).astype(np.float32)).view(torch.uint8)
    kv = torch.cat([vals, sc], 1).contiguous()                   # [nb, bs * 132]
    w = torch.from_numpy(rng.standard_normal((B * next_n, H)).astype(np.float32))
    bt = torch.from_numpy(np.stack([rng.permutation(nb)[:max_blocks] for _ in range(B)])
                          .astype(np.int32))
    return q, kv, w, bt


@pytest.mark.parametrize("bs", [64, 16])
def test_matches_vllm_restatement(bs):
    try:
        from vllm.v1.attention.ops.rocm_aiter_mla_sparse import fp8_paged_mqa_logits_torch
    except Exception as exc:   # pragma: no cover - vLLM is in this image
        pytest.skip(f"vLLM torch restatement unavailable: {exc}")
    rng = np.random.default_rng(bs)
    B, H, max_blocks = 5, 32, 12
    nb = B * max_blocks
    max_len = max_blocks * bs
    q, kv, w, bt = make_case(rng, B, 1, H, bs, nb, max_blocks)
    ctx = torch.tensor([1, bs - 1, bs + 3, max_len, max_len // 2], dtype=torch.int32)
    ref = fp8_paged_mqa_logits_torch(q, kv.view(nb, bs, 1, 132), w, ctx, bt, max_len).numpy()
    ours = IL.paged_mqa_logits(q.view(torch.uint8).numpy(), kv.numpy(), w.numpy(), ctx.numpy(),
                               bt.numpy(), max_len)
    fin = np.isfinite(ref)
    assert np.array_equal(fin, np.isfinite(ours))
    assert np.abs(ref[fin] - ours[fin]).max() <= 1e-5 * np.abs(ref[fin]).max()


def test_next_n_rows_are_per_token_rows():
    rng = np.random.default_rng(7)
    B, next_n, H, bs, max_blocks = 3, 4, 32, 64, 6
    q, kv, w, bt = make_case(rng, B, next_n, H, bs, B * max_blocks, max_blocks)
    ctx = np.array([7, 200, 384], np.int32)
    full = IL.paged_mqa_logits(q.view(torch.uint8).numpy(), kv.numpy(), w.numpy(), ctx, bt.numpy(),
                               384)
    lens = IL.row_lengths(ctx, next_n)
    for i in range(B):
        for j in range(next_n):
            one = IL.paged_mqa_logits(q.view(torch.uint8).numpy()[i:i + 1, j:j + 1], kv.numpy(),
                                      w.numpy()[i * next_n + j:i * next_n + j + 1],
                                      np.array([lens[i * next_n + j]]), bt.numpy()[i:i + 1], 384)
            assert np.array_equal(one[0], full[i * next_n + j])


@pytest.fixture(scope="module")
def lib():
    lib = ctypes.CDLL(G.library_path())
    lib.glm53_indexer_logits.argtypes = [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
        ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_int64, ctypes.c_int64,
        ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
        ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_void_p]
    return lib


def test_c_abi_validates_before_cuda(lib):
    f = lib.glm53_indexer_logits
    A = 0x10000
    # (q, kv, w, ctx, per_token, bt, B, next_n, H, D, nb, bs, block_bytes, bt_stride,
    #  max_blocks, logits, logits_stride, max_model_len, clean, stream)
    good = [A, A, A, A, 0, A, 4, 1, 64, 128, 100, 64, 64 * 132, 16, 16, A, 1024, 1024, 1, None]

    def call(**kw):
        args = list(good)
        names = ["q", "kv", "w", "ctx", "pt", "bt", "B", "next_n", "H", "D", "nb", "bs", "bb",
                 "bts", "mb", "lg", "ls", "mml", "clean", "s"]
        for k, v in kw.items():
            args[names.index(k)] = v
        return f(*args)

    assert call(B=0) == OK
    assert call(D=64) == E_DIM
    assert call(H=48) == E_HEADS
    assert call(next_n=3) == E_HEADS
    assert call(bb=64 * 130) == E_RANK          # block smaller than its rows and scales
    assert call(bs=48, bb=48 * 132) == E_RANK   # block size not a power of two
    assert call(bs=8, bb=8 * 132 + 16) == E_RANK  # block size below 16
    assert call(bb=64 * 132 + 4) == E_RANK      # block stride not a multiple of 16
    assert call(ls=512) == E_RANK               # logits rows shorter than max_model_len
    assert call(bts=8) == E_RANK                # table stride below its width
    assert call(lg=None) == E_ALIGN
    assert call(q=A + 8) == E_ALIGN


def test_op_schema_and_fake():
    sch = str(torch.ops.glm53_sparse_mla.fp8_paged_mqa_logits.default._schema)
    assert sch == ("glm53_sparse_mla::fp8_paged_mqa_logits(Tensor q, Tensor kv_cache, Tensor "
                   "weights, Tensor context_lens, Tensor block_tables, int max_model_len, bool "
                   "clean_logits, Tensor(a!) logits) -> ()")
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        q = torch.empty((2, 1, 64, 128), dtype=torch.float8_e4m3fn)
        torch.ops.glm53_sparse_mla.fp8_paged_mqa_logits(
            q, torch.empty((4, 64, 1, 132), dtype=torch.uint8), torch.empty((2, 64)),
            torch.empty(2, dtype=torch.int32), torch.empty((2, 4), dtype=torch.int32), 256, True,
            torch.empty((2, 256)))
