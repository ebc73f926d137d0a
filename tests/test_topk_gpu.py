"""The indexer's per-row top-k on a B200 (glm53_sparse_mla.top_k_per_row_decode
/ top_k_per_row_prefill, C ABI glm53_topk_per_row).

* every row checked by the oracle's row checker (oracle/topk_oracle.py): short
  rows give 0..len-1 then -1; longer rows give distinct in-range positions
  whose values are exactly the multiset of the k largest; decode with
  next_n 1, 2 and 4 (1-D seq_lens) and per-row lengths (2-D seq_lens), prefill
  with row offsets, k = 512, 1024 and 2048, rows kept in shared memory and
  rows too long for it, padded row strides, heavy ties, -inf and NaN;
* against vLLM's compiled top_k_per_row_decode / top_k_per_row_prefill on
  the same inputs (same multiset of selected values per row), when vLLM's
  compiled ops load;
* indexer -> attention: the positions it writes feed sparse_fwd_paged.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import topk_oracle as TK

pytestmark = pytest.mark.gpu

import glm53_sparse_mla as G  # noqa: E402

DEV = torch.device("cuda")


def _check(out, logits, starts, ends, k):
    o = out.cpu().numpy()
    lg = logits.cpu().numpy()
    for r in range(len(ends)):
        why = TK.check_row(o[r, :k], lg[r], int(starts[r]), int(ends[r]), k)
        assert why is None, (r, why, int(ends[r]) - int(starts[r]))


def _logits(rows, width, seed, kind="normal", stride=None):
    g = torch.Generator(device="cpu").manual_seed(seed)
    stride = stride or width
    x = torch.randn((rows, stride), generator=g)
    if kind == "ties":
        x = torch.round(x * 4) / 4                   # a few dozen distinct values
    elif kind == "special":
        x[:, ::7] = float("-inf")
        x[::3, 5] = float("nan")
        x[1::3, 11] = float("inf")
    elif kind == "heavy":
        # every 15th value positive, the rest exactly 0: for rows longer than
        # about 15k the k-th largest is a 0 shared by more keys than the
        # candidate buffer holds
        x = torch.zeros((rows, stride))
        x[:, ::15] = torch.randn((rows, (stride + 14) // 15), generator=g).abs() + 1.0
    return x.to(DEV)


@pytest.mark.parametrize("k", [512, 1024, 2048])
@pytest.mark.parametrize("next_n", [1, 2, 4])
def test_decode_rows(k, next_n):
    B, width = 24, 12000
    rng = np.random.default_rng(k + next_n)
    seq = rng.integers(next_n, width, B).astype(np.int32)
    seq[0] = k // 2 + next_n          # short rows
    seq[1] = k + next_n               # exactly k (last row of this batch entry)
    seq[2] = width                    # full width
    rows = B * next_n
    logits = _logits(rows, width, seed=k * 7 + next_n, stride=width + 64)
    out = torch.full((rows, k + 5), -9, dtype=torch.int32, device=DEV)
    G.top_k_per_row_decode(logits, next_n, torch.from_numpy(seq).to(DEV), out, rows,
                           logits.stride(0), 1, k)
    torch.cuda.synchronize()
    ends = TK.decode_row_ends(seq, next_n, rows)
    _check(out, logits, np.zeros_like(ends), ends, k)
    assert bool((out[:, k:] == -9).all())               # columns past k untouched


def test_decode_per_row_lengths_2d():
    B, next_n, width, k = 8, 3, 9000, 2048
    rng = np.random.default_rng(5)
    seq2 = np.sort(rng.integers(100, width, (B, next_n)), axis=1).astype(np.int32)
    rows = B * next_n
    logits = _logits(rows, width, seed=11)
    out = torch.empty((rows, k), dtype=torch.int32, device=DEV)
    G.top_k_per_row_decode(logits, next_n, torch.from_numpy(seq2).to(DEV), out, rows,
                           logits.stride(0), 1, k)
    torch.cuda.synchronize()
    ends = seq2.reshape(-1).astype(np.int64)
    _check(out, logits, np.zeros_like(ends), ends, k)


@pytest.mark.parametrize("kind", ["normal", "ties", "special"])
def test_prefill_rows(kind):
    rows, width, k = 300, 20000, 2048
    rng = np.random.default_rng(len(kind))
    starts = rng.integers(0, 8000, rows).astype(np.int32)
    ends = (starts + rng.integers(1, 12000, rows)).astype(np.int32)
    logits = _logits(rows, width, seed=3, kind=kind)
    out = torch.empty((rows, k), dtype=torch.int32, device=DEV)
    G.top_k_per_row_prefill(logits, torch.from_numpy(starts).to(DEV), torch.from_numpy(ends).to(DEV),
                            out, rows, logits.stride(0), 1, k)
    torch.cuda.synchronize()
    _check(out, logits, starts, ends, k)


@pytest.mark.parametrize("kind", ["normal", "ties", "special", "heavy"])
@pytest.mark.parametrize("rows,width", [(32, 20000), (60, 40000), (5, 131072)])
def test_cluster_rows(rows, width, kind):
    """Batches small enough for a cluster of CTAs per row (on a 148-SM part:
    4 CTAs per row at 32 and 5 rows, 2 at 60 rows), rows of 12K values and
    more: decode rows of ragged lengths (short ones, exactly k, k + 1, the
    full width), then prefill rows at unaligned offsets."""
    k = 2048
    rng = np.random.default_rng(rows * 7 + len(kind))
    seq = rng.integers(1, width + 1, rows).astype(np.int32)
    seq[0] = width
    seq[1] = k
    seq[2] = k + 1
    seq[3] = 100
    logits = _logits(rows, width, seed=rows + width, kind=kind)
    out = torch.full((rows, k), -9, dtype=torch.int32, device=DEV)
    G.top_k_per_row_decode(logits, 1, torch.from_numpy(seq).to(DEV), out, rows, logits.stride(0), 1, k)
    torch.cuda.synchronize()
    _check(out, logits, np.zeros(rows, np.int64), seq.astype(np.int64), k)

    starts = rng.integers(0, width // 3, rows).astype(np.int32)
    starts[0] = 0
    ends = np.minimum(starts.astype(np.int64) + rng.integers(1, width, rows), width).astype(np.int32)
    ends[0] = width
    out = torch.full((rows, k), -9, dtype=torch.int32, device=DEV)
    G.top_k_per_row_prefill(logits, torch.from_numpy(starts).to(DEV), torch.from_numpy(ends).to(DEV), out, rows,
                            logits.stride(0), 1, k)
    torch.cuda.synchronize()
    _check(out, logits, starts, ends, k)


def test_rows_longer_than_shared_memory():
    rows, width, k = 6, 131072, 2048
    seq = np.array([131072, 100000, 49153, 49152, 3000, 2048], np.int32)
    logits = _logits(rows, width, seed=17, kind="ties")
    out = torch.empty((rows, k), dtype=torch.int32, device=DEV)
    G.top_k_per_row_decode(logits, 1, torch.from_numpy(seq).to(DEV), out, rows, width, 1, k)
    torch.cuda.synchronize()
    _check(out, logits, np.zeros(rows, np.int64), seq.astype(np.int64), k)


def _vllm_ops():
    try:
        from vllm import _custom_ops as ops
        torch.ops._C.top_k_per_row_decode    # noqa: B018 - raises if the ops did not load
    except Exception as exc:   # vLLM's compiled ops are library code, optional here
        pytest.skip(f"vLLM top-k ops unavailable: {exc}")
    return ops


def _same_values(a, b, logits, k):
    lg = logits.cpu().numpy()
    a, b = a.cpu().numpy(), b.cpu().numpy()
    for r in range(a.shape[0]):
        ka = np.sort(TK.order_key(lg[r][a[r][a[r] >= 0]]))
        kb = np.sort(TK.order_key(lg[r][b[r][b[r] >= 0]]))
        assert np.array_equal(ka, kb), r
        assert (a[r] < 0).sum() == (b[r] < 0).sum(), r


@pytest.mark.parametrize("next_n", [1, 2])
def test_decode_matches_vllm_op(next_n):
    ops = _vllm_ops()
    B, width, k = 32, 8192, 2048
    rng = np.random.default_rng(next_n)
    seq = torch.from_numpy(rng.integers(next_n, width, B).astype(np.int32)).to(DEV)
    rows = B * next_n
    for kind in ("normal", "ties"):
        logits = _logits(rows, width, seed=23, kind=kind)
        ours = torch.empty((rows, k), dtype=torch.int32, device=DEV)
        theirs = torch.empty_like(ours)
        G.top_k_per_row_decode(logits, next_n, seq, ours, rows, width, 1, k)
        ops.top_k_per_row_decode(logits, next_n, seq, theirs, rows, width, 1, k)
        torch.cuda.synchronize()
        _same_values(ours, theirs, logits, k)


def test_prefill_matches_vllm_op():
    ops = _vllm_ops()
    rows, width, k = 64, 16384, 2048
    rng = np.random.default_rng(9)
    ks = torch.from_numpy(rng.integers(0, 4000, rows).astype(np.int32)).to(DEV)
    ke = ks + torch.from_numpy(rng.integers(1, 12000, rows).astype(np.int32)).to(DEV)
    logits = _logits(rows, width, seed=29)
    ours = torch.empty((rows, k), dtype=torch.int32, device=DEV)
    theirs = torch.empty_like(ours)
    G.top_k_per_row_prefill(logits, ks, ke, ours, rows, width, 1, k)
    ops.top_k_per_row_prefill(logits, ks, ke, theirs, rows, width, 1, k)
    torch.cuda.synchronize()
    _same_values(ours, theirs, logits, k)


def test_indexer_to_attention():
    """Decode step: top-k positions from logits, straight into the paged
    attention op (no conversion), equal to feeding the oracle's positions."""
    B, H, k, bs, ctx = 8, 64, 2048, 64, 6000
    rng = np.random.default_rng(31)
    seq = torch.full((B,), ctx, dtype=torch.int32, device=DEV)
    logits = _logits(B, 8192, seed=37)
    pos = torch.empty((B, k), dtype=torch.int32, device=DEV)
    G.top_k_per_row_decode(logits, 1, seq, pos, B, 8192, 1, k)
    blocks = (ctx + bs - 1) // bs
    bt = torch.from_numpy(np.stack([rng.permutation(B * blocks)[:blocks] for _ in range(B)])
                          .astype(np.int32)).to(DEV)
    req = torch.arange(B, dtype=torch.int32, device=DEV)
    kv = torch.randn((B * blocks * bs, 512), device=DEV).to(torch.bfloat16)
    q = torch.randn((B, H, 512), device=DEV).to(torch.bfloat16)
    out = G.sparse_fwd_paged(q, kv, pos, req, bt, bs, 512 ** -0.5)
    want_pos = torch.from_numpy(TK.topk_rows(logits.cpu().numpy(), np.zeros(B, np.int64),
                                             np.full(B, ctx), k)).to(DEV)
    # the same position sets in another order: the same attention up to
    # summation order
    ref = G.sparse_fwd_paged(q, kv, want_pos, req, bt, bs, 512 ** -0.5)
    torch.cuda.synchronize()
    assert torch.equal(torch.sort(pos, 1).values, torch.sort(want_pos, 1).values)
    torch.testing.assert_close(out.float(), ref.float(), rtol=2e-2, atol=2e-3)
